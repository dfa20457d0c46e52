"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle."""
import numpy as np
import pytest

from _helpers import (RTOL, assert_hot_cells, check_close, gather_subset, oracle_out,
                      plant_hot_keys, to_device)
from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu

EDGE_LENS = [0, 1, 15, 16, 17, 511, 512, 513, 1000]


def _run_dropin(entry, batch, qt, kt, vt, bt, sl, out):
    getattr(PA, entry)(out, qt, kt, vt, bt, sl, batch.num_seqs, batch.num_heads,
                       batch.head_size, batch.num_kv_heads, batch.scale, batch.max_blocks,
                       batch.block_size, batch.dtype_size, batch.kv_block_stride,
                       batch.kv_head_stride, None)


@pytest.mark.parametrize("entry", ["nxt_paged_attention", "nxt_paged_attention_v2",
                                   "nxt_paged_attention_flash"])
def test_config1_dropin_entries(cuda, entry):
    import torch
    b = W.config1()
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = torch.full_like(qt, float("nan"))
    _run_dropin(entry, b, qt, kt, vt, bt, sl, out)
    torch.cuda.synchronize()
    check_close(out, ref, what=entry)
    assert PA.device_status() == 0


@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("head_size", [64, 128, 256])
def test_fp16_groups_and_heads(cuda, group, head_size):
    hkv = 2
    b = W.make_batch("g", EDGE_LENS, hkv * group, hkv, head_size, "f16", 100 + group,
                     value_std=0.5)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what=f"GS={group} D={head_size}")
    expect = _native.NXT_PA_PATH_TMA_MMA if not (group > 8 and head_size == 256) \
        else _native.NXT_PA_PATH_GENERIC
    assert PA.kernel_path(kt, vt, b.num_heads, head_size, hkv, 16, 2, b.kv_block_stride,
                          b.kv_head_stride) == expect
    assert PA.device_status() == 0


@pytest.mark.parametrize("head_size", [32, 64, 80, 96, 112, 128, 192, 256])
@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_all_reference_head_sizes(cuda, head_size, dtype):
    # The reference dispatches head sizes 32..256 (include/operator_api.h:40-41).
    b = W.make_batch("h", [5, 33, 300], 8, 4, head_size, dtype, 7 + head_size)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what=f"{dtype} D={head_size}")


@pytest.mark.parametrize("block_size", [8, 32])
def test_other_page_sizes(cuda, block_size):
    b = W.make_batch("p", [1, 31, 32, 33, 700], 8, 2, 128, "f16", 17, block_size=block_size)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what=f"block_size={block_size}")


@pytest.mark.parametrize("lens", [[4096], [20000, 3, 513], [131072 // 8] * 2])
def test_split_context(cuda, lens):
    b = W.make_batch("s", lens, 16, 2, 128, "f16", 23)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what=f"split {lens}")


@pytest.mark.parametrize("head_size", [33, 65, 127])
@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_odd_head_sizes_split_context(cuda, head_size, dtype):
    """Odd head size, odd query-head count and an odd partition count: the
    partial outputs then end on a 4-byte boundary, and the (max, sum) pairs the
    merge reads as 8-byte loads must still start aligned. Also through a
    caller workspace of exactly the size the query reports."""
    import torch
    b = W.make_batch("odd", [5000, 3, 2049], 3, 1, head_size, dtype, 61 + head_size)
    need = PA.workspace_size(b.num_seqs, b.num_heads, head_size, 1, b.max_blocks,
                             dtype_size=b.dtype_size)
    assert need > 0
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v, f64=True)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what=f"{dtype} D={head_size} library workspace")
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    out2 = PA.paged_attention(qt, kt, vt, bt, sl, workspace=ws)
    check_close(out2, ref, what=f"{dtype} D={head_size} caller workspace")
    with pytest.raises(PA.PagedAttentionError) as ei:
        PA.paged_attention(qt, kt, vt, bt, sl,
                           workspace=torch.empty(need + 16, dtype=torch.uint8, device=cuda)[4:])
    assert ei.value.code == _native.NXT_PA_EINVAL
    assert PA.device_status() == 0


def test_prefix_shared_tables(cuda):
    b = W.config4(num_seqs=16)
    assert b.kv_bytes_unique() < b.kv_bytes()
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what="prefix shared")


def test_zero_inputs_give_zero_output(cuda):
    # The one numerical result the reference's own tests pin:
    # all-zero inputs give an all-zero output (tests/test_attention_bench.c:387-389).
    import torch
    b = W.make_batch("z", [32], 4, 2, 64, "f16", 1)
    qt = torch.zeros((1, 4, 64), dtype=torch.float16, device=cuda)
    kt = torch.zeros((b.num_blocks, 2, 16, 64), dtype=torch.float16, device=cuda)
    bt, sl = b.tables_torch(cuda)
    out = PA.paged_attention(qt, kt, kt.clone(), bt, sl)
    assert float(out.abs().max()) < 1e-3


def test_uniform_weights_give_mean_of_values(cuda):
    # Q = 0 makes every weight 1/L: the output is the mean of the visited V rows.
    import torch
    b = W.make_batch("u", [1, 17, 100, 600], 8, 2, 128, "f16", 3)
    q, k, v = b.values_numpy()
    q[:] = 0
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl).float().cpu().numpy()
    vv = v.astype(np.float64)
    for i in range(b.num_seqs):
        L = int(b.seq_lens[i])
        rows = [vv[b.block_tables[i, t // 16], :, t % 16, :] for t in range(L)]
        mean = np.mean(rows, axis=0)  # [Hkv, D]
        expect = np.repeat(mean, 4, axis=0)
        assert np.allclose(out[i], expect, rtol=2e-3, atol=2e-3)


def test_single_hot_key_selects_its_value(cuda):
    import torch
    b = W.make_batch("hot", [300], 4, 1, 64, "f16", 9)
    q, k, v = b.values_numpy()
    k[:] = 0
    q[:] = 1
    hot = 123
    page, slot = b.block_tables[0, hot // 16], hot % 16
    k[page, 0, slot, :] = 2.0  # score 2*64*0.125 = 16 nats above the rest
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl).float().cpu().numpy()
    ref = oracle_out(b, q, k, v)
    check_close(out, ref, what="hot key")
    assert np.allclose(out[0, 0], v[page, 0, slot].astype(np.float32), atol=1e-3 * 8)


def test_masked_pages_and_status(cuda):
    import torch
    b = W.make_batch("m", [200, 64], 8, 2, 128, "f16", 31)
    b.block_tables[0, 3] = -1          # a hole inside sequence 0
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    PA.device_status(clear=True)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what="masked page")
    assert PA.device_status() & _native.NXT_PA_DEV_BAD_PAGE


def test_out_of_range_pages_masked_with_num_blocks(cuda):
    b = W.make_batch("r", [100, 90], 8, 2, 128, "f16", 37)
    q, k, v = b.values_numpy()
    limit = int(b.block_tables[0, 2])  # every page id >= limit is out of range
    ref = oracle_out(b, q, k, v, num_blocks=limit)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    PA.device_status(clear=True)
    out = PA.paged_attention(qt, kt, vt, bt, sl, num_blocks=limit)
    check_close(out, ref, what="num_blocks mask")
    assert PA.device_status() & _native.NXT_PA_DEV_BAD_PAGE


def test_seq_len_clamped_to_table(cuda):
    import torch
    b = W.make_batch("c", [64, 40], 4, 2, 64, "f16", 41, max_blocks=4)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    sl_long = sl.clone()
    sl_long[0] = 10_000                 # beyond max_blocks * block_size = 64
    PA.device_status(clear=True)
    out = PA.paged_attention(qt, kt, vt, bt, sl_long)
    check_close(out, ref, what="clamp")
    assert PA.device_status() & _native.NXT_PA_DEV_SEQ_CLAMPED


def test_nan_garbage_past_seq_len_is_ignored(cuda):
    import torch
    b = W.make_batch("n", [20, 5], 8, 2, 128, "f16", 43)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    for i in range(b.num_seqs):
        L = int(b.seq_lens[i])
        last = b.block_tables[i, (L - 1) // 16]
        k[last, :, L % 16:, :] = np.inf
        v[last, :, L % 16:, :] = np.nan
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    check_close(out, ref, what="garbage tail")


def test_caller_workspace_and_stream(cuda):
    import torch
    b = W.make_batch("w", [3000, 70], 8, 2, 128, "f16", 47)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    need = PA.workspace_size(b.num_seqs, b.num_heads, 128, 2, b.max_blocks)
    assert need > 0
    small = torch.empty(need // 2, dtype=torch.uint8, device=cuda)
    with pytest.raises(PA.PagedAttentionError) as ei:
        PA.paged_attention(qt, kt, vt, bt, sl, workspace=small)
    assert ei.value.code == _native.NXT_PA_EWORKSPACE
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = PA.paged_attention(qt, kt, vt, bt, sl, workspace=ws, device_status=status, stream=s)
    s.synchronize()
    check_close(out, ref, what="caller workspace")
    assert int(status.item()) == 0


def test_first_call_of_a_fresh_host_thread(cuda):
    """A host thread whose first CUDA call is the library's has no current
    context yet: the call must still take the TMA path (not fall back to the
    CUDA-core kernel) and give the same bits as any other thread."""
    import threading
    import torch
    b = W.make_batch("fresh", [3000, 70, 9000], 32, 8, 128, "f16", 59)
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    ref = PA.paged_attention(qt, kt, vt, bt, sl)
    out = torch.empty_like(ref)
    torch.cuda.synchronize()
    seen = {}

    def worker():
        try:
            seen["path"] = PA.kernel_path(kt, vt, 32, 128, 8, 16, 2, b.kv_block_stride,
                                          b.kv_head_stride)
            PA.paged_attention(qt, kt, vt, bt, sl, out=out, stream=2)  # cudaStreamPerThread
        except Exception as e:  # reported below, on the test's thread
            seen["error"] = e

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    torch.cuda.synchronize()
    assert "error" not in seen, seen
    assert seen["path"] == _native.NXT_PA_PATH_TMA_MMA
    assert torch.equal(out, ref)


def test_per_thread_default_streams_of_two_threads(cuda):
    """cudaStreamPerThread is one handle for every host thread but a separate
    stream in each: two threads calling at once on it must not share the
    library's split-context workspace, and each thread's first call (no
    current context yet) must take the same path as the rest."""
    import threading
    import torch
    per_thread = 2  # cudaStreamPerThread
    inputs, refs = [], []
    for i, lens in enumerate(([9000, 4100, 7000, 300], [5000, 8192, 2500, 6000])):
        b = W.make_batch(f"pt{i}", lens * 4, 32, 8, 128, "f16", 60 + i)
        q, k, v = b.values_numpy()
        x = to_device(b, q, k, v, cuda)
        inputs.append(x)
        refs.append(PA.paged_attention(*x))
    torch.cuda.synchronize()
    outs = [[], []]
    errors = []

    def worker(i):
        try:
            for _ in range(20):
                outs[i].append(PA.paged_attention(*inputs[i], stream=per_thread))
        except Exception as e:  # reported below, on the test's thread
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in (0, 1)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    for i in (0, 1):
        assert len(outs[i]) == 20
        for o in outs[i]:
            assert torch.equal(o, refs[i])
    assert PA.device_status() == 0


def test_repeatable_bitwise(cuda):
    b = W.make_batch("d", [777, 4000], 32, 8, 128, "f16", 53)
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    a = PA.paged_attention(qt, kt, vt, bt, sl)
    c = PA.paged_attention(qt, kt, vt, bt, sl)
    assert bool((a == c).all())


def test_invalid_arguments_launch_nothing(cuda):
    import torch
    b = W.make_batch("i", [16], 6, 4, 64, "f16", 1)  # 6 % 4 != 0 after construction
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = torch.zeros_like(qt)
    with pytest.raises(PA.PagedAttentionError) as ei:
        PA.nxt_paged_attention(out, qt, kt, vt, bt, sl, 1, 6, 64, 4, 0.125, 1, 16, 2,
                               4 * 16 * 64, 16 * 64)
    assert ei.value.code == _native.NXT_PA_EINVAL
    with pytest.raises(PA.PagedAttentionError):
        PA.nxt_paged_attention(out, qt, kt, vt, bt, sl, 1, 4, 64, 4, 0.125, 1, 16, 3,
                               4 * 16 * 64, 16 * 64)
    assert float(out.abs().max()) == 0.0


@pytest.mark.parametrize("cfg", ["c2", "c3", "c4"])
def test_full_size_configs_sampled(cuda, cfg):
    """Full BASELINE sizes on the device; a sample of sequences is re-checked
    by the oracle from the device's own pages."""
    import torch
    b = W.CONFIGS[cfg]()
    qt, kt, vt = b.values_torch(cuda)
    bt, sl = b.tables_torch(cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl)
    torch.cuda.synchronize()
    assert PA.device_status() == 0
    lens = b.seq_lens
    picks = {int(np.argmin(lens)), int(np.argmax(lens))}
    if cfg != "c3":
        picks |= {0, b.num_seqs - 1}
    picks = sorted(picks)
    q, k, v, sbt, ssl = gather_subset(b, picks, qt, kt, vt)
    ref = O.attention(q, k, v, sbt, ssl, b.num_kv_heads, b.scale, threads=0)
    check_close(out[picks], ref, what=cfg)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("head_size,dtype,group,block_size", [
    (128, "f16", 4, 16),   # TMA + tensor-core path, split partitions
    (256, "f16", 2, 16),   # TMA path, D = 256
    (128, "f16", 16, 16),  # TMA path, two 8-head tiles
    (64, "f32", 1, 16),    # CUDA-core path, fp32
    (128, "f16", 4, 32),   # CUDA-core path, 32-token pages
])
def test_index_logic_bit_exact(cuda, head_size, dtype, group, block_size):
    """Block-table, slot and head indexing, checked by exact equality: one
    hot key per (sequence, KV head), V rows encoding their own cell
    (plant_hot_keys). Hot positions cover page edges and split partitions."""
    lens = [1, 15, 16, 17, 33, 511, 512, 513, 2000, 4097, 300, 64]
    b = W.make_batch("idx", lens, group * 2, 2, head_size, dtype, 91, block_size=block_size)
    q, k, v = b.values_numpy()
    rng = np.random.default_rng(6)

    def pick(i, h, L):
        picks = [L - 1, 0, block_size - 1, block_size, L // 2, int(rng.integers(0, L))]
        return min(picks[(2 * i + h) % len(picks)], L - 1)

    expect = plant_hot_keys(b, q, k, v, pick,
                            lambda p, s, h: (p % 1024 + 1, p // 1024 + 1, s + 1, h + 1))
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention(qt, kt, vt, bt, sl, num_blocks=b.num_blocks)
    assert PA.device_status() == 0
    assert_hot_cells(out, expect)


def test_inputs_written_by_the_previous_kernel(cuda):
    """The first kernel of a call is launched as a programmatic dependent of
    whatever kernel precedes it on the stream and waits for it before reading
    anything: query, pools and tables written by kernels right before the call
    (no synchronisation in between) must be the ones the call sees."""
    import torch
    b = W.make_batch("prev", [3000, 17, 700, 1], 32, 8, 128, "f16", 57, value_std=0.5)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = torch.empty_like(qt)
    q_stale, k_stale = torch.zeros_like(qt), torch.zeros_like(kt)
    bt_stale, sl_stale = torch.zeros_like(bt), torch.zeros_like(sl)
    for _ in range(3):
        # kernels (not copies) overwrite every input just before the call
        q_stale.mul_(0).add_(qt)
        k_stale.mul_(0).add_(kt)
        bt_stale.mul_(0).add_(bt)
        sl_stale.mul_(0).add_(sl)
        PA.paged_attention(q_stale, k_stale, vt, bt_stale, sl_stale, out=out,
                           num_blocks=b.num_blocks)
        check_close(out, ref, what="inputs written by the preceding kernels")
        q_stale.zero_()
        k_stale.zero_()
        sl_stale.zero_()
    assert PA.device_status() == 0
