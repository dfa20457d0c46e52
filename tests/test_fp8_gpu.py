"""One-byte KV cache on the GPU: attention over fp8 E4M3 / E5M2 and int8 pools equals the
oracle over the dequantised pools (fp64 oracle), and
the quantising append is bit-exact against the oracle's encoder."""
import numpy as np
import pytest

from _helpers import check_close
from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu

FMTS = [("e4m3", O.FP8_E4M3, 448.0), ("e5m2", O.FP8_E5M2, 57344.0), ("int8", O.KV_INT8, 127.0)]
EDGE_LENS = [0, 1, 15, 16, 17, 511, 512, 513, 1000]


def _quantised(b, fmt, fmax):
    q, k, v = b.values_numpy()
    ks = float(np.abs(k.astype(np.float32)).max()) / fmax
    vs = float(np.abs(v.astype(np.float32)).max()) / fmax
    k8 = O.fp8_encode(k.astype(np.float32) / np.float32(ks), fmt)
    v8 = O.fp8_encode(v.astype(np.float32) / np.float32(vs), fmt)
    return q, k8, v8, ks, vs


def _run(cuda, b, name, fmt, fmax, num_blocks=None):
    import torch
    q, k8, v8, ks, vs = _quantised(b, fmt, fmax)
    ref = O.attention_fp8(q, k8, v8, fmt, ks, vs, b.block_tables, b.seq_lens, b.num_kv_heads,
                          b.scale, block_size=b.block_size,
                          num_blocks=-1 if num_blocks is None else num_blocks, f64=True)
    bt, sl = b.tables_torch(cuda)
    out = PA.paged_attention_fp8(torch.from_numpy(q).to(cuda), torch.from_numpy(k8).to(cuda),
                                 torch.from_numpy(v8).to(cuda), bt, sl, name, ks, vs,
                                 scale=b.scale, num_blocks=num_blocks)
    torch.cuda.synchronize()
    return out, ref


@pytest.mark.parametrize("name,fmt,fmax", FMTS)
@pytest.mark.parametrize("head_size", [64, 128, 256])
@pytest.mark.parametrize("group", [1, 4, 8, 16])
def test_fp8_attention(cuda, name, fmt, fmax, head_size, group):
    if head_size == 256 and group > 8:
        pytest.skip("D = 256 takes at most 8 heads per KV head on the fast path; covered below")
    b = W.make_batch("f8", EDGE_LENS, 2 * group, 2, head_size, "f16", 300 + group, value_std=0.5)
    out, ref = _run(cuda, b, name, fmt, fmax)
    check_close(out, ref, what=f"{name} D={head_size} GS={group}")
    assert PA.device_status() == 0


@pytest.mark.parametrize("name,fmt,fmax", FMTS)
def test_fp8_split_context_and_long(cuda, name, fmt, fmax):
    b = W.make_batch("f8s", [20000, 3, 4097, 131], 16, 2, 128, "f16", 321, value_std=1.0)
    out, ref = _run(cuda, b, name, fmt, fmax)
    check_close(out, ref, what=f"{name} split")


@pytest.mark.parametrize("name,fmt,fmax", [FMTS[0], FMTS[2]])
def test_fp8_d256_group16_generic(cuda, name, fmt, fmax):
    b = W.make_batch("f8g", [300, 17], 32, 2, 256, "f16", 322)
    out, ref = _run(cuda, b, name, fmt, fmax)
    check_close(out, ref, what=f"{name} D=256 GS=16")


@pytest.mark.parametrize("name,fmt,fmax", [FMTS[1], FMTS[2]])
def test_fp8_other_page_size(cuda, name, fmt, fmax):
    b = W.make_batch("f8p", [1, 31, 32, 33, 700], 8, 2, 128, "f16", 323, block_size=32)
    out, ref = _run(cuda, b, name, fmt, fmax)
    check_close(out, ref, what=f"{name} block_size 32")


@pytest.mark.parametrize("name,fmt,fmax", [FMTS[0], FMTS[2]])
def test_fp8_bad_pages_masked(cuda, name, fmt, fmax):
    b = W.make_batch("f8b", [200, 64, 90], 8, 2, 128, "f16", 324)
    b.block_tables = b.block_tables.copy()
    b.block_tables[0, 3] = -1
    b.block_tables[2, 1] = b.num_blocks + 5
    PA.device_status(clear=True)
    out, ref = _run(cuda, b, name, fmt, fmax, num_blocks=b.num_blocks)
    check_close(out, ref, what="bad pages")
    assert PA.device_status(clear=True) & _native.NXT_PA_DEV_BAD_PAGE


@pytest.mark.parametrize("name,fmt,fmax", FMTS)
@pytest.mark.parametrize("head_size", [128, 40])
def test_fp8_append_bit_exact(cuda, name, fmt, fmax, head_size):
    import torch
    rng = np.random.default_rng(head_size)
    T, Hkv, nb, bs = 37, 4, 16, 16
    key = (rng.standard_normal((T, Hkv, head_size)) * 3).astype(np.float16)
    value = (rng.standard_normal((T, Hkv, head_size)) * 0.2).astype(np.float16)
    key[0, 0, :4] = np.array([60000, -60000, 0, -0.0], dtype=np.float16)  # saturation, zeros
    slots = rng.permutation(nb * bs)[:T].astype(np.int64)
    slots[5] = -1  # skipped
    ks, vs = 0.05, 0.001
    kc = np.zeros((nb, Hkv, bs, head_size), dtype=np.uint8)
    vc = np.zeros_like(kc)
    kcd, vcd = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    PA.reshape_and_cache_fp8(torch.from_numpy(key).to(cuda), torch.from_numpy(value).to(cuda),
                             kcd, vcd, torch.from_numpy(slots).to(cuda), name, ks, vs)
    torch.cuda.synchronize()
    k8 = O.fp8_encode(key.astype(np.float32) / np.float32(ks), fmt)
    v8 = O.fp8_encode(value.astype(np.float32) / np.float32(vs), fmt)
    O.reshape_and_cache(k8, v8, kc, vc, slots, block_size=bs)
    assert np.array_equal(kcd.cpu().numpy(), kc)
    assert np.array_equal(vcd.cpu().numpy(), vc)


def test_fp8_caller_workspace(cuda):
    import torch
    b = W.make_batch("f8w", [5000, 3000, 40], 8, 2, 128, "f16", 325)
    q, k8, v8, ks, vs = _quantised(b, O.FP8_E4M3, 448.0)
    need = _native.xpa().nxt_paged_attention_fp8_workspace_size(
        b.num_seqs, b.num_heads, b.head_size, b.num_kv_heads, b.max_blocks, b.block_size)
    assert need > 0
    bt, sl = b.tables_torch(cuda)
    args = (torch.from_numpy(q).to(cuda), torch.from_numpy(k8).to(cuda),
            torch.from_numpy(v8).to(cuda), bt, sl, "e4m3", ks, vs)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    out = PA.paged_attention_fp8(*args, scale=b.scale, workspace=ws)
    ref = O.attention_fp8(q, k8, v8, O.FP8_E4M3, ks, vs, b.block_tables, b.seq_lens,
                          b.num_kv_heads, b.scale, f64=True)
    check_close(out, ref, what="fp8 caller workspace")
    with pytest.raises(PA.PagedAttentionError) as e:
        PA.paged_attention_fp8(*args, scale=b.scale, workspace=ws[:need - 1])
    assert e.value.code == _native.NXT_PA_EWORKSPACE


@pytest.mark.parametrize("name,fmt,fmax", FMTS)
@pytest.mark.parametrize("hq,d", [(32, 128), (16, 256), (8, 64)])
def test_fp8_append_fused_decode_step(cuda, name, fmt, fmax, hq, d):
    import torch
    # lengths include the new token; 17, 33 and 2049 put it at slot 0 of a new page
    lens = [1, 17, 33, 500, 2049, 5000]
    hkv = 2
    b = W.make_batch("f8ap", lens, hq, hkv, d, "f16", 62, value_std=0.5)
    q, k8, v8, ks, vs = _quantised(b, fmt, fmax)
    rng = np.random.default_rng(10)
    new_k = (rng.standard_normal((b.num_seqs, hkv, d)) * 0.5).astype(np.float16)
    new_v = (rng.standard_normal((b.num_seqs, hkv, d)) * 0.5).astype(np.float16)
    slots = np.array([int(b.block_tables[i, (L - 1) // 16]) * 16 + (L - 1) % 16
                      for i, L in enumerate(b.seq_lens)], dtype=np.int64)
    # reference: quantise and scatter on the host, then attention over the codes
    kr, vr = k8.copy(), v8.copy()
    O.reshape_and_cache(O.fp8_encode(new_k.astype(np.float32) / np.float32(ks), fmt),
                        O.fp8_encode(new_v.astype(np.float32) / np.float32(vs), fmt), kr, vr,
                        slots, block_size=b.block_size)
    ref = O.attention_fp8(q, kr, vr, fmt, ks, vs, b.block_tables, b.seq_lens, b.num_kv_heads,
                          b.scale, f64=True)
    kt, vt = torch.from_numpy(k8).to(cuda), torch.from_numpy(v8).to(cuda)
    bt, sl = b.tables_torch(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = PA.paged_attention_fp8_append(torch.from_numpy(q).to(cuda), kt, vt, bt, sl,
                                        torch.from_numpy(new_k).to(cuda),
                                        torch.from_numpy(new_v).to(cuda),
                                        torch.from_numpy(slots).to(cuda), name, ks, vs,
                                        scale=b.scale, device_status=status)
    torch.cuda.synchronize()
    check_close(out, ref, what=f"{name} fused append D={d}")
    assert np.array_equal(kt.cpu().numpy(), kr) and np.array_equal(vt.cpu().numpy(), vr)
    assert int(status.item()) == 0


@pytest.mark.parametrize("name,fmt,head_size", [("int8", O.KV_INT8, 128), ("int8", O.KV_INT8, 64),
                                                ("e4m3", O.FP8_E4M3, 128)])
def test_one_byte_index_logic_bit_exact(cuda, name, fmt, head_size):
    """Indexing over one-byte pools, exact: plant_hot_keys with scale 1 and
    cell integers the format holds exactly (int8: up to 127; E4M3: up to
    16). D = 128 takes the TMA path, D = 64 the CUDA-core one."""
    import torch
    from _helpers import assert_hot_cells, plant_hot_keys
    lens = [1, 15, 16, 17, 33, 511, 512, 513, 2000, 4097, 300, 64]
    b = W.make_batch("idx8", lens, 8, 2, head_size, "f16", 92)
    q, k, v = b.values_numpy()
    rng = np.random.default_rng(7)

    def pick(i, h, L):
        picks = [L - 1, 0, 15, 16, L // 2, int(rng.integers(0, L))]
        return min(picks[(2 * i + h) % len(picks)], L - 1)

    if fmt == O.KV_INT8:
        enc = lambda p, s, h: (p % 100 + 1, p // 100 + 1, s + 1, h + 1)
    else:
        enc = lambda p, s, h: (p % 16 + 1, (p // 16) % 16 + 1, s + 1, h + 1)
    expect = plant_hot_keys(b, q, k, v, pick, enc)
    k8 = O.fp8_encode(k.astype(np.float32), fmt)
    v8 = O.fp8_encode(v.astype(np.float32), fmt)
    assert np.array_equal(O.fp8_decode(v8, fmt), v.astype(np.float32))  # cells held exactly
    bt, sl = b.tables_torch(cuda)
    out = PA.paged_attention_fp8(torch.from_numpy(q).to(cuda), torch.from_numpy(k8).to(cuda),
                                 torch.from_numpy(v8).to(cuda), bt, sl, name, 1.0, 1.0,
                                 scale=b.scale, num_blocks=b.num_blocks)
    assert PA.device_status() == 0
    assert_hot_cells(out, expect)
