"""Fused head gather (nxt_paged_attention_sharded) on one GPU.

Two ranks are emulated on one GPU: each rank's launch stores its heads into
both ranks' gather buffers. The end-of-step barrier waits for every rank's
signal; here those signals are set on the host before the launches, so no
launch ever waits on another launch on the same GPU. With one signal left
unset (a flag that nothing sets) the barrier's bounded wait must run out and
report NXT_PA_DEV_TIMEOUT, leaving the context usable."""
import ctypes

import numpy as np
import pytest

from _helpers import check_close
from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import sharding as S
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu

WORLD = 2


def _buffers(lib, B, H, D, es, world):
    half = B * H * D * es
    flags_off = (2 * half + 255) // 256 * 256
    bufs = []
    for _ in range(world):
        p = ctypes.c_void_p()
        h = (ctypes.c_char * _native.NXT_PA_IPC_HANDLE_BYTES)()
        assert lib.nxt_pa_peer_alloc(flags_off + 8 * world, ctypes.byref(p), h) == 0
        bufs.append(p.value)
    return bufs, half, flags_off


def _shards(bufs, flags_off, H, world):
    out = []
    for r in range(world):
        sh = S.NxtPaShard()
        sh.world_size, sh.rank, sh.total_heads, sh.head_offset = world, r, H, r * (H // world)
        for p in range(world):
            sh.peer_out[p] = bufs[p]
            sh.peer_flags[p] = bufs[p] + flags_off
        out.append(sh)
    return out


def _flags(ptr, world, dev):
    import torch
    return torch.as_tensor(S._DeviceArray(ptr, (world,), "<i8"), device=dev)


def _call(lib, sh, step, b, qs, ks, vs, bt, sl, status):
    return lib.nxt_paged_attention_sharded(
        ctypes.byref(sh), step, qs.data_ptr(), ks.data_ptr(), vs.data_ptr(), bt.data_ptr(),
        sl.data_ptr(), b.num_seqs, qs.shape[1], b.head_size, ks.shape[1], b.scale, b.max_blocks,
        16, 2, ks.shape[1] * 16 * b.head_size, 16 * b.head_size, b.num_blocks,
        status.data_ptr(), None)


def _setup(cuda):
    import torch
    b = W.make_batch("fg", [1, 700, 2100, 0, 5000, 16], 32, 8, 128, "f16", 81, value_std=0.5)
    q, k, v = b.values_numpy()
    ref = O.attention(q, k, v, b.block_tables, b.seq_lens, b.num_kv_heads, b.scale)
    bt, sl = b.tables_torch(cuda)
    ranks = []
    for r in range(WORLD):
        qs, ks, vs = S.shard_heads(q, k, v, b.num_kv_heads, WORLD, r)
        ranks.append(tuple(torch.from_numpy(x).to(cuda) for x in (qs, ks, vs)))
    return b, ref, bt, sl, ranks


def test_emulated_ranks_gather_into_every_buffer(cuda):
    import torch
    lib = _native.xpa()
    b, ref, bt, sl, ranks = _setup(cuda)
    bufs, half, flags_off = _buffers(lib, b.num_seqs, 32, 128, 2, WORLD)
    shards = _shards(bufs, flags_off, 32, WORLD)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for step in (1, 2, 3):
            for r in range(WORLD):
                _flags(bufs[r] + flags_off, WORLD, cuda).fill_(step)
            for r in range(WORLD):
                assert _call(lib, shards[r], step, b, *ranks[r], bt, sl, status) == 0
            torch.cuda.synchronize()
            for r in range(WORLD):
                view = torch.as_tensor(S._DeviceArray(bufs[r] + (step & 1) * half,
                                                      (b.num_seqs, 32, 128), "<f2"), device=cuda)
                check_close(view, ref, what=f"step {step} buffer {r}")
        assert int(status.item()) == 0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.nxt_pa_peer_free(p)


def test_missing_peer_signal_times_out(cuda):
    import torch
    lib = _native.xpa()
    b, ref, bt, sl, ranks = _setup(cuda)
    bufs, half, flags_off = _buffers(lib, b.num_seqs, 32, 128, 2, WORLD)
    shards = _shards(bufs, flags_off, 32, WORLD)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    prev = lib.nxt_paged_attention_set_wait_budget_ns(20_000_000)  # 20 ms
    try:
        # rank 1 never runs: its signal in rank 0's flag array stays unset
        assert _call(lib, shards[0], 1, b, *ranks[0], bt, sl, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) & _native.NXT_PA_DEV_TIMEOUT
    finally:
        lib.nxt_paged_attention_set_wait_budget_ns(prev)
    # the context is still usable: a complete step succeeds
    status.zero_()
    for r in range(WORLD):
        _flags(bufs[r] + flags_off, WORLD, cuda).fill_(2)
    for r in range(WORLD):
        assert _call(lib, shards[r], 2, b, *ranks[r], bt, sl, status) == 0
    torch.cuda.synchronize()
    view = torch.as_tensor(S._DeviceArray(bufs[0], (b.num_seqs, 32, 128), "<f2"), device=cuda)
    check_close(view, ref, what="after timeout")
    assert int(status.item()) == 0
    for p in bufs:
        lib.nxt_pa_peer_free(p)


@pytest.mark.parametrize("name,fmt,fmax", [("e4m3", O.FP8_E4M3, 448.0), ("int8", O.KV_INT8, 127.0)])
def test_emulated_ranks_one_byte_pools(cuda, name, fmt, fmax):
    """nxt_paged_attention_fp8_sharded: each emulated rank reads its heads'
    one-byte pools and stores fp16 rows into both ranks' gather buffers; the
    gathered output equals the oracle over the dequantised pools."""
    import torch
    lib = _native.xpa()
    b = W.make_batch("fg8", [1, 700, 2100, 0, 5000, 16], 32, 8, 128, "f16", 83, value_std=0.5)
    q, k, v = b.values_numpy()
    ks = float(np.abs(k.astype(np.float32)).max()) / fmax
    vs = float(np.abs(v.astype(np.float32)).max()) / fmax
    k8 = O.fp8_encode(k.astype(np.float32) / np.float32(ks), fmt)
    v8 = O.fp8_encode(v.astype(np.float32) / np.float32(vs), fmt)
    ref = O.attention_fp8(q, k8, v8, fmt, ks, vs, b.block_tables, b.seq_lens, b.num_kv_heads,
                          b.scale, f64=True)
    bt, sl = b.tables_torch(cuda)
    bufs, half, flags_off = _buffers(lib, b.num_seqs, 32, 128, 2, WORLD)
    shards = _shards(bufs, flags_off, 32, WORLD)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for r in range(WORLD):
            _flags(bufs[r] + flags_off, WORLD, cuda).fill_(1)
        for r in range(WORLD):
            qs, k8s, v8s = (torch.from_numpy(np.ascontiguousarray(x)).to(cuda) for x in
                            S.shard_heads(q, k8, v8, b.num_kv_heads, WORLD, r))
            rc = lib.nxt_paged_attention_fp8_sharded(
                ctypes.byref(shards[r]), 1, qs.data_ptr(), k8s.data_ptr(), v8s.data_ptr(),
                bt.data_ptr(), sl.data_ptr(), b.num_seqs, qs.shape[1], b.head_size,
                k8s.shape[1], b.scale, b.max_blocks, 16, fmt, ks, vs,
                k8s.shape[1] * 16 * b.head_size, 16 * b.head_size, b.num_blocks,
                status.data_ptr(), None)
            assert rc == 0
            torch.cuda.synchronize()
        for r in range(WORLD):
            view = torch.as_tensor(S._DeviceArray(bufs[r] + half, (b.num_seqs, 32, 128), "<f2"),
                                   device=cuda)
            check_close(view, ref, what=f"{name} buffer {r}")
        assert int(status.item()) == 0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.nxt_pa_peer_free(p)


def test_fused_head_gather_class_one_rank(cuda):
    """FusedHeadGather (the class bench.py drives at N > 1) with one rank:
    fp16 pools, then fp8 pools through run(kv_format=...), each equal to the
    oracle, and a batch larger than its buffers refused on the host."""
    import torch
    b = W.make_batch("fgc", [1, 700, 2100, 0, 5000, 16], 32, 8, 128, "f16", 84, value_std=0.5)
    q, k, v = b.values_numpy()
    bt, sl = b.tables_torch(cuda)
    qt, kt, vt = (torch.from_numpy(x).to(cuda) for x in (q, k, v))
    fg = S.FusedHeadGather(b.num_seqs, 32, 128, 2, 1, 0, lambda blob: [blob], cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        out = fg.run(qt, kt, vt, bt, sl, b.scale, b.num_blocks, device_status=status)
        torch.cuda.synchronize()
        check_close(out, O.attention(q, k, v, b.block_tables, b.seq_lens, 8, b.scale),
                    what="fp16 pools")
        ks = float(np.abs(k.astype(np.float32)).max()) / 448.0
        vs = float(np.abs(v.astype(np.float32)).max()) / 448.0
        k8 = O.fp8_encode(k.astype(np.float32) / np.float32(ks), O.FP8_E4M3)
        v8 = O.fp8_encode(v.astype(np.float32) / np.float32(vs), O.FP8_E4M3)
        out = fg.run(qt, torch.from_numpy(k8).to(cuda), torch.from_numpy(v8).to(cuda), bt, sl,
                     b.scale, b.num_blocks, device_status=status, kv_format="e4m3",
                     k_scale=ks, v_scale=vs)
        torch.cuda.synchronize()
        check_close(out, O.attention_fp8(q, k8, v8, O.FP8_E4M3, ks, vs, b.block_tables,
                                         b.seq_lens, 8, b.scale, f64=True), what="fp8 pools")
        assert int(status.item()) == 0
        with pytest.raises(ValueError):
            fg.run(torch.cat([qt, qt]), kt, vt, torch.cat([bt, bt]), torch.cat([sl, sl]),
                   b.scale, b.num_blocks)
    finally:
        fg.close()


@pytest.mark.parametrize("world", [2, 8])
def test_config5_shape_emulated_ranks(cuda, world):
    """BASELINE config 5 at full size (B = 512, 64 query / 8 KV heads, D 128,
    fp16, context U[4096, 16384]) with `world` ranks emulated on one GPU, as
    at 2 and 8 GPUs: each rank's own pool and block tables (its KV heads),
    its launch storing into every rank's [512, 64, 128] gather buffer. A
    sample of sequences of each rank's heads is checked against the fp64
    oracle over that rank's pools, and every buffer must equal every other
    bit for bit, so every head of every buffer is covered. Ranks run one
    after another (their signals set on the host), holding one rank's
    pools at a time."""
    import torch
    from _helpers import gather_subset
    lib = _native.xpa()
    H, D = 64, 128
    bufs, half, flags_off = _buffers(lib, 512, H, D, 2, world)
    shards = _shards(bufs, flags_off, H, world)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    seqs = [0, 170, 341, 511]
    try:
        for r in range(world):
            _flags(bufs[r] + flags_off, world, cuda).fill_(1)
        for r in range(world):
            b = W.config5(world_size=world, rank=r)
            assert b.num_seqs == 512 and b.num_heads == H // world
            q, k, v = b.values_torch(cuda)
            bt, sl = b.tables_torch(cuda)
            assert _call(lib, shards[r], 1, b, q, k, v, bt, sl, status) == 0
            torch.cuda.synchronize()
            qs, ks, vs, bts, sls = gather_subset(b, seqs, q, k, v)
            ref = O.attention(qs, ks, vs, bts, sls, b.num_kv_heads, b.scale, f64=True)
            view = torch.as_tensor(S._DeviceArray(bufs[0] + half, (512, H, D), "<f2"),
                                   device=cuda)
            h0 = r * b.num_heads
            check_close(view[seqs][:, h0:h0 + b.num_heads], ref, what=f"rank {r} of {world}")
            del q, k, v
        first = torch.as_tensor(S._DeviceArray(bufs[0] + half, (512, H, D), "<i2"), device=cuda)
        for r in range(1, world):
            other = torch.as_tensor(S._DeviceArray(bufs[r] + half, (512, H, D), "<i2"),
                                    device=cuda)
            assert torch.equal(first, other), f"buffer {r} differs from buffer 0"
        assert int(status.item()) == 0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.nxt_pa_peer_free(p)
