"""KV-head-group sharding on CPU ranks (gloo, world size 2): sharded attention
plus all-gather and head interleave equals the unsharded result, for fp16 and
for one-byte pools; a rank that leaves before the collective is detected by
the others as an error."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _one_byte(q, k, v, fmt):
    """Pools quantised with one scale per full pool (every rank derives the
    same scales from the same seeded values)."""
    from oracle import oracle as O
    fmax = 127.0 if fmt == O.KV_INT8 else 448.0
    ks = float(np.abs(k.astype(np.float32)).max()) / fmax
    vs = float(np.abs(v.astype(np.float32)).max()) / fmax
    return (O.fp8_encode(k.astype(np.float32) / np.float32(ks), fmt),
            O.fp8_encode(v.astype(np.float32) / np.float32(vs), fmt), ks, vs)


def _sharded_rank(rank, world, port, result_dir, fmt=0):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    from xllms_b200 import sharding
    from xllms_b200 import workloads as W
    _init(rank, world, port)
    try:
        b = W.make_batch("shard", [1, 40, 300, 517], 16, 4, 64, "f16", 77)
        q, k, v = b.values_numpy()
        if fmt:  # one-byte pools: shard the codes, attend over the dequantised shard
            k8, v8, ksc, vsc = _one_byte(q, k, v, fmt)
            qs, ks, vs = sharding.shard_heads(q, k8, v8, b.num_kv_heads, world, rank)
            local = O.attention_fp8(qs, ks, vs, fmt, ksc, vsc, b.block_tables, b.seq_lens,
                                    b.num_kv_heads // world, b.scale)
        else:
            qs, ks, vs = sharding.shard_heads(q, k, v, b.num_kv_heads, world, rank)
            local = O.attention(qs, ks, vs, b.block_tables, b.seq_lens, b.num_kv_heads // world,
                                b.scale)
        g = sharding.gather_heads(torch.from_numpy(local))
        full = sharding.interleave_heads(g).numpy()
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", [0, 1, 3], ids=["fp16", "e4m3", "int8"])
def test_sharded_attention_equals_unsharded(tmp_path, fmt):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    from xllms_b200 import workloads as W
    world = 2
    mp.start_processes(_sharded_rank, args=(world, _free_port(), str(tmp_path), fmt),
                       nprocs=world, start_method="spawn", join=True)
    b = W.make_batch("shard", [1, 40, 300, 517], 16, 4, 64, "f16", 77)
    q, k, v = b.values_numpy()
    if fmt:
        k8, v8, ksc, vsc = _one_byte(q, k, v, fmt)
        ref = O.attention_fp8(q, k8, v8, fmt, ksc, vsc, b.block_tables, b.seq_lens,
                              b.num_kv_heads, b.scale)
    else:
        ref = O.attention(q, k, v, b.block_tables, b.seq_lens, b.num_kv_heads, b.scale)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(got, ref)  # same arithmetic per head, bit-identical


def _leaving_rank(rank, world, port, result_dir):
    import sys
    sys.path.insert(0, ROOT)
    from xllms_b200 import sharding
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # leaves between steps, with nothing in flight
        os._exit(0)
    out = torch.zeros(2, 3, 4)
    try:
        sharding.gather_heads(out)
        status = "no-error"
    except Exception as exc:  # the missing peer surfaces as an error, not a hang
        status = "error:" + type(exc).__name__
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_missing_rank_is_detected(tmp_path):
    world = 2
    ctx = mp.start_processes(_leaving_rank, args=(world, _free_port(), str(tmp_path)),
                             nprocs=world, start_method="spawn", join=False)
    deadline = 120
    while not ctx.join(timeout=deadline):
        pass
    status = (tmp_path / "rank0.txt").read_text()
    assert status.startswith("error:"), status
