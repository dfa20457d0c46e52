"""KV-head-group sharding on CPU ranks (gloo, world size 2): sharded attention
plus all-gather and head interleave equals the unsharded result; a rank that
leaves before the collective is detected by the others as an error."""
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


def _sharded_rank(rank, world, port, result_dir):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    from xllms_b200 import sharding
    from xllms_b200 import workloads as W
    _init(rank, world, port)
    try:
        b = W.make_batch("shard", [1, 40, 300, 517], 16, 4, 64, "f16", 77)
        q, k, v = b.values_numpy()
        qs, ks, vs = sharding.shard_heads(q, k, v, b.num_kv_heads, world, rank)
        local = O.attention(qs, ks, vs, b.block_tables, b.seq_lens, b.num_kv_heads // world,
                            b.scale)
        g = sharding.gather_heads(torch.from_numpy(local))
        full = sharding.interleave_heads(g).numpy()
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), full)
    finally:
        dist.destroy_process_group()


def test_sharded_attention_equals_unsharded(tmp_path):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    from xllms_b200 import workloads as W
    world = 2
    mp.start_processes(_sharded_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    b = W.make_batch("shard", [1, 40, 300, 517], 16, 4, 64, "f16", 77)
    q, k, v = b.values_numpy()
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
