"""bench.py's output check on CPU tensors: the sampled-sequence comparison
with the oracle, and (gloo, two ranks) the cross-rank bitwise comparison of
the gathered buffers. A planted error in one element must fail the check on
every rank."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def _full_output(batch, q, k, v):
    """The oracle's output of this rank's heads (fp16), as the kernels would
    store it."""
    from oracle import oracle as O
    ref = O.attention(q, k, v, batch.block_tables, batch.seq_lens, batch.num_kv_heads,
                      batch.scale, f64=True)
    return torch.from_numpy(ref.astype(np.float16))


def test_parity_sample_covers_first_and_last():
    bench = _bench()
    assert bench.parity_sample(512) == [0, 170, 341, 511]
    assert bench.parity_sample(1) == [0]


def test_single_rank_check_passes_and_catches_a_planted_error():
    bench = _bench()
    from xllms_b200 import workloads as W
    b = W.make_batch("chk", [3, 700, 40, 2100, 16], 16, 4, 64, "f16", 31, value_std=0.5)
    q, k, v = b.values_numpy()
    full = _full_output(b, q, k, v)
    qt, kt, vt = (torch.from_numpy(x) for x in (q, k, v))
    ok, worst = bench.verify_output(b, qt, kt, vt, full, 0, 1, "cpu")
    assert ok and worst <= 1.0
    bad = full.clone()
    bad[bench.parity_sample(b.num_seqs)[1], 5, 7] += 0.25
    ok, worst = bench.verify_output(b, qt, kt, vt, bad, 0, 1, "cpu")
    assert not ok and worst > 1.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, plant, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        bench = _bench()
        from xllms_b200 import sharding
        from xllms_b200 import workloads as W
        b = W.make_batch("chk2", [5, 900, 33, 1500], 16, 4, 64, "f16", 41, value_std=0.5,
                         world_size=world, rank=rank)
        q, k, v = b.values_numpy()
        local = _full_output(b, q, k, v)                      # [B, Hq/P, D]
        full = sharding.interleave_heads(sharding.gather_heads(local))
        if plant and rank == 1:
            full[2, 0, 3] += 1.0  # rank 0's head in rank 1's buffer
        qt, kt, vt = (torch.from_numpy(x) for x in (q, k, v))
        ok, worst = bench.verify_output(b, qt, kt, vt, full.contiguous(), rank, world, "cpu")
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write(f"{int(ok)} {worst}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", [False, True])
def test_two_rank_check_over_gloo(tmp_path, plant):
    mp.spawn(_rank, args=(2, _free_port(), plant, str(tmp_path)), nprocs=2, join=True)
    res = [open(tmp_path / f"r{r}").read().split() for r in range(2)]
    oks = {int(x[0]) for x in res}
    assert oks == ({0} if plant else {1})
