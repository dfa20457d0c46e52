"""Fused head gather across two GPUs: one process per GPU, IPC buffers
exchanged through torch.distributed, each rank's kernels store its heads into
both GPUs' buffers over NVLink and a bounded cross-GPU barrier ends each
step. Skipped unless two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir, multicast=False):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from xllms_b200 import sharding as S
    from xllms_b200 import workloads as W
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    worst = []
    try:
        b = W.make_batch("fg2", [1, 700, 2100, 0, 5000, 16, 3333], 32, 8, 128, "f16", 82,
                         value_std=0.5)
        q, k, v = b.values_numpy()
        ref = O.attention(q, k, v, b.block_tables, b.seq_lens, b.num_kv_heads, b.scale)
        qs, ks, vs = (torch.from_numpy(x).to(dev) for x in
                      S.shard_heads(q, k, v, b.num_kv_heads, world, rank))
        bt, sl = b.tables_torch(dev)
        fg = S.FusedHeadGather(b.num_seqs, 32, 128, 2, world, rank, S.torch_exchange(), dev,
                               multicast=multicast)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(4):
            out = fg.run(qs, ks, vs, bt, sl, b.scale, b.num_blocks, device_status=status)
            torch.cuda.synchronize()
            ok, w = O.rel_err_ok(out.float().cpu().numpy(), ref, 1e-3)
            worst.append(w if ok else float("inf"))
        worst.append(float(status.item()))
        fg.close(dist.barrier)
    finally:
        dist.destroy_process_group()
    np.save(os.path.join(outdir, f"rank{rank}.npy"), np.array(worst))


@pytest.mark.parametrize("multicast", [False, True], ids=["peer_stores", "multimem"])
def test_two_gpu_fused_gather(tmp_path, multicast):
    """peer_stores: IPC buffers, one store per peer. multimem: buffers from
    torch symmetric memory, one multimem store per row chunk when the GPUs
    support multicast (peer stores into the same buffers otherwise)."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path), multicast), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        res = np.load(tmp_path / f"rank{r}.npy")
        assert np.all(res[:-1] <= 1.0), res   # every step within tolerance
        assert res[-1] == 0.0                  # no device status bits
