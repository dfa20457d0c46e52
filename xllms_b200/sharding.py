"""KV-head-group sharding of paged decode attention across the GPUs of a box.

Rank r of P owns KV heads [r*Hkv/P, (r+1)*Hkv/P) with their query heads, its
own page pool and block tables, and computes attention for them with the
single-GPU kernels. Query heads stay contiguous per rank, so the attention
output of the whole batch is the rank slices side by side along the head
axis: an all-gather of [B, Hq/P, D] per rank into [P, B, Hq/P, D] followed
by a head-axis interleave to [B, Hq, D]. That gather is the only exchange;
there is no reduction because every query head's softmax is local to its KV
head. The reference has no multi-device code; this is new.

torch.distributed carries the collective (NCCL on GPUs, gloo on CPU tests).
"""
from __future__ import annotations

from typing import Tuple


def head_range(num_heads: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Half-open range of heads rank `rank` owns."""
    if num_heads % world_size:
        raise ValueError(f"{num_heads} heads do not split over {world_size} ranks")
    n = num_heads // world_size
    return rank * n, (rank + 1) * n


def shard_heads(q, k, v, num_kv_heads: int, world_size: int, rank: int):
    """Rank `rank`'s slice of full inputs: q [B, Hq, D] -> its query heads,
    pools [NB, Hkv, P, D] -> its KV heads (same page ids). Returns copies."""
    Hq = q.shape[1]
    q0, q1 = head_range(Hq, world_size, rank)
    k0, k1 = head_range(num_kv_heads, world_size, rank)
    return q[:, q0:q1].copy(), k[:, k0:k1].copy(), v[:, k0:k1].copy()


def gather_heads(out_local, gathered=None, group=None):
    """All-gathers every rank's [B, Hq/P, D] slice; returns [P, B, Hq/P, D]."""
    import torch
    import torch.distributed as dist
    P = dist.get_world_size(group)
    if gathered is None:
        gathered = torch.empty((P,) + tuple(out_local.shape), dtype=out_local.dtype,
                               device=out_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, out_local.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), out_local.contiguous(), group=group)
    return gathered


def interleave_heads(gathered, out=None):
    """[P, B, Hq/P, D] -> [B, Hq, D] (rank-major head order = global head order)."""
    P, B, h, D = gathered.shape
    view = gathered.permute(1, 0, 2, 3)
    if out is None:
        return view.reshape(B, P * h, D)
    out.view(B, P, h, D).copy_(view)
    return out
