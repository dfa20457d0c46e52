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

import ctypes
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


# ── fused head gather over NVLink peer stores ────────────────────────────
class NxtPaShard(ctypes.Structure):
    """Layout of NxtPaShard (include/operator_api.h)."""
    _fields_ = [
        ("world_size", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("total_heads", ctypes.c_int),
        ("head_offset", ctypes.c_int),
        ("peer_out", ctypes.c_void_p * 8),
        ("peer_flags", ctypes.c_void_p * 8),
        ("mc_out", ctypes.c_void_p),
    ]


class _DeviceArray:
    """Zero-copy view of device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def torch_exchange(group=None):
    """Handle exchange over torch.distributed: bytes -> every rank's bytes."""
    import torch.distributed as dist

    def exchange(blob: bytes):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, blob, group=group)
        return [bytes(x) for x in out]
    return exchange


def multicast_supported(device) -> bool:
    """Whether torch symmetric memory can give an NVLink multicast address
    on `device` (False when the query itself is unavailable)."""
    try:
        import torch
        import torch.distributed._symmetric_memory as symm_mem
        idx = torch.device(device).index
        return bool(symm_mem._SymmetricMemory.has_multicast_support(
            symm_mem.DeviceType.CUDA, idx if idx is not None else torch.cuda.current_device()))
    except Exception:
        return False


class FusedHeadGather:
    """KV-head-sharded decode attention whose output all-gather is fused into
    the kernels (nxt_paged_attention_sharded): each rank's kernels store its
    heads straight into every rank's gather buffer over NVLink, and a bounded
    cross-GPU barrier ends the step. The buffers are exchanged once, here,
    through `exchange` (e.g. torch_exchange()).

    run() enqueues step s and returns a [B, total_heads, D] view of half
    (s & 1) of this rank's buffer, complete once the stream reaches it.

    multicast=True takes the buffers from torch symmetric memory over `group`
    (a torch.distributed process group; `exchange` is then unused) and, when
    the GPUs support it, passes their NVLink multicast address so that each
    16-byte row chunk leaves the GPU once and NVSwitch writes it into every
    rank's buffer (`self.multicast` says whether that address exists).
    Failure tests keep the default: a rank that dies while its memory is
    bound to a multicast object can fault its peers' GPUs."""

    def __init__(self, num_seqs: int, total_heads: int, head_size: int, dtype_size: int,
                 world_size: int, rank: int, exchange, device=None, multicast: bool = False,
                 group=None):
        from . import _native
        self.lib = _native.xpa()
        self.B, self.H, self.D, self.es = num_seqs, total_heads, head_size, dtype_size
        self.world, self.rank = world_size, rank
        if total_heads % world_size:
            raise ValueError("total_heads must split evenly over the ranks")
        half = num_seqs * total_heads * head_size * dtype_size
        self.half_bytes = half
        self.flags_off = (2 * half + 255) // 256 * 256
        total = self.flags_off + 8 * world_size
        self.opened = []
        self.own = 0
        self.symm = None
        self.multicast = False
        self.shard = NxtPaShard()
        self.shard.world_size, self.shard.rank = world_size, rank
        self.shard.total_heads = total_heads
        self.shard.head_offset = rank * (total_heads // world_size)
        if multicast:
            bases, mc = self._symmetric(total, device, group)
            for r in range(world_size):
                self.shard.peer_out[r] = bases[r]
                self.shard.peer_flags[r] = bases[r] + self.flags_off
            self.shard.mc_out = mc or None
            self.multicast = bool(mc)
            base_own = bases[rank]
        else:
            own = ctypes.c_void_p()
            handle = (ctypes.c_char * _native.NXT_PA_IPC_HANDLE_BYTES)()
            rc = self.lib.nxt_pa_peer_alloc(total, ctypes.byref(own), handle)
            if rc != 0:
                raise RuntimeError(f"nxt_pa_peer_alloc: {_native.strerror(rc)}")
            self.own = own.value
            base_own = self.own
            handles = exchange(bytes(handle))
            for r in range(world_size):
                if r == rank:
                    base = self.own
                else:
                    p = ctypes.c_void_p()
                    rc = self.lib.nxt_pa_peer_open(handles[r], ctypes.byref(p))
                    if rc != 0:
                        raise RuntimeError(f"nxt_pa_peer_open(rank {r}): {_native.strerror(rc)}")
                    base = p.value
                    self.opened.append(base)
                self.shard.peer_out[r] = base
                self.shard.peer_flags[r] = base + self.flags_off
        self.step = 0
        self.device = device
        # Views of the two halves, made once: importing device memory into
        # torch per step would cost host time on every step.
        import torch
        typestr = "<f2" if self.es == 2 else "<f4"
        self.views = [torch.as_tensor(_DeviceArray(base_own + i * self.half_bytes,
                                                   (self.B, self.H, self.D), typestr),
                                      device=device) for i in (0, 1)]

    def _symmetric(self, nbytes, device, group):
        """Buffers from torch symmetric memory: every rank's base address as
        mapped here, and the multicast address (0 when unsupported)."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group or dist.group.WORLD
        self.symm = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.symm.zero_()
        torch.cuda.synchronize(device)
        hdl = symm_mem.rendezvous(self.symm, group)
        self.symm_handle = hdl
        off = self.symm.data_ptr() - int(hdl.buffer_ptrs[self.rank])
        bases = [int(x) + off for x in hdl.buffer_ptrs]
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        mc = int(hdl.multicast_ptr) if multicast_supported(dev) else 0
        dist.barrier(group)
        return bases, (mc + off) if mc else 0

    def output(self, step: int):
        """[B, total_heads, D] view of the half that holds step `step`."""
        return self.views[step & 1]

    def run(self, query, key_cache, value_cache, block_tables, seq_lens, scale, num_blocks,
            device_status=None, stream=None, kv_format=None, k_scale=1.0, v_scale=1.0):
        """Enqueues the next step. With `kv_format` ("e4m3", "e5m2" or "int8")
        the pools are one-byte pools holding encode(x / scale) and the query
        is fp16 (nxt_paged_attention_fp8_sharded)."""
        from . import _native
        from .operator_api import (_check_attention_inputs, _dtype_size, _fp8_code, _ptr,
                                   _stream_ptr)
        _check_attention_inputs("FusedHeadGather.run", query, key_cache, value_cache,
                                block_tables, seq_lens, None, one_byte=kv_format is not None)
        B, Hq, D = query.shape
        nb, Hkv, bs, _ = key_cache.shape
        # the peer buffers were sized for these: anything larger would be
        # stored past their end on another GPU
        if (B != self.B or Hq != self.H // self.world or D != self.D
                or _dtype_size(query) != self.es):
            raise ValueError(f"FusedHeadGather.run: batch [{B}, {Hq}, {D}] x {query.dtype} does "
                             f"not match the buffers' [{self.B}, {self.H // self.world}, {self.D}]"
                             f" x {self.es}-byte elements")
        self.step += 1
        head = (ctypes.byref(self.shard), self.step, _ptr(query), _ptr(key_cache),
                _ptr(value_cache), _ptr(block_tables), _ptr(seq_lens), B, Hq, D, Hkv, float(scale),
                block_tables.shape[1], bs)
        tail = (Hkv * bs * D, bs * D, int(num_blocks), _ptr(device_status), _stream_ptr(stream))
        if kv_format is None:
            name = "nxt_paged_attention_sharded"
            rc = self.lib.nxt_paged_attention_sharded(*head, self.es, *tail)
        else:
            name = "nxt_paged_attention_fp8_sharded"
            rc = self.lib.nxt_paged_attention_fp8_sharded(*head, _fp8_code(kv_format),
                                                         float(k_scale), float(v_scale), *tail)
        if rc != 0:
            raise RuntimeError(f"{name}: {_native.strerror(rc)}")
        return self.output(self.step)

    def close(self, barrier=None):
        """Unmaps the peers' buffers and frees this rank's; `barrier` (e.g.
        torch.distributed.barrier) must keep every rank here until all are
        done with every buffer."""
        import torch
        torch.cuda.synchronize()
        if barrier:
            barrier()
        for p in self.opened:
            self.lib.nxt_pa_peer_close(p)
        self.opened = []
        if barrier:
            barrier()
        self.views = []
        if self.own:
            self.lib.nxt_pa_peer_free(self.own)
            self.own = 0
        self.symm_handle = None
        self.symm = None
