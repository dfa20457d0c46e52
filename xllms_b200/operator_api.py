"""Host-side mirror of the xLLMs paged-attention operator interface.

Three layers, all calling the C ABI of libxpa.so (include/operator_api.h):

* :func:`nxt_paged_attention`, :func:`nxt_paged_attention_v2`,
  :func:`nxt_paged_attention_flash` — the reference's entry points
  (include/operator_api.h:63-115 of the xLLMs project) with the same
  argument names, order and meaning. Pointer arguments accept torch CUDA
  tensors or raw device addresses. Unlike the reference (which returns
  nothing and checks nothing), a rejected call raises :class:`PagedAttentionError`.
* :func:`paged_attention` — tensor-level convenience over the status-returning
  ``nxt_paged_attention_ex`` that derives sizes and strides from the tensors.
* :class:`CudaBackendPlugin` — the dlopen'd plugin path
  (backends/cuda_backend.c:35-120), driven the way the reference's backend
  manager drives it (src/core/backend_manager.c:264-344).

torch is used for device memory and streams only; all arithmetic happens in
the native kernels.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Union

from . import _native

Pointer = Union[int, None, "torch.Tensor"]  # noqa: F821


class PagedAttentionError(RuntimeError):
    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {_native.strerror(code)} ({code})")


def _ptr(x: Pointer) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available() and torch.cuda.is_initialized():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:  # pragma: no cover
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _dropin(name: str, out, query, key_cache, value_cache, block_tables, seq_lens,
            num_seqs, num_heads, head_size, num_kv_heads, scale, max_num_blocks_per_seq,
            block_size, dtype_size, kv_block_stride, kv_head_stride, stream=None) -> None:
    lib = _native.xpa()
    getattr(lib, name)(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), int(num_seqs), int(num_heads), int(head_size), int(num_kv_heads),
        float(scale), int(max_num_blocks_per_seq), int(block_size), int(dtype_size),
        int(kv_block_stride), int(kv_head_stride), _stream_ptr(stream))
    rc = lib.nxt_paged_attention_last_error()
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, name)


def nxt_paged_attention(out, query, key_cache, value_cache, block_tables, seq_lens,
                        num_seqs, num_heads, head_size, num_kv_heads, scale,
                        max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride,
                        kv_head_stride, stream=None) -> None:
    """Reference ``nxt_paged_attention`` (operators/page_attention.cu:170)."""
    _dropin("nxt_paged_attention", out, query, key_cache, value_cache, block_tables, seq_lens,
            num_seqs, num_heads, head_size, num_kv_heads, scale, max_num_blocks_per_seq,
            block_size, dtype_size, kv_block_stride, kv_head_stride, stream)


def nxt_paged_attention_v2(out, query, key_cache, value_cache, block_tables, seq_lens,
                           num_seqs, num_heads, head_size, num_kv_heads, scale,
                           max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride,
                           kv_head_stride, stream=None) -> None:
    """Reference ``nxt_paged_attention_v2`` (operators/page_attention_v2.cu:262)."""
    _dropin("nxt_paged_attention_v2", out, query, key_cache, value_cache, block_tables,
            seq_lens, num_seqs, num_heads, head_size, num_kv_heads, scale,
            max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride, kv_head_stride,
            stream)


def nxt_paged_attention_flash(out, query, key_cache, value_cache, block_tables, seq_lens,
                              num_seqs, num_heads, head_size, num_kv_heads, scale,
                              max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride,
                              kv_head_stride, stream=None) -> None:
    """Reference ``nxt_paged_attention_flash`` (operators/flashinfer_adapter.cu:329)."""
    _dropin("nxt_paged_attention_flash", out, query, key_cache, value_cache, block_tables,
            seq_lens, num_seqs, num_heads, head_size, num_kv_heads, scale,
            max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride, kv_head_stride,
            stream)


def _dtype_size(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return 2
    if t.dtype == torch.float32:
        return 4
    raise PagedAttentionError(_native.NXT_PA_EINVAL, f"dtype {t.dtype}")


def _check_attention_inputs(where, query, key_cache, value_cache, block_tables, seq_lens, out,
                            one_byte=False):
    """Host checks before any pointer reaches the C ABI: ranks, shapes, dtypes,
    contiguity and device. The kernels read raw pointers in the reference
    layout, so a mismatch there would be misread, not reported."""
    import torch

    def bad(msg):
        raise PagedAttentionError(_native.NXT_PA_EINVAL, f"{where}: {msg}")
    if query.dim() != 3 or key_cache.dim() != 4:
        bad("query must be [B, Hq, D] and the pools [num_blocks, Hkv, block_size, D]")
    B, Hq, D = query.shape
    if key_cache.shape[3] != D or tuple(value_cache.shape) != tuple(key_cache.shape):
        bad("cache shapes")
    if one_byte:
        if query.dtype != torch.float16:
            bad("query must be fp16")
        if key_cache.element_size() != 1 or value_cache.element_size() != 1:
            bad("one-byte pools must be 1-byte tensors")
    else:
        _dtype_size(query)
        if key_cache.dtype != query.dtype or value_cache.dtype != query.dtype:
            bad("the K/V pools must have the query's dtype")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] < B:
        bad("block_tables must be int32 [B, max_blocks]")
    if seq_lens.dtype != torch.int32 or seq_lens.numel() < B:
        bad("seq_lens must be int32 [B]")
    ts = [query, key_cache, value_cache, block_tables, seq_lens]
    if out is not None:
        if tuple(out.shape) != tuple(query.shape) or out.dtype != query.dtype:
            bad("out must have the query's shape and dtype")
        ts.append(out)
    if not all(t.is_contiguous() for t in ts):
        bad("non-contiguous input")
    if not all(t.is_cuda and t.device == query.device for t in ts):
        bad("every tensor must be on the query's CUDA device")


def paged_attention(query, key_cache, value_cache, block_tables, seq_lens, *,
                    scale: Optional[float] = None, out=None, num_blocks: Optional[int] = None,
                    workspace=None, device_status=None, stream=None):
    """Decode attention of one new token per sequence over a paged KV cache.

    query [B, Hq, D]; key_cache/value_cache [num_blocks, Hkv, block_size, D]
    (contiguous, the reference layout); block_tables [B, max_blocks] int32;
    seq_lens [B] int32; all on the same CUDA device. Returns out [B, Hq, D] in
    query's dtype. ``scale`` defaults to 1/sqrt(D). ``num_blocks`` defaults to
    key_cache.shape[0], which lets the kernels mask out-of-range pages.
    """
    import torch
    _check_attention_inputs("paged_attention", query, key_cache, value_cache, block_tables,
                            seq_lens, out)
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    if out is None:
        out = torch.empty_like(query)
    ds = _dtype_size(query)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    ws_bytes = 0
    if workspace is not None:
        ws_bytes = workspace.numel() * workspace.element_size()
    rc = _native.xpa().nxt_paged_attention_ex(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), B, Hq, D, Hkv, float(scale), block_tables.shape[1], bs, ds,
        Hkv * bs * D, bs * D, nb if num_blocks is None else int(num_blocks),
        _ptr(workspace), ws_bytes, _ptr(device_status), _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_paged_attention_ex")
    return out


def workspace_size(num_seqs, num_heads, head_size, num_kv_heads, max_num_blocks_per_seq,
                   block_size=16, dtype_size=2) -> int:
    return int(_native.xpa().nxt_paged_attention_workspace_size(
        num_seqs, num_heads, head_size, num_kv_heads, max_num_blocks_per_seq, block_size,
        dtype_size))


def kernel_path(key_cache, value_cache, num_heads, head_size, num_kv_heads, block_size,
                dtype_size, kv_block_stride, kv_head_stride) -> int:
    """NXT_PA_PATH_* the kernels take for these arguments."""
    return int(_native.xpa().nxt_paged_attention_path(
        _ptr(key_cache), _ptr(value_cache), num_heads, head_size, num_kv_heads, block_size,
        dtype_size, kv_block_stride, kv_head_stride))


def device_status(clear: bool = True) -> int:
    """NXT_PA_DEV_* bits of the current device's library status word."""
    rc = _native.xpa().nxt_paged_attention_device_status(1 if clear else 0)
    if rc < 0:
        raise PagedAttentionError(rc, "nxt_paged_attention_device_status")
    return rc


# ── plugin path ───────────────────────────────────────────────────────────
class NxtBackend(ctypes.Structure):
    """Layout of the reference's NxtBackend (include/backend.h:141-151)."""
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("so_path", ctypes.c_char_p),
        ("dl_handle", ctypes.c_void_p),
        ("api", ctypes.c_void_p * 8),
        ("state", ctypes.c_int),
        ("priority", ctypes.c_int32),
        ("model_count", ctypes.c_uint32),
        ("models", ctypes.c_void_p),
        ("backend_state", ctypes.c_void_p),
    ]


class NxtPagedAttentionInput(ctypes.Structure):
    """Layout of the reference's NxtPagedAttentionInput (backends/cuda_backend.h:29-46)."""
    _fields_ = [
        ("query", ctypes.c_void_p),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("num_seqs", ctypes.c_int),
        ("num_heads", ctypes.c_int),
        ("head_size", ctypes.c_int),
        ("num_kv_heads", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("max_num_blocks_per_seq", ctypes.c_int),
        ("block_size", ctypes.c_int),
        ("dtype_size", ctypes.c_int),
        ("kv_block_stride", ctypes.c_int),
        ("kv_head_stride", ctypes.c_int),
        ("stream", ctypes.c_void_p),
    ]


NXT_BACKEND_STATE_UNINITIALIZED = 0
NXT_BACKEND_STATE_READY = 2


class CudaBackendPlugin:
    """libxllm_cuda_backend.so driven like the reference backend manager does:
    init on load, run(input descriptor, output), fini on unload."""

    def __init__(self, name: str = "cuda"):
        self.lib = _native.plugin()
        self.backend = NxtBackend()
        self.backend.name = name.encode()
        self.backend.so_path = _native.PLUGIN_PATH.encode()
        rc = self.lib.nxt_backend_init(ctypes.byref(self.backend))
        if rc != 0:
            raise PagedAttentionError(_native.NXT_PA_ECUDA, "nxt_backend_init")

    def run(self, pa: NxtPagedAttentionInput, output: Pointer) -> int:
        return int(self.lib.nxt_backend_run(ctypes.byref(self.backend), ctypes.byref(pa),
                                            _ptr(output)))

    def close(self) -> int:
        return int(self.lib.nxt_backend_fini(ctypes.byref(self.backend)))


def make_input(query, key_cache, value_cache, block_tables, seq_lens, scale=None,
               stream=None) -> NxtPagedAttentionInput:
    """Fills the plugin's input descriptor from tensors in the reference layout."""
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    pa = NxtPagedAttentionInput()
    pa.query = _ptr(query)
    pa.key_cache = _ptr(key_cache)
    pa.value_cache = _ptr(value_cache)
    pa.block_tables = _ptr(block_tables)
    pa.seq_lens = _ptr(seq_lens)
    pa.num_seqs, pa.num_heads, pa.head_size, pa.num_kv_heads = B, Hq, D, Hkv
    pa.scale = 1.0 / math.sqrt(D) if scale is None else scale
    pa.max_num_blocks_per_seq = block_tables.shape[1]
    pa.block_size = bs
    pa.dtype_size = _dtype_size(query)
    pa.kv_block_stride = Hkv * bs * D
    pa.kv_head_stride = bs * D
    pa.stream = _stream_ptr(stream)
    return pa


# ── KV append ─────────────────────────────────────────────────────────────
def _index_ok(slot_mapping, n, like) -> bool:
    """slot_mapping: contiguous int64 with >= n entries on `like`'s device."""
    import torch
    return (slot_mapping.dtype == torch.int64 and slot_mapping.is_contiguous()
            and slot_mapping.numel() >= n and slot_mapping.device == like.device)


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, stream=None) -> None:
    """Scatter key/value [T, Hkv, D] into the pools [NB, Hkv, P, D] at
    slot_mapping[t] (int64; page = slot // P, slot % P; negative: skipped)."""
    T, Hkv, D = key.shape
    nb, hk, bs, dk = key_cache.shape
    if (hk != Hkv or dk != D or tuple(value.shape) != tuple(key.shape)
            or tuple(value_cache.shape) != tuple(key_cache.shape)
            or not (key_cache.is_contiguous() and value_cache.is_contiguous())
            or key.stride(2) != 1 or key.stride(1) != D or value.stride() != key.stride()
            or key.dtype != key_cache.dtype or value.dtype != key_cache.dtype
            or value_cache.dtype != key_cache.dtype
            or not _index_ok(slot_mapping, T, key) or not key.is_cuda
            or len({t.device for t in (key, value, key_cache, value_cache)}) != 1):
        raise PagedAttentionError(_native.NXT_PA_EINVAL, "reshape_and_cache: shapes")
    rc = _native.xpa().nxt_reshape_and_cache(
        _ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache), _ptr(slot_mapping), T, Hkv, D,
        bs, _dtype_size(key), Hkv * bs * D, bs * D, key.stride(0), _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_reshape_and_cache")


def paged_attention_append(query, key_cache, value_cache, block_tables, seq_lens, new_key,
                           new_value, slot_mapping, *, scale=None, out=None, num_blocks=None,
                           device_status=None, stream=None):
    """One decode step with the KV append fused in: new_key/new_value
    [B, Hkv, D] are written at slot_mapping[b] and included in the attention
    (seq_lens count them)."""
    import torch
    _check_attention_inputs("paged_attention_append", query, key_cache, value_cache,
                            block_tables, seq_lens, out)
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    if (tuple(new_key.shape) != (B, Hkv, D) or tuple(new_value.shape) != (B, Hkv, D)
            or new_key.dtype != query.dtype or new_value.dtype != query.dtype
            or not (new_key.is_contiguous() and new_value.is_contiguous())
            or not _index_ok(slot_mapping, B, query) or new_key.device != query.device
            or new_value.device != query.device):
        raise PagedAttentionError(_native.NXT_PA_EINVAL, "paged_attention_append: shapes")
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rc = _native.xpa().nxt_paged_attention_append_ex(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), _ptr(new_key), _ptr(new_value), _ptr(slot_mapping), B, Hq, D, Hkv,
        float(scale), block_tables.shape[1], bs, _dtype_size(query), Hkv * bs * D, bs * D,
        nb if num_blocks is None else int(num_blocks), _ptr(device_status), _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_paged_attention_append_ex")
    return out


# ── shared-prefix (cascade) attention ─────────────────────────────────────
class PrefixGroups:
    """Device arrays of nxt_paged_attention_prefix_ex, built once from a host
    list of (member sequence ids, shared prefix pages) pairs."""

    def __init__(self, groups, num_seqs, device=None, *, prefix_pages=None, offsets=None,
                 members=None, bounds=None):
        import torch
        if bounds is not None:  # (num_groups, max_group_size, max_prefix_pages)
            self.num_groups, self.max_group_size, self.max_prefix_pages = (int(x) for x in bounds)
        else:
            self.num_groups = len(groups)
            self.max_group_size = max((len(m) for m, _ in groups), default=0)
            self.max_prefix_pages = max((int(p) for _, p in groups), default=0)
        if prefix_pages is None:
            pp, off, mem = self.host_arrays(groups, num_seqs)
            t = lambda x: torch.from_numpy(x).to(device)
            prefix_pages, offsets, members = t(pp), t(off), t(mem)
        self.prefix_pages, self.offsets, self.members = prefix_pages, offsets, members

    @staticmethod
    def host_arrays(groups, num_seqs):
        """(prefix_pages [num_seqs], offsets [G+1], members [sum of sizes]) as int32."""
        import numpy as np
        pp = np.zeros(max(1, num_seqs), dtype=np.int32)
        off = [0]
        mem = []
        for seqs, pages in groups:
            for b in seqs:
                if not 0 <= int(b) < num_seqs:
                    raise ValueError(f"group member {b} outside the batch")
                if pp[int(b)]:
                    raise ValueError(f"sequence {b} is in two prefix groups")
                pp[int(b)] = int(pages)
            mem.extend(int(b) for b in seqs)
            off.append(len(mem))
        return (pp, np.asarray(off, dtype=np.int32),
                np.asarray(mem if mem else [0], dtype=np.int32))


def paged_attention_prefix(query, key_cache, value_cache, block_tables, seq_lens, groups, *,
                           scale=None, out=None, num_blocks=None, device_status=None,
                           stream=None):
    """Decode attention for a batch with shared prefixes. `groups` is a
    PrefixGroups or a host list of (member sequence ids, shared prefix pages);
    every member's seq_len covers its prefix and its block-table row starts
    with the group's shared pages. The result equals paged_attention's."""
    import torch
    _check_attention_inputs("paged_attention_prefix", query, key_cache, value_cache,
                            block_tables, seq_lens, out)
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    if not isinstance(groups, PrefixGroups):
        groups = PrefixGroups(groups, B, query.device)
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rc = _native.xpa().nxt_paged_attention_prefix_ex(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), _ptr(groups.prefix_pages), _ptr(groups.offsets), _ptr(groups.members),
        groups.num_groups, groups.max_group_size, groups.max_prefix_pages, B, Hq, D, Hkv,
        float(scale), block_tables.shape[1], bs, _dtype_size(query), Hkv * bs * D, bs * D,
        nb if num_blocks is None else int(num_blocks), None, 0, _ptr(device_status),
        _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_paged_attention_prefix_ex")
    return out


# ── activations (operators/activation_kernels.cu of the reference) ─────────
ACTIVATIONS = {
    "silu_and_mul": _native.NXT_ACT_SILU_AND_MUL,
    "mul_and_silu": _native.NXT_ACT_MUL_AND_SILU,
    "gelu_and_mul": _native.NXT_ACT_GELU_AND_MUL,
    "gelu_tanh_and_mul": _native.NXT_ACT_GELU_TANH_AND_MUL,
    "gelu": _native.NXT_ACT_GELU,
    "silu": _native.NXT_ACT_SILU,
}


def activation(name, x, *, out=None, stream=None):
    """Gated ops take x [..., 2d] ([gate | up]) and return [..., d]; the
    element-wise ops (gelu, silu) keep x's shape. fp16 or fp32, contiguous."""
    import torch
    op = ACTIVATIONS[name]
    if not x.is_contiguous():
        raise ValueError("activation input must be contiguous")
    gated = op <= _native.NXT_ACT_GELU_TANH_AND_MUL
    width = x.shape[-1]
    if gated and width % 2:
        raise ValueError("gated activation input needs an even last dimension")
    d = width // 2 if gated else width
    rows = x.numel() // width if width else 0
    if out is None:
        out = torch.empty(tuple(x.shape[:-1]) + (d,), dtype=x.dtype, device=x.device)
    elif out.numel() != rows * d or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("activation output does not match the input")
    rc = _native.xpa().nxt_activation_ex(op, _ptr(out), _ptr(x), rows, d, _dtype_size(x),
                                         _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_activation_ex")
    return out


# ── one-byte KV cache (fp8 E4M3 / E5M2, int8) ──────────────────────────────
FP8_FORMATS = {"e4m3": _native.NXT_KV_FP8_E4M3, "e5m2": _native.NXT_KV_FP8_E5M2,
               "int8": _native.NXT_KV_INT8}


def _fp8_code(fmt):
    return FP8_FORMATS[fmt] if isinstance(fmt, str) else int(fmt)


def paged_attention_fp8(query, key_cache, value_cache, block_tables, seq_lens, fmt, k_scale,
                        v_scale, *, scale=None, out=None, num_blocks=None, workspace=None,
                        device_status=None, stream=None):
    """Decode attention over one-byte pools (uint8 / int8 / float8 tensors
    [NB, Hkv, P, D] holding encode(x / scale) in format `fmt`: "e4m3", "e5m2"
    or "int8"); query and output fp16 [B, Hq, D]."""
    import torch
    _check_attention_inputs("paged_attention_fp8", query, key_cache, value_cache, block_tables,
                            seq_lens, out, one_byte=True)
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (_ptr(workspace),
                                                            workspace.numel() * workspace.element_size())
    rc = _native.xpa().nxt_paged_attention_fp8_ex(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), B, Hq, D, Hkv, float(scale), block_tables.shape[1], bs, _fp8_code(fmt),
        float(k_scale), float(v_scale), Hkv * bs * D, bs * D,
        nb if num_blocks is None else int(num_blocks), ws_ptr, ws_bytes, _ptr(device_status),
        _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_paged_attention_fp8_ex")
    return out


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping, fmt, k_scale, v_scale,
                          stream=None) -> None:
    """Quantise fp16 key/value [T, Hkv, D] into the one-byte pools
    [NB, Hkv, P, D] (format `fmt`) at slot_mapping[t] (int64; negative:
    skipped)."""
    import torch
    T, Hkv, D = key.shape
    nb, hk, bs, dk = key_cache.shape
    if (hk != Hkv or dk != D or tuple(value.shape) != tuple(key.shape)
            or tuple(value_cache.shape) != tuple(key_cache.shape)
            or key_cache.element_size() != 1 or value_cache.element_size() != 1
            or not (key_cache.is_contiguous() and value_cache.is_contiguous())
            or key.stride(2) != 1 or key.stride(1) != D or value.stride() != key.stride()
            or key.dtype != torch.float16 or value.dtype != torch.float16
            or not _index_ok(slot_mapping, T, key) or not key.is_cuda
            or len({t.device for t in (key, value, key_cache, value_cache)}) != 1):
        raise PagedAttentionError(_native.NXT_PA_EINVAL, "reshape_and_cache_fp8: shapes")
    rc = _native.xpa().nxt_reshape_and_cache_fp8(
        _ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache), _ptr(slot_mapping), T, Hkv, D,
        bs, _fp8_code(fmt), float(k_scale), float(v_scale), Hkv * bs * D, bs * D, key.stride(0),
        _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_reshape_and_cache_fp8")


def paged_attention_fp8_append(query, key_cache, value_cache, block_tables, seq_lens, new_key,
                               new_value, slot_mapping, fmt, k_scale, v_scale, *, scale=None,
                               out=None, num_blocks=None, device_status=None, stream=None):
    """One decode step on one-byte pools with the quantising append fused in:
    new_key/new_value (fp16 [B, Hkv, D]) are stored at slot_mapping[b] in
    format `fmt` and included in the attention (seq_lens count them)."""
    import torch
    _check_attention_inputs("paged_attention_fp8_append", query, key_cache, value_cache,
                            block_tables, seq_lens, out, one_byte=True)
    B, Hq, D = query.shape
    nb, Hkv, bs, _ = key_cache.shape
    if (tuple(new_key.shape) != (B, Hkv, D) or tuple(new_value.shape) != (B, Hkv, D)
            or new_key.dtype != torch.float16 or new_value.dtype != torch.float16
            or not (new_key.is_contiguous() and new_value.is_contiguous())
            or not _index_ok(slot_mapping, B, query) or new_key.device != query.device
            or new_value.device != query.device):
        raise PagedAttentionError(_native.NXT_PA_EINVAL, "paged_attention_fp8_append: shapes")
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rc = _native.xpa().nxt_paged_attention_fp8_append_ex(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(seq_lens), _ptr(new_key), _ptr(new_value), _ptr(slot_mapping), B, Hq, D, Hkv,
        float(scale), block_tables.shape[1], bs, _fp8_code(fmt), float(k_scale), float(v_scale),
        Hkv * bs * D, bs * D, nb if num_blocks is None else int(num_blocks),
        _ptr(device_status), _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_paged_attention_fp8_append_ex")
    return out


# ── block-table builder ────────────────────────────────────────────────────
class BlockTables:
    """One decode step's kernel inputs on the device, built by
    nxt_build_block_tables: tables [B, max_blocks] int32, seq_lens [B],
    slots [B] int64 (the newest token's slot), prefix (PrefixGroups or None)."""

    def __init__(self, buffer, offsets, B, max_blocks, bounds):
        import torch
        self.buffer = buffer

        def view(key, n, dtype):
            o = offsets[key]
            es = torch.tensor([], dtype=dtype).element_size()
            return buffer[o:o + n * es].view(dtype)
        self.tables = view(_native.NXT_BT_TABLES, B * max_blocks, torch.int32).view(B, max_blocks)
        self.seq_lens = view(_native.NXT_BT_SEQ_LENS, B, torch.int32)
        self.slots = view(_native.NXT_BT_SLOTS, B, torch.int64)
        pp = view(_native.NXT_BT_PREFIX_PAGES, B, torch.int32)
        go = view(_native.NXT_BT_GROUP_OFFSETS, B + 1, torch.int32)
        mem = view(_native.NXT_BT_GROUP_MEMBERS, B, torch.int32)
        self.prefix = (PrefixGroups(None, B, prefix_pages=pp, offsets=go, members=mem,
                                    bounds=bounds) if bounds[0] > 0 else None)


def build_block_tables(page_lists, seq_lens, max_blocks, *, block_size=16, prefix_node=None,
                       prefix_pages=None, device=None, stream=None, staging=None):
    """page_lists: per sequence, its physical pages in token order; seq_lens:
    context tokens (newest included); prefix_node / prefix_pages: per
    sequence, the radix node of its shared prefix (-1: none) and the whole
    pages it covers. Returns BlockTables on `device`."""
    import numpy as np
    import torch
    B = len(page_lists)
    counts = np.array([len(p) for p in page_lists], dtype=np.int64)
    offs = np.zeros(B + 1, dtype=np.int32)
    np.cumsum(counts, out=offs[1:])
    ids = (np.concatenate([np.asarray(p, dtype=np.int32) for p in page_lists])
           if B and offs[-1] else np.zeros(1, dtype=np.int32))
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    node = None if prefix_node is None else np.ascontiguousarray(prefix_node, dtype=np.int32)
    ppg = None if prefix_pages is None else np.ascontiguousarray(prefix_pages, dtype=np.int32)
    lib = _native.xpa()
    offsets = (ctypes.c_size_t * _native.NXT_BT_NUM_ARRAYS)()
    total = lib.nxt_block_tables_layout(B, int(max_blocks), int(offs[-1]), offsets)
    buf = torch.empty(max(total, 16), dtype=torch.uint8, device=device)
    g = (ctypes.c_int * 3)()
    ptr = lambda a: None if a is None else a.ctypes.data
    st_ptr, st_bytes = (None, 0) if staging is None else (staging.data_ptr(),
                                                          staging.numel() * staging.element_size())
    rc = lib.nxt_build_block_tables(
        ptr(offs), ptr(ids), ptr(sl), ptr(node), ptr(ppg), B, int(max_blocks), int(block_size),
        _ptr(buf), total, st_ptr, st_bytes, ctypes.addressof(g),
        ctypes.addressof(g) + 4, ctypes.addressof(g) + 8, _stream_ptr(stream))
    if rc != _native.NXT_PA_OK:
        raise PagedAttentionError(rc, "nxt_build_block_tables")
    return BlockTables(buf, list(offsets), B, int(max_blocks), (g[0], g[1], g[2]))
