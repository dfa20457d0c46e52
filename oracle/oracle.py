"""ctypes bindings of the CPU oracle (pa_oracle.c) and of the reference's own
CPU attention (ref_shim.c over examples/run_gpt2.c of the xLLMs project).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, always as the checker or the timed
CPU baseline, never by the product path. Build with ``make -C oracle``.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libpa_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libxllm_ref_cpu.so")

_P = ctypes.c_void_p
_I, _F, _I64 = ctypes.c_int, ctypes.c_float, ctypes.c_int64
_ORACLE_ARGS = [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _I, _I, _I64, _I64, _I64]

_oracle = None
_ref = None


def _c(a: np.ndarray) -> int:
    return a.ctypes.data


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle`")
        lib = ctypes.CDLL(ORACLE_SO)
        lib.pa_oracle_f32.restype = _I
        lib.pa_oracle_f32.argtypes = _ORACLE_ARGS
        lib.pa_oracle_f64.restype = _I
        lib.pa_oracle_f64.argtypes = _ORACLE_ARGS
        lib.pa_oracle_f32_omp.restype = _I
        lib.pa_oracle_f32_omp.argtypes = _ORACLE_ARGS + [_I]
        lib.pa_oracle_split_partials.restype = _I
        lib.pa_oracle_split_partials.argtypes = [_P, _P, _P] + _ORACLE_ARGS[1:] + [_I, _I]
        lib.pa_oracle_merge_partials.restype = None
        lib.pa_oracle_merge_partials.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        lib.pa_oracle_gather_checksum.restype = _I
        lib.pa_oracle_gather_checksum.argtypes = [_P, _P, _P, _I, _I, _I, _I, _I, _I64]
        lib.pa_oracle_reshape_and_cache.restype = None
        lib.pa_oracle_reshape_and_cache.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                                                    _I64, _I64, _I64]
        lib.pa_gather_mix.restype = ctypes.c_uint64
        lib.pa_gather_mix.argtypes = [ctypes.c_uint64] * 3
        lib.pa_fp8_decode.restype = None
        lib.pa_fp8_decode.argtypes = [_P, _P, _I64, _I]
        lib.pa_fp8_encode.restype = None
        lib.pa_fp8_encode.argtypes = [_P, _P, _I64, _I]
        lib.act_oracle.restype = _I
        lib.act_oracle.argtypes = [_I, _P, _P, _I, _I, _I]
        lib.pa_half_to_float.restype = _F
        lib.pa_half_to_float.argtypes = [ctypes.c_uint16]
        lib.pa_float_to_half.restype = ctypes.c_uint16
        lib.pa_float_to_half.argtypes = [_F]
        _oracle = lib
    return _oracle


def activation(op: int, x: np.ndarray) -> np.ndarray:
    """The activation oracle on x [rows, 2d] (gated ops 0-3) or [rows, d]
    (element-wise ops 4, 5); fp16 or fp32, result in x's dtype."""
    x = np.ascontiguousarray(x)
    rows, width = x.shape
    d = width // 2 if op <= 3 else width
    out = np.zeros((rows, d), dtype=x.dtype)
    rc = oracle_lib().act_oracle(int(op), _c(out), _c(x), rows, d, x.dtype.itemsize)
    if rc != 0:
        raise ValueError("activation oracle rejected the arguments")
    return out


REF_ACT_SO = os.path.join(HERE, "_ref", "libxllm_ref_act.so")
_ref_act = None


def ref_act_available() -> bool:
    return os.path.exists(REF_ACT_SO)


def ref_act_lib() -> ctypes.CDLL:
    """The reference's own activation kernels (GPU), built by oracle/Makefile."""
    global _ref_act
    if _ref_act is None:
        lib = ctypes.CDLL(REF_ACT_SO)
        lib.ref_activation.restype = _I
        lib.ref_activation.argtypes = [_I, _P, _P, _I, _I, _I, _P]
        _ref_act = lib
    return _ref_act


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle` with the reference")
        lib = ctypes.CDLL(REF_SO)
        lib.ref_run_gpt2_paged_attention.restype = None
        lib.ref_run_gpt2_paged_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _P]
        lib.ref_run_gpt2_batch.restype = None
        lib.ref_run_gpt2_batch.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I]
        lib.ref_run_gpt2_max_threads.restype = _I
        lib.ref_run_gpt2_max_threads.argtypes = []
        _ref = lib
    return _ref


def _as(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _common(q, k, v, block_tables, seq_lens):
    ds = 2 if q.dtype == np.float16 else 4
    npd = np.float16 if ds == 2 else np.float32
    return (_as(q, npd), _as(k, npd), _as(v, npd), _as(block_tables, np.int32),
            _as(seq_lens, np.int32), ds)


def attention(q, k, v, block_tables, seq_lens, num_kv_heads, scale, block_size=16,
              kv_block_stride=None, kv_head_stride=None, num_blocks=-1, f64=False,
              threads: Optional[int] = None) -> np.ndarray:
    """Oracle output [B, Hq, D] (fp32, or fp64 with f64=True). q is [B, Hq, D];
    k/v are flat pools in the reference layout (any shape, C order)."""
    q, k, v, bt, sl, ds = _common(q, k, v, block_tables, seq_lens)
    B, H, D = q.shape
    kbs = num_kv_heads * block_size * D if kv_block_stride is None else kv_block_stride
    khs = block_size * D if kv_head_stride is None else kv_head_stride
    lib = oracle_lib()
    args = (_c(q), _c(k), _c(v), _c(bt), _c(sl), B, H, D, num_kv_heads, float(scale),
            bt.shape[1], block_size, ds, kbs, khs, int(num_blocks))
    if f64:
        out = np.zeros((B, H, D), dtype=np.float64)
        rc = lib.pa_oracle_f64(_c(out), *args)
    elif threads is not None:
        out = np.zeros((B, H, D), dtype=np.float32)
        rc = lib.pa_oracle_f32_omp(_c(out), *args, int(threads))
    else:
        out = np.zeros((B, H, D), dtype=np.float32)
        rc = lib.pa_oracle_f32(_c(out), *args)
    if rc != 0:
        raise ValueError("oracle rejected the arguments")
    return out


def build_block_tables(page_offsets, page_ids, seq_lens, max_blocks, block_size=16,
                       prefix_node=None, prefix_pages=None):
    """Restatement of the block-table builder (xllms_b200/csrc/pa_tables.cu):
    padded tables (-1), newest-token slots, and prefix groups (sequences
    sharing a radix node with >= 1 whole page; groups of two or more, by
    node id, members in sequence order). Returns (tables, slots,
    prefix_pages_out, group_offsets, members, num_groups, max_group_size,
    max_prefix_pages)."""
    off = np.asarray(page_offsets, dtype=np.int64)
    ids = np.asarray(page_ids, dtype=np.int64)
    sl = np.asarray(seq_lens, dtype=np.int64)
    B = len(sl)
    tables = np.full((B, max_blocks), -1, dtype=np.int32)
    slots = np.full(B, -1, dtype=np.int64)
    for b in range(B):
        row = ids[off[b]:off[b + 1]]
        tables[b, :len(row)] = row
        if sl[b] > 0:
            slots[b] = row[(sl[b] - 1) // block_size] * block_size + (sl[b] - 1) % block_size
    pp = np.zeros(B, dtype=np.int32)
    go = np.zeros(B + 1, dtype=np.int32)
    mem = np.zeros(B, dtype=np.int32)
    G = nm = max_size = max_pages = 0
    if prefix_node is not None:
        nodes = {}
        for b in range(B):
            if prefix_node[b] >= 0 and prefix_pages[b] > 0:
                nodes.setdefault(int(prefix_node[b]), []).append(b)
        for node in sorted(nodes):
            m = nodes[node]
            if len(m) < 2:
                continue
            for b in m:
                pp[b] = prefix_pages[m[0]]
                mem[nm] = b
                nm += 1
            G += 1
            go[G] = nm
            max_size = max(max_size, len(m))
            max_pages = max(max_pages, int(prefix_pages[m[0]]))
        go[G + 1:] = nm
    return tables, slots, pp, go, mem, G, max_size, max_pages


FP8_E4M3, FP8_E5M2, KV_INT8 = 1, 2, 3  # one-byte KV formats


def fp8_decode(codes, fmt) -> np.ndarray:
    """uint8 codes -> float32 values (exact); fmt FP8_E4M3, FP8_E5M2 or KV_INT8."""
    c = _as(codes, np.uint8)
    out = np.zeros(c.shape, dtype=np.float32)
    oracle_lib().pa_fp8_decode(_c(out), _c(c), c.size, int(fmt))
    return out


def fp8_encode(x, fmt) -> np.ndarray:
    """float32 -> uint8 codes (round to nearest even, saturating; KV_INT8
    codes are two's complement and NaN encodes as 0)."""
    x = _as(x, np.float32)
    out = np.zeros(x.shape, dtype=np.uint8)
    oracle_lib().pa_fp8_encode(_c(out), _c(x), x.size, int(fmt))
    return out


def attention_fp8(q, k_codes, v_codes, fmt, k_scale, v_scale, block_tables, seq_lens,
                  num_kv_heads, scale, block_size=16, num_blocks=-1, f64=False) -> np.ndarray:
    """Attention over a one-byte KV cache: K = decode(k_codes) * k_scale (V alike),
    Q widened to fp32; then the same oracle as the fp16 / fp32 paths."""
    k = fp8_decode(k_codes, fmt) * np.float32(k_scale)
    v = fp8_decode(v_codes, fmt) * np.float32(v_scale)
    q32 = np.asarray(q, dtype=np.float32)
    return attention(q32, k, v, block_tables, seq_lens, num_kv_heads, scale,
                     block_size=block_size, num_blocks=num_blocks, f64=f64)


def split_partials(q, k, v, block_tables, seq_lens, num_kv_heads, scale, part_pages,
                   max_parts, block_size=16, num_blocks=-1):
    q, k, v, bt, sl, ds = _common(q, k, v, block_tables, seq_lens)
    B, H, D = q.shape
    m = np.zeros((B, H, max_parts), dtype=np.float32)
    l = np.zeros((B, H, max_parts), dtype=np.float32)
    o = np.zeros((B, H, max_parts, D), dtype=np.float32)
    n = oracle_lib().pa_oracle_split_partials(
        _c(m), _c(l), _c(o), _c(q), _c(k), _c(v), _c(bt), _c(sl), B, H, D, num_kv_heads,
        float(scale), bt.shape[1], block_size, ds, num_kv_heads * block_size * D,
        block_size * D, int(num_blocks), part_pages, max_parts)
    if n < 0:
        raise ValueError("oracle rejected the arguments")
    return m, l, o, n


def merge_partials(m, l, o, seq_lens, block_size, part_pages) -> np.ndarray:
    B, H, P = m.shape
    D = o.shape[-1]
    out = np.zeros((B, H, D), dtype=np.float32)
    oracle_lib().pa_oracle_merge_partials(
        _c(out), _c(_as(m, np.float32)), _c(_as(l, np.float32)), _c(_as(o, np.float32)),
        _c(_as(seq_lens, np.int32)), B, H, D, block_size, part_pages, P)
    return out


def reshape_and_cache(key, value, key_cache, value_cache, slots, block_size=16):
    """In-place scatter of key/value [T][Hkv][D] into the pools [NB][Hkv][P][D]."""
    key = np.ascontiguousarray(key)
    value = np.ascontiguousarray(value)
    slots = _as(slots, np.int64)
    T, Hkv, D = key.shape
    assert key_cache.flags.c_contiguous and value_cache.flags.c_contiguous
    oracle_lib().pa_oracle_reshape_and_cache(
        _c(key), _c(value), _c(key_cache), _c(value_cache), _c(slots), T, Hkv, D, block_size,
        key.dtype.itemsize, Hkv * block_size * D, block_size * D, Hkv * D)


def gather_checksum(block_tables, seq_lens, num_heads, num_kv_heads, block_size=16,
                    num_blocks=-1) -> np.ndarray:
    bt, sl = _as(block_tables, np.int32), _as(seq_lens, np.int32)
    out = np.zeros((bt.shape[0], num_heads), dtype=np.uint64)
    rc = oracle_lib().pa_oracle_gather_checksum(_c(out), _c(bt), _c(sl), bt.shape[0], num_heads,
                                                num_kv_heads, bt.shape[1], block_size,
                                                int(num_blocks))
    if rc != 0:
        raise ValueError("oracle rejected the arguments")
    return out


# ── reference CPU path (examples/run_gpt2.c:46-83) ─────────────────────────
def to_run_gpt2_layout(k, v, num_kv_heads, num_heads, block_size=16):
    """Reference-layout pools [NB][Hkv][P][D] -> run_gpt2's [NB][P][Hq][D],
    each KV head repeated for its query heads (kv = h / (Hq/Hkv)), as fp32."""
    nb = k.shape[0]
    D = k.shape[-1]
    group = num_heads // num_kv_heads
    out = []
    for pool in (k, v):
        x = np.asarray(pool, dtype=np.float32).reshape(nb, num_kv_heads, block_size, D)
        x = np.repeat(x, group, axis=1)             # [NB][Hq][P][D]
        out.append(np.ascontiguousarray(x.transpose(0, 2, 1, 3)))  # [NB][P][Hq][D]
    return out[0], out[1]


def per_token_tables(block_tables, seq_lens, block_size=16) -> np.ndarray:
    """run_gpt2's page_table: one entry per token (page of token t)."""
    bt = np.asarray(block_tables, dtype=np.int32)
    T = max(1, bt.shape[1] * block_size)
    t = np.arange(T)
    return np.ascontiguousarray(bt[:, t // block_size], dtype=np.int32)


def reference_attention(q, k_ref, v_ref, page_tables, seq_lens, block_size=16,
                        threads: int = 1) -> np.ndarray:
    """The reference's own paged_attention over a batch (fp32, scale 1/sqrt(D))."""
    q = _as(q, np.float32)
    B, H, D = q.shape
    pt = _as(page_tables, np.int32)
    sl = _as(seq_lens, np.int32)
    out = np.zeros((B, H, D), dtype=np.float32)
    ref_lib().ref_run_gpt2_batch(_c(q), _c(_as(k_ref, np.float32)), _c(_as(v_ref, np.float32)),
                                 _c(pt), _c(sl), B, pt.shape[1], H, D, block_size, _c(out),
                                 int(threads))
    return out


def rel_err_ok(x: np.ndarray, ref: np.ndarray, rtol: float, eps_frac: float = 1e-2) -> tuple:
    """Element-wise |x - ref| <= rtol * max(|ref|, eps) with eps = eps_frac * rms(ref).
    Returns (ok, worst ratio |x-ref| / (rtol*max(|ref|, eps)))."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    eps = max(eps_frac * rms, 1e-30)
    bound = rtol * np.maximum(np.abs(ref), eps)
    ratio = np.abs(x - ref) / bound
    worst = float(ratio.max()) if ratio.size else 0.0
    return bool(np.all(np.isfinite(x)) and worst <= 1.0), worst
