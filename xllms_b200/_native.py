"""Loads the in-tree native libraries built from xllms_b200/csrc.

``libxpa.so`` carries the sm_100a kernels behind the C ABI of
include/operator_api.h; ``libxllm_cuda_backend.so`` is the dlopen'd backend
plugin of include/cuda_backend.h. There is no fallback: when a library is
missing, every entry point raises :class:`NativeLibraryMissing`.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
XPA_PATH = os.path.join(LIB_DIR, "libxpa.so")
PLUGIN_PATH = os.path.join(LIB_DIR, "libxllm_cuda_backend.so")

# Status codes and device status bits (include/operator_api.h).
NXT_PA_OK = 0
NXT_PA_EINVAL = -22
NXT_PA_ENOMEM = -12
NXT_PA_EWORKSPACE = -28
NXT_PA_ECUDA = -5
NXT_PA_ESCRATCH = -27
NXT_PA_NOALLOC_SCRATCH_BYTES = 32 << 20
NXT_PA_DEV_TIMEOUT = 0x1
NXT_PA_DEV_BAD_PAGE = 0x2
NXT_PA_DEV_SEQ_CLAMPED = 0x4
NXT_PA_PATH_NONE = 0
NXT_PA_PATH_TMA_MMA = 1
NXT_PA_PATH_GENERIC = 2
NXT_BT_TABLES = 0
NXT_BT_SEQ_LENS = 1
NXT_BT_SLOTS = 2
NXT_BT_PREFIX_PAGES = 3
NXT_BT_GROUP_OFFSETS = 4
NXT_BT_GROUP_MEMBERS = 5
NXT_BT_NUM_ARRAYS = 6
NXT_KV_FP8_E4M3 = 1
NXT_KV_FP8_E5M2 = 2
NXT_KV_INT8 = 3
NXT_ACT_SILU_AND_MUL = 0
NXT_ACT_MUL_AND_SILU = 1
NXT_ACT_GELU_AND_MUL = 2
NXT_ACT_GELU_TANH_AND_MUL = 3
NXT_ACT_GELU = 4
NXT_ACT_SILU = 5
NXT_PA_MAX_PEERS = 8
NXT_PA_IPC_HANDLE_BYTES = 64

# Every function include/operator_api.h declares, with its ctypes signature.
_VP, _CVP, _IP = ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p
_I, _F, _I64, _SZ = ctypes.c_int, ctypes.c_float, ctypes.c_int64, ctypes.c_size_t
_DROPIN_ARGS = [_VP, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _I, _I, _VP]
SIGNATURES = {
    "nxt_paged_attention": (None, _DROPIN_ARGS),
    "nxt_paged_attention_v2": (None, _DROPIN_ARGS),
    "nxt_paged_attention_flash": (None, _DROPIN_ARGS),
    "nxt_paged_attention_last_error": (_I, []),
    "nxt_paged_attention_strerror": (ctypes.c_char_p, [_I]),
    "nxt_paged_attention_ex": (
        _I,
        [_VP, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _I64, _I64, _I64,
         _VP, _SZ, _VP, _VP],
    ),
    "nxt_paged_attention_workspace_size": (_SZ, [_I, _I, _I, _I, _I, _I, _I]),
    "nxt_paged_attention_path": (_I, [_CVP, _CVP, _I, _I, _I, _I, _I, _I64, _I64]),
    "nxt_paged_attention_device_status": (_I, [_I]),
    "nxt_paged_attention_release_workspaces": (_I, []),
    "nxt_paged_attention_noalloc": (
        _I,
        [_VP, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _I64, _I64, _I64,
         _VP, _VP],
    ),
    "nxt_paged_attention_profile_next": (_I, [_VP, _VP]),
    "nxt_paged_attention_profile_next_ex": (_I, [_VP, _VP, _VP]),
    "nxt_block_tables_layout": (_SZ, [_I, _I, _I, _VP]),
    "nxt_block_tables_staging_size": (_SZ, [_I, _I]),
    "nxt_build_block_tables": (
        _I, [_IP, _IP, _IP, _IP, _IP, _I, _I, _I, _VP, _SZ, _VP, _SZ, _IP, _IP, _IP, _VP]),
    "nxt_silu_and_mul": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_mul_and_silu": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_gelu_and_mul": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_gelu_tanh_and_mul": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_gelu_elementwise": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_silu_elementwise": (None, [_VP, _CVP, _I, _I, _I, _VP]),
    "nxt_activation_ex": (_I, [_I, _VP, _CVP, _I, _I, _I, _VP]),
    "nxt_activation_last_error": (_I, []),
    "nxt_paged_attention_prefix_ex": (
        _I,
        [_VP, _CVP, _CVP, _CVP, _IP, _IP, _IP, _IP, _IP, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
         _I, _I64, _I64, _I64, _VP, _SZ, _VP, _VP],
    ),
    "nxt_paged_attention_prefix_workspace_size": (_SZ, [_I, _I, _I, _I, _I, _I, _I]),
    "nxt_paged_attention_fp8_ex": (
        _I,
        [_VP, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _F, _F, _I64, _I64,
         _I64, _VP, _SZ, _VP, _VP]),
    "nxt_paged_attention_fp8_workspace_size": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "nxt_reshape_and_cache_fp8": (
        _I, [_CVP, _CVP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _F, _F, _I64, _I64, _I64, _VP]),
    "nxt_paged_attention_fp8_append_ex": (
        _I,
        [_VP, _CVP, _VP, _VP, _IP, _IP, _CVP, _CVP, _VP, _I, _I, _I, _I, _F, _I, _I, _I, _F, _F,
         _I64, _I64, _I64, _VP, _VP],
    ),
    "nxt_reshape_and_cache": (
        _I, [_CVP, _CVP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I64, _I64, _I64, _VP]),
    "nxt_paged_attention_append_ex": (
        _I,
        [_VP, _CVP, _VP, _VP, _IP, _IP, _CVP, _CVP, _VP, _I, _I, _I, _I, _F, _I, _I, _I, _I64,
         _I64, _I64, _VP, _VP],
    ),
    "nxt_pa_peer_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _VP]),
    "nxt_pa_peer_open": (_I, [_VP, ctypes.POINTER(ctypes.c_void_p)]),
    "nxt_pa_peer_close": (_I, [_VP]),
    "nxt_pa_peer_free": (_I, [_VP]),
    "nxt_paged_attention_sharded": (
        _I,
        [_VP, ctypes.c_uint64, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _I64,
         _I64, _I64, _VP, _VP],
    ),
    "nxt_paged_attention_fp8_sharded": (
        _I,
        [_VP, ctypes.c_uint64, _CVP, _CVP, _CVP, _IP, _IP, _I, _I, _I, _I, _F, _I, _I, _I, _F, _F,
         _I64, _I64, _I64, _VP, _VP],
    ),
    "nxt_paged_attention_set_wait_budget_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "nxt_paged_attention_device_info": (
        _I, [ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.c_char_p, _I]),
}
PLUGIN_SIGNATURES = {
    "nxt_backend_init": (_I, [_VP]),
    "nxt_backend_run": (_I, [_VP, _VP, _VP]),
    "nxt_backend_fini": (_I, [_VP]),
}


class NativeLibraryMissing(RuntimeError):
    """A native library of this package was not built or cannot be loaded."""


_lock = threading.Lock()
_xpa = None
_plugin = None


def _load(path: str, sigs: dict) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise NativeLibraryMissing(
            f"{os.path.basename(path)} not found in {LIB_DIR}; build it with "
            "`make -C xllms_b200/csrc` (or __graft_entry__.build())")
    try:
        lib = ctypes.CDLL(path)
    except OSError as exc:  # pragma: no cover - depends on the host
        raise NativeLibraryMissing(f"cannot load {path}: {exc}") from exc
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def xpa() -> ctypes.CDLL:
    """The kernel library (libxpa.so)."""
    global _xpa
    with _lock:
        if _xpa is None:
            _xpa = _load(XPA_PATH, SIGNATURES)
        return _xpa


def plugin() -> ctypes.CDLL:
    """The backend plugin (libxllm_cuda_backend.so), loaded like the xLLMs
    backend manager loads it (dlopen, then the three entry points by name)."""
    global _plugin
    with _lock:
        if _plugin is None:
            _plugin = _load(PLUGIN_PATH, PLUGIN_SIGNATURES)
        return _plugin


def strerror(code: int) -> str:
    return xpa().nxt_paged_attention_strerror(code).decode()
