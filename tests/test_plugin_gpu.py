"""The dlopen'd backend plugin, driven as the reference backend manager drives it."""
import ctypes

import pytest

from _helpers import check_close, oracle_out, to_device
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_plugin_init_run_fini(cuda):
    import torch
    b = W.make_batch("plug", [1, 100, 1000], 32, 8, 128, "f16", 61, value_std=0.5)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    plug = PA.CudaBackendPlugin()
    assert plug.backend.state == PA.NXT_BACKEND_STATE_READY
    out = torch.full_like(qt, float("nan"))
    pa = PA.make_input(qt, kt, vt, bt, sl)
    assert plug.run(pa, out) == 0
    torch.cuda.synchronize()
    check_close(out, ref, what="plugin")
    # NULL input / output keep the reference's -1 (backends/cuda_backend.c:72-73)
    lib = _native.plugin()
    assert lib.nxt_backend_run(ctypes.byref(plug.backend), None, out.data_ptr()) == -1
    assert lib.nxt_backend_run(ctypes.byref(plug.backend), ctypes.byref(pa), None) == -1
    # a rejected shape is reported (the reference returns 0 regardless)
    bad = PA.make_input(qt, kt, vt, bt, sl)
    bad.dtype_size = 3
    assert plug.run(bad, out) == -1
    assert plug.close() == 0
    assert plug.backend.state == PA.NXT_BACKEND_STATE_UNINITIALIZED
    assert plug.run(pa, out) == -1  # state freed
    # fini released the library's workspaces and status words: the next
    # backend (and any direct call) allocates them again
    again = PA.CudaBackendPlugin()
    out.fill_(float("nan"))
    assert again.run(pa, out) == 0
    torch.cuda.synchronize()
    check_close(out, ref, what="plugin after fini")
    check_close(PA.paged_attention(qt, kt, vt, bt, sl), ref, what="direct call after fini")
    assert PA.device_status() == 0
    assert again.close() == 0


def test_reference_smoke_calls(cuda):
    """The reference's own GPU smoke calls (tests/test_attention.c:127-287),
    each checked numerically here instead of only for a launch error."""
    import torch
    for hs in (32, 64, 80, 96, 112, 128, 192, 256):
        b = W.make_batch("smoke", [16], 1, 1, hs, "f16", hs)
        q, k, v = b.values_numpy()
        ref = oracle_out(b, q, k, v)
        qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
        out = torch.empty_like(qt)
        PA.nxt_paged_attention(out, qt, kt, vt, bt, sl, 1, 1, hs, 1, 1.0 / hs ** 0.5, 1, 16, 2,
                               16 * hs, 16 * hs)
        torch.cuda.synchronize()
        check_close(out, ref, what=f"v1 hs={hs}")
        b2 = W.make_batch("smoke2", [16], 2, 2, hs, "f16", hs + 1)
        q, k, v = b2.values_numpy()
        ref = oracle_out(b2, q, k, v)
        qt, kt, vt, bt, sl = to_device(b2, q, k, v, cuda)
        out = torch.empty_like(qt)
        PA.nxt_paged_attention_v2(out, qt, kt, vt, bt, sl, 1, 2, hs, 2, 1.0 / hs ** 0.5, 1, 16,
                                  2, 2 * 16 * hs, 16 * hs)
        torch.cuda.synchronize()
        check_close(out, ref, what=f"v2 hs={hs}")
