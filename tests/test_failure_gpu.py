"""Failure detection on the GPU without faulting it: the kernels' bounded
pipeline waits are made to run out (a tiny wait budget), the device status
word reports NXT_PA_DEV_TIMEOUT, and the same context then computes correct
results again (the split-context counters are back at zero)."""
import pytest

from _helpers import check_close, oracle_out, to_device
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_stays_usable(cuda):
    import torch
    lib = _native.xpa()
    b = W.make_batch("timeout", [4000, 1500, 300, 9000, 2048, 17], 32, 8, 128, "f16", 71,
                     value_std=0.5)
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    assert PA.kernel_path(kt, vt, 32, 128, 8, 16, 2, b.kv_block_stride,
                          b.kv_head_stride) == _native.NXT_PA_PATH_TMA_MMA
    PA.device_status(clear=True)
    prev = lib.nxt_paged_attention_set_wait_budget_ns(0)
    try:
        PA.paged_attention(qt, kt, vt, bt, sl)
        torch.cuda.synchronize()
    finally:
        lib.nxt_paged_attention_set_wait_budget_ns(prev)
    assert PA.device_status(clear=True) & _native.NXT_PA_DEV_TIMEOUT
    for _ in range(2):
        out = PA.paged_attention(qt, kt, vt, bt, sl)
        torch.cuda.synchronize()
        check_close(out, ref, what="after timeout")
        assert PA.device_status(clear=True) == 0
