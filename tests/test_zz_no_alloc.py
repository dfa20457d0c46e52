"""nxt_paged_attention_noalloc: decode attention for callers that cannot
allocate device memory.

A serving engine that has reserved nearly all of HBM for its KV page pool, or
a host that routes every device allocation through its own pool, cannot let a
library call cudaMalloc (and cudaMalloc/cudaFree would synchronise the device
in the middle of the decode loop). This entry point keeps its split-context
partials in a fixed array compiled into the library. It is checked here
through the C ABI against the regular entry point and against the CPU oracle,
on two calls in a row. This file is collected last on purpose.
"""
import numpy as np
import pytest

from _helpers import check_close, oracle_out, to_device
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _noalloc(b, qt, kt, vt, bt, sl, out, status=None, max_blocks=None):
    import torch
    return _native.xpa().nxt_paged_attention_noalloc(
        out.data_ptr(), qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), bt.data_ptr(),
        sl.data_ptr(), b.num_seqs, b.num_heads, b.head_size, b.num_kv_heads, b.scale,
        b.max_blocks if max_blocks is None else max_blocks, b.block_size, b.dtype_size,
        b.kv_block_stride, b.kv_head_stride, b.num_blocks,
        None if status is None else status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


CASES = {
    # fp16 GQA, TMA + tensor-core kernel, sequences split into many partitions
    "fast_fp16": lambda: W.make_batch("na16", [3000, 700, 1, 5000], 32, 8, 128, "f16", 91,
                                      value_std=0.5),
    # fp32 MHA, CUDA-core kernel, split as well
    "generic_fp32": lambda: W.make_batch("na32", [2000, 33], 12, 12, 64, "f32", 92),
    # odd head size, odd query heads, odd partition count: the (max, sum)
    # pairs still start on an aligned boundary of the scratch
    "generic_odd_d": lambda: W.make_batch("na33", [5000, 3, 2049], 3, 1, 33, "f16", 94),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_matches_regular_entry_point_on_two_calls(cuda, case):
    import torch
    b = CASES[case]()
    need = PA.workspace_size(b.num_seqs, b.num_heads, b.head_size, b.num_kv_heads,
                             b.max_blocks, b.block_size, b.dtype_size)
    assert 0 < need <= _native.NXT_PA_NOALLOC_SCRATCH_BYTES  # the case uses the scratch
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    regular = PA.paged_attention(qt, kt, vt, bt, sl, num_blocks=b.num_blocks)
    torch.cuda.synchronize()
    expect = regular.float().cpu().numpy()
    ref = oracle_out(b, q, k, v, f64=True)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in range(2):
        out = torch.full_like(qt, float("nan"))
        assert _noalloc(b, qt, kt, vt, bt, sl, out, status) == _native.NXT_PA_OK
        torch.cuda.synchronize()
        check_close(out, expect, what=f"{case} call {call + 1} vs regular entry point")
        check_close(out, ref, what=f"{case} call {call + 1} vs oracle")
    assert int(status.item()) == 0


def test_noalloc_follows_the_wait_budget(cuda):
    """The thread's wait budget bounds this entry point's pipeline waits too:
    a zero budget makes them run out (NXT_PA_DEV_TIMEOUT in the caller's
    status word, no fault), and the next call with the budget restored is
    correct again."""
    import torch
    lib = _native.xpa()
    b = CASES["fast_fp16"]()
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    assert PA.kernel_path(kt, vt, b.num_heads, b.head_size, b.num_kv_heads, b.block_size,
                          b.dtype_size, b.kv_block_stride,
                          b.kv_head_stride) == _native.NXT_PA_PATH_TMA_MMA
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty_like(qt)
    prev = lib.nxt_paged_attention_set_wait_budget_ns(0)
    try:
        assert _noalloc(b, qt, kt, vt, bt, sl, out, status) == _native.NXT_PA_OK
        torch.cuda.synchronize()
    finally:
        lib.nxt_paged_attention_set_wait_budget_ns(prev)
    assert int(status.item()) & _native.NXT_PA_DEV_TIMEOUT
    status.zero_()
    ref = oracle_out(b, q, k, v, f64=True)
    for _ in range(2):
        assert _noalloc(b, qt, kt, vt, bt, sl, out, status) == _native.NXT_PA_OK
        torch.cuda.synchronize()
        check_close(out, ref, what="after timeout")
    assert int(status.item()) == 0


def test_noalloc_calls_allocate_nothing(cuda):
    import torch
    b = CASES["fast_fp16"]()
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    outs = [torch.empty_like(qt) for _ in range(3)]
    assert _noalloc(b, qt, kt, vt, bt, sl, outs[0]) == 0  # first call on the device: set-up
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for out in outs[1:]:
        assert _noalloc(b, qt, kt, vt, bt, sl, out) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert torch.equal(outs[1], outs[2])


def test_noalloc_rejects_requests_beyond_its_scratch(cuda):
    import torch
    # Llama-3-70B long-context shape with 64 sequences of 8192-page rows: ~136 MB of partials.
    b = W.make_batch("big", [16] * 64, 64, 8, 128, "f16", 93, max_blocks=8192)
    need = PA.workspace_size(64, 64, 128, 8, 8192, 16, 2)
    assert need > _native.NXT_PA_NOALLOC_SCRATCH_BYTES
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = torch.full_like(qt, 7.0)
    rc = _noalloc(b, qt, kt, vt, bt, sl, out)
    torch.cuda.synchronize()
    assert rc == _native.NXT_PA_ESCRATCH
    assert "scratch" in _native.strerror(rc)
    assert bool((out == 7.0).all())  # nothing was launched
