"""The library's calls captured in a CUDA graph: the kernels of a call (the
attention grid, the split-context merge launched as its programmatic
dependent, the cascade's prefix grid) replay with the same bits as eager
calls, replay after replay. Capture runs on a stream whose library workspace
already exists (a call made on it before capturing), since a workspace cannot
be allocated inside a capture."""
import numpy as np
import pytest

from _helpers import to_device
from oracle import oracle as O
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _capture_and_compare(cuda, call, out):
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        eager = call(side).clone()  # creates this stream's workspace
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        call(side)
    for _ in range(3):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    del graph
    assert PA.device_status() == 0


def test_split_context_call_in_a_graph(cuda):
    import torch
    b = W.make_batch("graph", [9000, 1, 700, 4100, 0, 16], 32, 8, 128, "f16", 71)
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = torch.empty_like(qt)
    _capture_and_compare(cuda, lambda st: PA.paged_attention(qt, kt, vt, bt, sl, out=out,
                                                             stream=st), out)


def test_one_byte_call_in_a_graph(cuda):
    import torch
    b = W.make_batch("graph8", [5000, 33, 2048], 16, 2, 128, "f16", 73)
    q, k, v = b.values_numpy()
    ks = float(np.abs(k.astype(np.float32)).max()) / 448.0
    vs = float(np.abs(v.astype(np.float32)).max()) / 448.0
    k8 = O.fp8_encode(k.astype(np.float32) / np.float32(ks), O.FP8_E4M3)
    v8 = O.fp8_encode(v.astype(np.float32) / np.float32(vs), O.FP8_E4M3)
    qt, k8t, v8t = (torch.from_numpy(x).to(cuda) for x in (q, k8, v8))
    bt, sl = b.tables_torch(cuda)
    out = torch.empty_like(qt)
    _capture_and_compare(cuda, lambda st: PA.paged_attention_fp8(
        qt, k8t, v8t, bt, sl, "e4m3", ks, vs, scale=b.scale, out=out, stream=st), out)


def test_cascade_call_in_a_graph(cuda):
    import torch
    rng = np.random.default_rng(29)
    members = [6, 3]
    prefix = [1024, 128]
    prefix_of = [g for g, n in enumerate(members) for _ in range(n)] + [-1]
    suffix = rng.integers(0, 400, size=len(prefix_of))
    lens = [(prefix[g] if g >= 0 else 0) + int(s) for g, s in zip(prefix_of, suffix)]
    b = W.make_batch("graphpfx", lens, 16, 4, 128, "f16", 31, prefix=prefix,
                     prefix_of=prefix_of)
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    groups = PA.PrefixGroups(b.prefix_groups, b.num_seqs, cuda)  # device arrays, made once
    out = torch.empty_like(qt)
    _capture_and_compare(cuda, lambda st: PA.paged_attention_prefix(
        qt, kt, vt, bt, sl, groups, out=out, stream=st), out)
