"""Activation kernels (xllms_b200/csrc/pa_act.cu) on the GPU: bit-exact
against the reference's own kernels (operators/activation_kernels.cu, built by
oracle/Makefile) and within rounding of the CPU oracle."""
import numpy as np
import pytest

from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import operator_api as PA

pytestmark = pytest.mark.gpu

NAMES = list(PA.ACTIVATIONS)
SHAPES = [(1, 8), (3, 7), (64, 4096), (257, 14336 // 8), (5, 1000), (2, 1)]


def _input(op, rows, d, dtype, seed):
    rng = np.random.default_rng([seed, op, rows, d])
    x = rng.standard_normal((rows, 2 * d if op <= 3 else d)).astype(np.float32) * 4
    x[:, :3] = np.array([0.0, 30.0, -30.0], dtype=np.float32)[: min(3, x.shape[1])]
    return x.astype(dtype)


def _ulp_close(got, ref, dtype, x, op):
    """|got - ref| within a few ulps of the result, plus a few fp32 ulps of
    the operands' product: libm's and CUDA's expf / erff / tanhf may differ
    by an ulp, and x (1 + erf(x)) or x (1 + tanh(.)) cancels for negative x,
    which turns that ulp into a larger relative error of a small result."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    x = x.astype(np.float64)
    d = ref.shape[1]
    mag = np.abs(x[:, :d] * x[:, d:]) if op <= 3 else np.abs(x)
    if dtype == np.float32:
        tol = 4 * np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64) + 1e-38
    else:
        tol = 2 * np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64) + 6e-8
    tol += 4 * 2.0 ** -24 * mag
    return float(np.max(np.abs(got - ref) - tol, initial=-1.0)) <= 0.0


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("shape", SHAPES)
def test_matches_oracle(cuda, name, dtype, shape):
    import torch
    op = PA.ACTIVATIONS[name]
    rows, d = shape
    x = _input(op, rows, d, dtype, 1)
    out = PA.activation(name, torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert _ulp_close(out, O.activation(op, x), dtype, x, op), name


@pytest.mark.skipif(not O.ref_act_available(), reason="reference kernels not built")
@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("shape", SHAPES)
def test_bit_exact_vs_reference_kernels(cuda, name, dtype, shape):
    import torch
    op = PA.ACTIVATIONS[name]
    rows, d = shape
    x = torch.from_numpy(_input(op, rows, d, dtype, 2)).to(cuda)
    ours = PA.activation(name, x)
    ref = torch.empty_like(ours)
    rc = O.ref_act_lib().ref_activation(op, ref.data_ptr(), x.data_ptr(), rows, d,
                                        x.element_size(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16 if dtype == np.float16 else torch.int32),
                       ref.view(torch.int16 if dtype == np.float16 else torch.int32)), name


def test_dropin_entry_points(cuda):
    import torch
    lib = _native.xpa()
    x = torch.randn(16, 2 * 256, device=cuda, dtype=torch.float16)
    for name, fn in [("silu_and_mul", lib.nxt_silu_and_mul), ("mul_and_silu", lib.nxt_mul_and_silu),
                     ("gelu_and_mul", lib.nxt_gelu_and_mul),
                     ("gelu_tanh_and_mul", lib.nxt_gelu_tanh_and_mul)]:
        out = torch.empty(16, 256, device=cuda, dtype=torch.float16)
        fn(out.data_ptr(), x.data_ptr(), 16, 256, 2, None)
        assert lib.nxt_activation_last_error() == 0
        assert torch.equal(out, PA.activation(name, x))
    for name, fn in [("gelu", lib.nxt_gelu_elementwise), ("silu", lib.nxt_silu_elementwise)]:
        out = torch.empty_like(x)
        fn(out.data_ptr(), x.data_ptr(), 16, 512, 2, None)
        assert lib.nxt_activation_last_error() == 0
        assert torch.equal(out, PA.activation(name, x))


def test_unaligned_rows_take_the_scalar_path(cuda):
    import torch
    op = PA.ACTIVATIONS["silu_and_mul"]
    base = torch.from_numpy(_input(op, 9, 16, np.float16, 3).reshape(-1)).to(cuda)
    buf = torch.empty(base.numel() + 1, dtype=torch.float16, device=cuda)
    buf[1:] = base
    x = buf[1:].view(9, 32)  # 2-byte aligned: no 16-byte vectors
    out = PA.activation("silu_and_mul", x)
    xs = base.cpu().numpy().reshape(9, 32)
    assert _ulp_close(out.cpu().numpy(), O.activation(op, xs), np.float16, xs, op)
