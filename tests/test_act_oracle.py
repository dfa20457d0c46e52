"""The activation oracle (oracle/act_oracle.c) against float64 restatements of
the reference's formulas (operators/activation_kernels.cu:25-50), and the C
ABI's argument checks (no GPU work)."""
import math

import numpy as np
import pytest

from oracle import oracle as O
from xllms_b200 import _native


def _f64(op, g, u):
    g = g.astype(np.float64)
    u = u.astype(np.float64)
    silu = lambda x: x / (1.0 + np.exp(-x))
    erf = np.vectorize(math.erf)
    gelu = lambda x: 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))
    gelu_t = lambda x: 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))
    return {0: silu(g) * u, 1: g * silu(u), 2: gelu(g) * u, 3: gelu_t(g) * u,
            4: gelu(g), 5: silu(g)}[op]


@pytest.mark.parametrize("op", range(6))
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_oracle_matches_float64(op, dtype):
    rng = np.random.default_rng(op)
    d, rows = 37, 11
    x = (rng.standard_normal((rows, 2 * d if op <= 3 else d)) * 3).astype(dtype)
    got = O.activation(op, x).astype(np.float64)
    g, u = (x[:, :d], x[:, d:]) if op <= 3 else (x, x)
    ref = _f64(op, g, u)
    # fp32: a few ulp; fp16: the activation and the product are each rounded once
    rtol = 1e-6 if dtype == np.float32 else 2 ** -10
    assert np.allclose(got, ref, rtol=rtol, atol=1e-6 if dtype == np.float32 else 1e-4)


def test_oracle_extremes():
    x = np.array([[0.0, -0.0, 80.0, -80.0, 1e-30, -1e-30, 30.0, -30.0]], dtype=np.float32)
    silu = O.activation(5, x)[0]
    assert silu[0] == 0.0 and silu[2] == 80.0 and abs(silu[3]) < 1e-30
    gelu = O.activation(4, x)[0]
    assert gelu[2] == 80.0 and gelu[3] == 0.0


def test_abi_argument_checks_without_gpu():
    lib = _native.xpa()
    ok, einval = _native.NXT_PA_OK, _native.NXT_PA_EINVAL
    # nothing to do: no device work, OK
    assert lib.nxt_activation_ex(0, None, None, 0, 16, 2, None) == ok
    assert lib.nxt_activation_ex(9, None, None, 1, 16, 2, None) == einval   # unknown op
    assert lib.nxt_activation_ex(0, None, None, 1, 0, 2, None) == einval    # d <= 0
    assert lib.nxt_activation_ex(0, None, None, -1, 16, 2, None) == einval  # num_tokens < 0
    assert lib.nxt_activation_ex(0, None, None, 1, 16, 3, None) == einval   # dtype
    assert lib.nxt_activation_ex(0, None, None, 1, 16, 2, None) == einval   # NULL buffers
    lib.nxt_silu_and_mul(None, None, 1, 16, 8, None)
    assert lib.nxt_activation_last_error() == einval
    lib.nxt_gelu_elementwise(None, None, 0, 16, 2, None)
    assert lib.nxt_activation_last_error() == ok
