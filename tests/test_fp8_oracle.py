"""One-byte KV codecs of the oracle (fp8 pinned against torch's float8
types, int8 against torch's round-half-even and clamp), and the one-byte
C-ABI argument checks (no GPU work)."""
import numpy as np
import pytest

from oracle import oracle as O
from xllms_b200 import _native

torch = pytest.importorskip("torch")
FORMATS = [(O.FP8_E4M3, torch.float8_e4m3fn, 448.0), (O.FP8_E5M2, torch.float8_e5m2, 57344.0)]


@pytest.mark.parametrize("fmt,tdtype,fmax", FORMATS)
def test_decode_all_codes_match_torch(fmt, tdtype, fmax):
    codes = np.arange(256, dtype=np.uint8)
    got = O.fp8_decode(codes, fmt)
    ref = torch.from_numpy(codes.copy()).view(tdtype).float().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(got[fin], ref[fin])
    assert np.nanmax(got[np.isfinite(got)]) == fmax


@pytest.mark.parametrize("fmt,tdtype,fmax", FORMATS)
def test_encode_matches_torch_in_range(fmt, tdtype, fmax):
    rng = np.random.default_rng(fmt)
    x = np.concatenate([rng.standard_normal(100000) * (fmax / 10),
                        rng.standard_normal(100000) * 1e-3,
                        np.ldexp(rng.random(20000), rng.integers(-30, 5, 20000))]).astype(np.float32)
    x = x[np.abs(x) <= fmax]
    ref = torch.from_numpy(x).to(tdtype).view(torch.uint8).numpy()
    assert np.array_equal(O.fp8_encode(x, fmt), ref)


@pytest.mark.parametrize("fmt,tdtype,fmax", FORMATS)
def test_encode_round_trip_and_saturation(fmt, tdtype, fmax):
    codes = np.arange(256, dtype=np.uint8)
    vals = O.fp8_decode(codes, fmt)
    ok = np.isfinite(vals)
    assert np.array_equal(O.fp8_encode(vals[ok], fmt), codes[ok])  # every finite code round-trips
    big = np.array([fmax * 4, -fmax * 4, np.inf, -np.inf], dtype=np.float32)
    assert np.array_equal(O.fp8_decode(O.fp8_encode(big, fmt), fmt), [fmax, -fmax, fmax, -fmax])
    assert np.isnan(O.fp8_decode(O.fp8_encode(np.array([np.nan], np.float32), fmt), fmt))[0]


def test_encode_ties_to_even():
    # 1 + 1/16 lies halfway between E4M3's 1 (mantissa 000) and 1.125 (001): even wins
    assert O.fp8_decode(O.fp8_encode(np.array([1.0625, 1.1875], np.float32), 1), 1).tolist() == \
        [1.0, 1.25]


def test_fp8_abi_argument_checks_without_gpu():
    lib = _native.xpa()
    einval = _native.NXT_PA_EINVAL
    buf = np.zeros(64, dtype=np.uint8)
    p = buf.ctypes.data
    bt = np.zeros(4, dtype=np.int32)
    sl = np.ones(1, dtype=np.int32)
    args = lambda fmt, ks, vs: (p, p, p, p, bt.ctypes.data, sl.ctypes.data, 1, 1, 16, 1, 1.0,
                                1, 16, fmt, ks, vs, 256, 256, 1, None, 0, None, None)
    assert lib.nxt_paged_attention_fp8_ex(*args(4, 1.0, 1.0)) == einval   # format
    assert lib.nxt_paged_attention_fp8_ex(*args(0, 1.0, 1.0)) == einval
    assert lib.nxt_paged_attention_fp8_ex(*args(1, 0.0, 1.0)) == einval   # scale
    assert lib.nxt_paged_attention_fp8_ex(*args(1, 1.0, float("nan"))) == einval
    sm = np.zeros(1, dtype=np.int64)
    assert lib.nxt_reshape_and_cache_fp8(p, p, p, p, sm.ctypes.data, 1, 1, 16, 16, 7, 1.0, 1.0,
                                         256, 256, 16, None) == einval
    assert lib.nxt_reshape_and_cache_fp8(p, p, p, p, sm.ctypes.data, 1, 1, 16, 16, 1, -1.0, 1.0,
                                         256, 256, 16, None) == einval
    assert lib.nxt_reshape_and_cache_fp8(None, None, None, None, None, 0, 1, 16, 16, 1, 1.0, 1.0,
                                         256, 256, 16, None) == _native.NXT_PA_OK


def test_int8_codec():
    codes = np.arange(256, dtype=np.uint8)
    assert np.array_equal(O.fp8_decode(codes, O.KV_INT8), codes.view(np.int8).astype(np.float32))
    assert np.array_equal(O.fp8_encode(O.fp8_decode(codes, O.KV_INT8), O.KV_INT8), codes)
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(200000) * 60).astype(np.float32)
    ref = torch.from_numpy(x).round().clamp(-128, 127).to(torch.int8).view(torch.uint8).numpy()
    assert np.array_equal(O.fp8_encode(x, O.KV_INT8), ref)
    ties = np.array([0.5, 1.5, 2.5, -0.5, -1.5, 126.5, -127.5, 127.5, -128.5], np.float32)
    assert O.fp8_decode(O.fp8_encode(ties, O.KV_INT8), O.KV_INT8).tolist() == \
        [0, 2, 2, 0, -2, 126, -128, 127, -128]
    odd = np.array([np.nan, np.inf, -np.inf, 1e30, -1e30, -0.0], np.float32)
    assert O.fp8_decode(O.fp8_encode(odd, O.KV_INT8), O.KV_INT8).tolist() == \
        [0, 127, -128, 127, -128, 0]


def test_fp8_append_step_argument_checks_without_gpu():
    lib = _native.xpa()
    buf = np.zeros(64, dtype=np.uint8)
    p = buf.ctypes.data
    bt = np.zeros(4, dtype=np.int32)
    sl = np.ones(1, dtype=np.int32)
    sm = np.zeros(1, dtype=np.int64)
    args = lambda B, fmt, ks: (p, p, p, p, bt.ctypes.data, sl.ctypes.data, p, p, sm.ctypes.data,
                               B, 1, 16, 1, 1.0, 1, 16, fmt, ks, 1.0, 256, 256, 1, None, None)
    assert lib.nxt_paged_attention_fp8_append_ex(*args(1, 5, 1.0)) == _native.NXT_PA_EINVAL
    assert lib.nxt_paged_attention_fp8_append_ex(*args(1, 3, 0.0)) == _native.NXT_PA_EINVAL
    assert lib.nxt_paged_attention_fp8_append_ex(*args(0, 3, 1.0)) == _native.NXT_PA_OK
