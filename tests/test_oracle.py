"""The CPU oracle pinned against the reference's own CPU attention, its golden
fixtures and a pure-Python restatement (CPU only)."""
import glob
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O
from xllms_b200 import workloads as W

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


def _load_golden(path):
    import sys
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_golden
    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    return make_golden, meta, z["out"]


def py_attention(q, k, v, bt, sl, hkv, scale, bs=16, num_blocks=-1):
    """Pure-Python loops, small cases only: examples/text_gen.c:1284-1309 over
    the paged layout, masked pages excluded."""
    B, H, D = q.shape
    g = H // hkv
    out = np.zeros((B, H, D), dtype=np.float64)
    for b in range(B):
        L = max(0, min(int(sl[b]), bt.shape[1] * bs))
        for h in range(H):
            kh = h // g
            sc = []
            for t in range(L):
                phys = int(bt[b, t // bs])
                if phys < 0 or (num_blocks > 0 and phys >= num_blocks):
                    continue
                kr = k[phys, kh, t % bs].astype(np.float64)
                sc.append((sum(float(q[b, h, d]) * kr[d] for d in range(D)) * scale, phys, t % bs))
            if not sc:
                continue
            mx = max(s for s, _, _ in sc)
            e = [math.exp(s - mx) for s, _, _ in sc]
            tot = sum(e)
            for w, (_, phys, slot) in zip(e, sc):
                out[b, h] += (w / tot) * v[phys, kh, slot].astype(np.float64)
    return out


def test_half_conversions_match_ieee():
    lib = O.oracle_lib()
    bits = np.arange(0, 65536, 97, dtype=np.uint16)
    f = bits.view(np.float16).astype(np.float32)
    for b_, x in zip(bits, f):
        y = lib.pa_half_to_float(int(b_))
        assert (np.isnan(x) and np.isnan(y)) or y == x
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                         np.float32([0, -0.0, 65504, 65519, 65520, 1e-8, 5.96e-8, 6.1e-5,
                                     2.98e-8, np.inf, -np.inf])])
    for x in xs:
        assert lib.pa_float_to_half(float(x)) == int(np.float32(x).astype(np.float16).view(np.uint16))


@pytest.mark.skipif(not O.ref_available(), reason="reference CPU path not built")
@pytest.mark.parametrize("make", [
    lambda: W.config1(),
    lambda: W.make_batch("gqa", [1, 15, 16, 17, 100, 513], 8, 2, 128, "f16", 5),
    lambda: W.make_batch("gqa16", [40, 3], 16, 1, 64, "f32", 6),
    lambda: W.config4(num_seqs=4),
])
def test_oracle_matches_reference_cpu_path(make):
    """Against the reference's paged_attention (examples/run_gpt2.c:46-83) run
    on the same inputs (GQA realised by repeating each KV head for its group)."""
    b = make()
    q, k, v = b.values_numpy()
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, b.num_kv_heads, b.scale)
    kr, vr = O.to_run_gpt2_layout(k, v, b.num_kv_heads, b.num_heads)
    r = O.reference_attention(q.astype(np.float32), kr, vr,
                              O.per_token_tables(b.block_tables, b.seq_lens), b.seq_lens)
    # Both are fp32 accumulations over up to ~3000 tokens (the reference without
    # max subtraction); against an fp64 evaluation each is within ~2e-4, so
    # they are held to the north_star tolerance of 1e-3.
    ok, worst = O.rel_err_ok(o, r, 1e-3)
    assert ok, worst


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_reproduces_golden_fixtures(path):
    mg, meta, ref_out = _load_golden(path)
    b = mg.build_case(meta["spec"])
    q, k, v = b.values_numpy()
    assert mg.input_digest(b, q, k, v) == meta["inputs_sha256"], "input generator drifted"
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, b.num_kv_heads, b.scale)
    ok, worst = O.rel_err_ok(o, ref_out, 1e-3)
    assert ok, worst


def test_golden_fixtures_present():
    names = {os.path.basename(p) for p in GOLDEN}
    assert {"c1_gpt2_small_fp32.npz", "gqa4_fp16_edges.npz", "prefix_shared_fp16.npz"} <= names


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_matches_python_loops(seed):
    b = W.make_batch("py", [0, 1, 9, 16, 17, 40], 4, 2, 16, "f16", seed, block_size=8)
    b.block_tables[4, 1] = -1  # a masked page inside sequence 4
    q, k, v = b.values_numpy()
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, block_size=8)
    p = py_attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, bs=8)
    assert np.allclose(o, p, rtol=1e-5, atol=1e-6)
    lim = int(b.block_tables[5, 2])
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, block_size=8,
                    num_blocks=lim)
    p = py_attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, bs=8, num_blocks=lim)
    assert np.allclose(o, p, rtol=1e-5, atol=1e-6)


def test_fp64_twin_bounds_fp32_oracle():
    b = W.make_batch("f", [3000, 17], 16, 2, 128, "f16", 9)
    q, k, v = b.values_numpy()
    o32 = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale)
    o64 = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, f64=True)
    # the fp32 oracle spends at most half of the 1e-3 budget
    ok, worst = O.rel_err_ok(o32, o64, 1e-3)
    assert ok and worst < 0.5, worst


def test_split_partials_merge_to_direct_result():
    b = W.make_batch("sp", [0, 5, 512, 513, 2000], 8, 2, 64, "f16", 12)
    q, k, v = b.values_numpy()
    direct = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale)
    for pp in (1, 4, 32):
        mp = -(-b.max_blocks // pp)
        m, l, o, n = O.split_partials(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, pp, mp)
        assert n == -(-(-(-2000 // 16)) // pp)
        merged = O.merge_partials(m, l, o, b.seq_lens, 16, pp)
        assert np.allclose(merged, direct, rtol=2e-5, atol=2e-6)


def test_empty_and_zero_inputs():
    b = W.make_batch("z", [0, 32], 4, 2, 64, "f32", 1)
    q, k, v = b.values_numpy()
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale)
    assert not o[0].any()
    z = O.attention(np.zeros_like(q), np.zeros_like(k), np.zeros_like(v), b.block_tables,
                    b.seq_lens, 2, b.scale)
    assert not z.any()


def test_seq_len_clamped_to_block_table_row():
    b = W.make_batch("c", [64], 4, 2, 64, "f32", 1, max_blocks=4)
    q, k, v = b.values_numpy()
    o = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale)
    sl = b.seq_lens.copy()
    sl[0] = 999
    o2 = O.attention(q, k, v, b.block_tables, sl, 2, b.scale)
    assert np.array_equal(o, o2)


def test_gather_checksum_matches_python():
    b = W.config4(num_seqs=6)
    b.block_tables[2, 5] = -7
    cs = O.gather_checksum(b.block_tables, b.seq_lens, b.num_heads, b.num_kv_heads)
    lib = O.oracle_lib()
    g = b.num_heads // b.num_kv_heads
    for s in range(b.num_seqs):
        for h in range(0, b.num_heads, 5):
            acc = 0
            for t in range(int(b.seq_lens[s])):
                phys = int(b.block_tables[s, t // 16])
                if phys < 0:
                    continue
                acc = (acc + lib.pa_gather_mix(phys, t % 16, h // g)) % (1 << 64)
            assert int(cs[s, h]) == acc


@pytest.mark.parametrize("head_size,dtype,group,block_size,fmt", [
    (128, "f16", 4, 16, 0), (64, "f32", 1, 16, 0), (128, "f16", 4, 32, 0),
    (64, "f16", 4, 16, O.KV_INT8), (64, "f16", 4, 16, O.FP8_E4M3)])
def test_oracle_index_logic_exact(head_size, dtype, group, block_size, fmt):
    """The oracle returns each (sequence, KV head)'s hot cell exactly under
    the GPU tests' hot-key fixture (plant_hot_keys), for plain and one-byte
    pools: the fixture's expectation is exact for the fp32 restatement too."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from _helpers import plant_hot_keys
    lens = [1, 15, 16, 17, 33, 511, 512, 513, 2000, 300, 64]
    b = W.make_batch("idxo", lens, group * 2, 2, head_size, dtype, 94, block_size=block_size)
    q, k, v = b.values_numpy()
    rng = np.random.default_rng(8)

    def pick(i, h, L):
        picks = [L - 1, 0, block_size - 1, block_size, L // 2, int(rng.integers(0, L))]
        return min(picks[(2 * i + h) % len(picks)], L - 1)

    if fmt == O.FP8_E4M3:
        enc = lambda p, s, h: (p % 16 + 1, (p // 16) % 16 + 1, s + 1, h + 1)
    else:
        enc = lambda p, s, h: (p % 100 + 1, p // 100 + 1, s + 1, h + 1)
    expect = plant_hot_keys(b, q, k, v, pick, enc)
    if fmt:
        k8 = O.fp8_encode(k.astype(np.float32), fmt)
        v8 = O.fp8_encode(v.astype(np.float32), fmt)
        out = O.attention_fp8(q, k8, v8, fmt, 1.0, 1.0, b.block_tables, b.seq_lens, 2, b.scale,
                              block_size=block_size)
    else:
        out = O.attention(q, k, v, b.block_tables, b.seq_lens, 2, b.scale, block_size=block_size)
    out = np.asarray(out, dtype=np.float64)
    assert np.array_equal(out[:, :, :4], expect)
    assert not np.any(out[:, :, 4:])
