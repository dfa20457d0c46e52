"""Seeded workload generators: determinism, page ownership, prefix aliasing,
head sharding and the byte accounting the benchmark reports (CPU only)."""
import numpy as np
import pytest

from xllms_b200 import workloads as W


def test_deterministic():
    a, b = W.config2(), W.config2()
    assert np.array_equal(a.block_tables, b.block_tables)
    assert np.array_equal(a.seq_lens, b.seq_lens)
    qa = W.config1().values_numpy()
    qb = W.config1().values_numpy()
    for x, y in zip(qa, qb):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3"])
def test_private_pages_disjoint_and_in_pool(cfg):
    b = W.CONFIGS[cfg]()
    seen = set()
    for i in range(b.num_seqs):
        n = int(b.pages_per_seq()[i])
        row = b.block_tables[i, :n]
        assert (row >= 0).all() and (row < b.num_blocks).all()
        assert not (set(row.tolist()) & seen)
        seen |= set(row.tolist())
        assert (b.block_tables[i, n:] == -1).all()


def test_config_shapes_match_baseline():
    c1 = W.config1()
    assert c1.seq_lens.tolist() == [37, 128, 255, 512] and c1.num_blocks == 256
    assert int(c1.pages_per_seq().sum()) == 59 and c1.dtype == "f32"
    c2 = W.config2()
    assert (c2.num_seqs, c2.num_heads, c2.num_kv_heads, c2.head_size) == (64, 32, 8, 128)
    assert c2.seq_lens.min() >= 1024 and c2.seq_lens.max() <= 8192
    assert c2.num_blocks == int(np.ceil(c2.pages_per_seq().sum() * 1.1))
    # ~1.208 GB of KV at the mean length 4608
    assert 0.9e9 < c2.kv_bytes() < 1.5e9
    c3 = W.config3()
    assert c3.group == 8 and c3.max_blocks == 8192 and c3.seq_lens.min() >= 32768
    c5 = W.config5()
    assert (c5.num_seqs, c5.num_heads, c5.num_kv_heads) == (512, 64, 8)


def test_prefix_sharing_aliases_pages():
    b = W.config4()
    a0 = b.block_tables[0, :128]
    for i in range(1, 128):
        assert np.array_equal(b.block_tables[i, :128], a0)
    b0 = b.block_tables[128, :32]
    for i in range(129, 256):
        assert np.array_equal(b.block_tables[i, :32], b0)
    assert not (set(a0.tolist()) & set(b0.tolist()))
    priv = []
    for i in range(256):
        start = 128 if i < 128 else 32
        priv.extend(b.block_tables[i, start:int(b.pages_per_seq()[i])].tolist())
    assert len(priv) == len(set(priv))
    assert b.kv_bytes_unique() < 0.4 * b.kv_bytes()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_sharding(world):
    shards = [W.config5(world_size=world, rank=r) for r in range(world)]
    for r, s in enumerate(shards):
        assert s.num_kv_heads == 8 // world and s.num_heads == 64 // world
        assert np.array_equal(s.seq_lens, shards[0].seq_lens)
    assert sum(s.kv_bytes() for s in shards) == W.config5().kv_bytes()


def test_algorithmic_bytes_formula():
    b = W.config2()
    L = b.seq_lens.astype(np.int64)
    kv = int(L.sum()) * 8 * 128 * 2 * 2
    qo = 2 * 64 * 32 * 128 * 2
    bt = int(((L + 15) // 16).sum()) * 4
    assert b.algorithmic_bytes() == kv + qo + bt + 64 * 4
    assert b.flops() == int(L.sum()) * 32 * 4 * 128


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c4", "c5"])
def test_cpu_sample_fits_reference_offsets(cfg):
    # The reference CPU attention forms page offsets as 32-bit int products
    # (examples/run_gpt2.c:63); the bench's CPU sample keeps its pool inside.
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    b = W.CONFIGS[cfg]()
    seqs, lens = bench.sample_plan(b, 8)
    assert seqs == list(range(len(seqs))) and 1 <= len(seqs) <= 8
    pages = sum(-(-L // b.block_size) for L in lens)
    per_page = b.block_size * b.num_heads * b.head_size
    assert pages * per_page <= min(2**31 - 1, bench.REF_SAMPLE_ELEMS)
    for s, L in zip(seqs, lens):
        assert 0 < L <= int(b.seq_lens[s]) or (L == 0 and b.seq_lens[s] == 0)
    if cfg == "c2":  # every sequence whole, as before the bound
        assert len(seqs) == 8 and lens == [int(x) for x in b.seq_lens[:8]]
