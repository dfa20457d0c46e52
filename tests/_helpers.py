"""Shared test helpers: run the CUDA path and the oracle on the same seeded inputs."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O
from xllms_b200 import workloads as W

# north_star tolerance: 1e-3 relative error for fp32/fp16 KV with fp32
# accumulation, element-wise |x - ref| <= RTOL * max(|ref|, eps), where
# eps = 1e-2 * rms(ref) keeps elements that are ~0 in the reference from
# turning rounding noise into an unbounded relative error.
RTOL = 1e-3


def oracle_out(batch: W.PagedBatch, q, k, v, num_blocks=-1, f64=False) -> np.ndarray:
    """The oracle's output; f64=True accumulates in fp64 (the exact reference
    for contexts long enough that the fp32 oracle's own rounding is a sizeable
    share of the tolerance)."""
    return O.attention(q, k, v, batch.block_tables, batch.seq_lens, batch.num_kv_heads,
                       batch.scale, block_size=batch.block_size, num_blocks=num_blocks,
                       f64=f64)


def to_device(batch: W.PagedBatch, q, k, v, dev):
    import torch
    qt = torch.from_numpy(q).to(dev)
    kt = torch.from_numpy(k).to(dev)
    vt = torch.from_numpy(v).to(dev)
    bt, sl = batch.tables_torch(dev)
    return qt, kt, vt, bt, sl


def check_close(out, ref, rtol=RTOL, what=""):
    x = out.float().cpu().numpy() if hasattr(out, "cpu") else np.asarray(out)
    ok, worst = O.rel_err_ok(x, ref, rtol)
    assert ok, f"{what}: worst |x-ref|/(rtol*max(|ref|,eps)) = {worst:.3f}"
    return worst


def gather_subset(batch: W.PagedBatch, seqs, q_t, k_t, v_t):
    """Copies the pages of the chosen sequences off the device and relabels the
    block tables, so the oracle can check a few sequences of a full-size batch."""
    import torch
    rows = []
    pages = []
    for b in seqs:
        npg = int(batch.pages_per_seq()[b])
        ids = batch.block_tables[b, :npg]
        rows.append(np.arange(len(pages), len(pages) + npg, dtype=np.int32))
        pages.extend(int(x) for x in ids)
    idx = torch.tensor(pages, dtype=torch.long, device=k_t.device)
    k = k_t.index_select(0, idx).cpu().numpy()
    v = v_t.index_select(0, idx).cpu().numpy()
    q = q_t[list(seqs)].cpu().numpy()
    mb = max(len(r) for r in rows)
    bt = np.full((len(seqs), max(1, mb)), -1, dtype=np.int32)
    for i, r in enumerate(rows):
        bt[i, :len(r)] = r
    sl = batch.seq_lens[list(seqs)].astype(np.int32)
    return q, k, v, bt, sl


def plant_hot_keys(b: W.PagedBatch, q, k, v, pick, encode):
    """Index-logic fixture, modified in place: Q = 1 and K = 0 except one
    hot key (8.0 in every dim) per (sequence, KV head) at token
    pick(i, h, L); V rows hold encode(page, slot, kv_head), four integers
    >= 1, in dims 0-3 and 0 elsewhere. The hot key's score is 8*sqrt(D)
    nats above the rest, so its weight is 1 and every query head of the
    group must return the hot cell's integers exactly. Returns those
    expected rows [B, Hq, 4]."""
    q[:] = 1
    k[:] = 0
    v[:] = 0
    nb, hkv, bs, _ = k.shape
    pages, heads, slots = np.meshgrid(np.arange(nb), np.arange(hkv), np.arange(bs),
                                      indexing="ij")
    for c, x in enumerate(encode(pages, slots, heads)):
        v[..., c] = x
    group = q.shape[1] // hkv
    expect = np.zeros((b.num_seqs, q.shape[1], 4), dtype=np.float64)
    for i, L in enumerate(int(x) for x in b.seq_lens):
        if L == 0:
            continue
        for h in range(hkv):
            t = pick(i, h, L)
            page, slot = int(b.block_tables[i, t // bs]), t % bs
            k[page, h, slot, :] = 8.0
            expect[i, h * group:(h + 1) * group] = encode(page, slot, h)
    return expect


def assert_hot_cells(out, expect):
    """Bit-exact check of plant_hot_keys' expected rows; dims >= 4 are 0."""
    got = out.double().cpu().numpy() if hasattr(out, "cpu") else np.asarray(out, np.float64)
    assert np.array_equal(got[:, :, :4], expect)
    assert not np.any(got[:, :, 4:])
