"""Block-table builder: the oracle restatement against the seeded workloads'
own tables, and the C ABI's argument checks (no GPU work)."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import workloads as W


def page_lists(batch):
    return [batch.block_tables[b, :int(n)].tolist() for b, n in enumerate(batch.pages_per_seq())]


def csr(lists):
    off = np.zeros(len(lists) + 1, dtype=np.int32)
    np.cumsum([len(p) for p in lists], out=off[1:])
    ids = np.concatenate([np.asarray(p, dtype=np.int32) for p in lists]) if off[-1] else \
        np.zeros(0, dtype=np.int32)
    return off, ids


def prefix_inputs(batch):
    node = np.full(batch.num_seqs, -1, dtype=np.int32)
    pages = np.zeros(batch.num_seqs, dtype=np.int32)
    for g, (members, p) in enumerate(batch.prefix_groups):
        node[members] = 10 + g
        pages[members] = p
    return node, pages


def test_oracle_rebuilds_config4_tables_and_groups():
    b = W.config4(num_seqs=24)
    off, ids = csr(page_lists(b))
    node, pages = prefix_inputs(b)
    t, slots, pp, go, mem, G, gmax, pmax = O.build_block_tables(
        off, ids, b.seq_lens, b.max_blocks, 16, node, pages)
    assert np.array_equal(t, b.block_tables)
    L = b.seq_lens.astype(np.int64)
    assert np.array_equal(slots, b.block_tables[np.arange(b.num_seqs), (L - 1) // 16] * 16 + (L - 1) % 16)
    assert G == len(b.prefix_groups)
    for g, (members, p) in enumerate(b.prefix_groups):
        assert mem[go[g]:go[g + 1]].tolist() == members
        assert (pp[members] == p).all()
    assert gmax == max(len(m) for m, _ in b.prefix_groups) and pmax == 128


def _call(off, ids, sl, node, pages, B, max_blocks, buf=0x1000, nbytes=1 << 30):
    lib = _native.xpa()
    g = (ctypes.c_int * 3)()
    p = lambda a: None if a is None else a.ctypes.data
    return lib.nxt_build_block_tables(p(off), p(ids), p(sl), p(node), p(pages), B, max_blocks, 16,
                                      buf, nbytes, None, 0, ctypes.addressof(g),
                                      ctypes.addressof(g) + 4, ctypes.addressof(g) + 8, None)


def test_argument_checks_without_gpu():
    einval = _native.NXT_PA_EINVAL
    off = np.array([0, 3, 5], dtype=np.int32)
    ids = np.array([7, 8, 9, 7, 8], dtype=np.int32)
    sl = np.array([40, 20], dtype=np.int32)
    assert _call(off, ids, sl, None, None, 2, 2) == einval            # a row longer than max_blocks
    assert _call(off, ids, np.array([49, 20], np.int32), None, None, 2, 4) == einval  # seq beyond pages
    node = np.array([1, 1], dtype=np.int32)
    assert _call(off, ids, sl, node, np.array([2, 1], np.int32), 2, 4) == einval  # page counts differ
    ids2 = np.array([7, 8, 9, 7, 6], dtype=np.int32)
    assert _call(off, ids2, sl, node, np.array([2, 2], np.int32), 2, 4) == einval  # page ids differ
    assert _call(off, ids, sl, node, None, 2, 4) == einval            # node without pages
    assert _call(off, ids, sl, None, None, 2, 4, nbytes=16) == _native.NXT_PA_EWORKSPACE
    assert _call(off, ids, sl, None, None, 2, 4, buf=0x1004) == _native.NXT_PA_EWORKSPACE
    assert _call(None, None, None, None, None, 0, 4) == _native.NXT_PA_OK  # nothing to build


def test_layout_offsets_are_aligned_and_disjoint():
    lib = _native.xpa()
    offs = (ctypes.c_size_t * _native.NXT_BT_NUM_ARRAYS)()
    B, mb, P = 37, 100, 1234
    total = lib.nxt_block_tables_layout(B, mb, P, offs)
    sizes = {_native.NXT_BT_TABLES: B * mb * 4, _native.NXT_BT_SEQ_LENS: B * 4,
             _native.NXT_BT_SLOTS: B * 8, _native.NXT_BT_PREFIX_PAGES: B * 4,
             _native.NXT_BT_GROUP_OFFSETS: (B + 1) * 4, _native.NXT_BT_GROUP_MEMBERS: B * 4}
    spans = sorted((offs[k], offs[k] + n) for k, n in sizes.items())
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:])) and spans[-1][1] <= total
    assert offs[_native.NXT_BT_SLOTS] % 16 == 0 and offs[_native.NXT_BT_TABLES] % 16 == 0
    assert lib.nxt_block_tables_staging_size(B, P) <= offs[_native.NXT_BT_SLOTS]
