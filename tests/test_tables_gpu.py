"""Block-table builder on the GPU: bit-exact against the oracle, and its
output drives the cascade attention of config 4 to the plain result."""
import numpy as np
import pytest

from _helpers import check_close
from oracle import oracle as O
from test_tables import csr, page_lists, prefix_inputs
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _check(bt, lists, sl, max_blocks, node=None, pages=None):
    off, ids = csr(lists)
    t, slots, pp, go, mem, G, gmax, pmax = O.build_block_tables(off, ids, sl, max_blocks, 16,
                                                                node, pages)
    assert np.array_equal(bt.tables.cpu().numpy(), t)
    assert np.array_equal(bt.seq_lens.cpu().numpy(), np.asarray(sl, np.int32))
    assert np.array_equal(bt.slots.cpu().numpy(), slots)
    if G:
        assert bt.prefix is not None
        assert (bt.prefix.num_groups, bt.prefix.max_group_size, bt.prefix.max_prefix_pages) == \
            (G, gmax, pmax)
        assert np.array_equal(bt.prefix.prefix_pages.cpu().numpy(), pp)
        assert np.array_equal(bt.prefix.offsets.cpu().numpy()[:G + 1], go[:G + 1])
        assert np.array_equal(bt.prefix.members.cpu().numpy()[:go[G]], mem[:go[G]])
    else:
        assert bt.prefix is None


def test_random_batches(cuda):
    rng = np.random.default_rng(7)
    for B, mb in [(1, 1), (5, 3), (64, 512), (300, 40)]:
        lens = rng.integers(0, mb * 16 + 1, size=B)
        lists = [rng.permutation(100000)[:(L + 15) // 16].tolist() for L in lens]
        bt = PA.build_block_tables(lists, lens, mb, device=cuda)
        _check(bt, lists, lens, mb)


def test_pinned_staging(cuda):
    import torch
    from xllms_b200 import _native
    lists = [[3, 4, 5], [], [9]]
    lens = [40, 0, 1]
    staging = torch.empty(_native.xpa().nxt_block_tables_staging_size(3, 4),
                          dtype=torch.uint8).pin_memory()
    bt = PA.build_block_tables(lists, lens, 4, device=cuda, staging=staging)
    torch.cuda.synchronize()
    _check(bt, lists, lens, 4)


def test_config4_groups_and_cascade(cuda):
    import torch
    b = W.config4()
    lists = page_lists(b)
    node, pages = prefix_inputs(b)
    node[5] = 99  # a group of one: dropped
    pages[5] = 128
    bt = PA.build_block_tables(lists, b.seq_lens, b.max_blocks, prefix_node=node,
                               prefix_pages=pages, device=cuda)
    _check(bt, lists, b.seq_lens, b.max_blocks, node, pages)
    assert bt.prefix.num_groups == 2
    q, k, v = b.values_torch(cuda)
    a = PA.paged_attention_prefix(q, k, v, bt.tables, bt.seq_lens, bt.prefix,
                                  num_blocks=b.num_blocks)
    ref = PA.paged_attention(q, k, v, bt.tables, bt.seq_lens, num_blocks=b.num_blocks)
    torch.cuda.synchronize()
    check_close(a, ref.float().cpu().numpy(), rtol=2e-3, what="builder-driven cascade")
