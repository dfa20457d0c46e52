"""Shared-prefix (cascade) attention: nxt_paged_attention_prefix_ex must give
the plain attention's result on the same inputs (checked against the oracle),
for groups larger than one 64-row tile, prefixes split into several chunks,
groups of one, members without a private suffix and sequences in no group."""
import numpy as np
import pytest

from _helpers import check_close, gather_subset, oracle_out, to_device
from oracle import oracle as O
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _batch(prefix, members, suffix, hq, hkv, d, seed, no_group=0, dtype="f16"):
    """members[g] sequences share prefix[g] tokens (a multiple of 16); then
    `no_group` sequences without a shared prefix. suffix: private tokens per
    sequence, in that order."""
    prefix_of = [g for g, n in enumerate(members) for _ in range(n)] + [-1] * no_group
    assert len(suffix) == len(prefix_of)
    lens = [(prefix[g] if g >= 0 else 0) + int(s) for g, s in zip(prefix_of, suffix)]
    return W.make_batch("pfx", lens, hq, hkv, d, dtype, seed, value_std=0.5, prefix=prefix,
                        prefix_of=prefix_of)


def _check(cuda, b, what):
    # fp64 oracle: prefixes here run to ~20k tokens, where the fp32 oracle's
    # own rounding takes up to ~0.4 of the tolerance.
    q, k, v = b.values_numpy()
    ref = oracle_out(b, q, k, v, f64=True)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention_prefix(qt, kt, vt, bt, sl, b.prefix_groups)
    check_close(out, ref, what=what)
    assert PA.device_status() == 0
    return out


@pytest.mark.parametrize("group", [1, 4, 8])
@pytest.mark.parametrize("head_size", [64, 128, 256])
def test_prefix_groups_gs_and_heads(cuda, group, head_size):
    rng = np.random.default_rng([head_size, group])
    members = [5, 3, 1]
    suffix = rng.integers(0, 300, size=sum(members) + 2)
    suffix[1] = 0     # a member with no private suffix
    suffix[6] = 16    # exactly one private page
    b = _batch([512, 64, 48], members, suffix, 2 * group, 2, head_size, 31 + group,
               no_group=2)
    _check(cuda, b, f"GS={group} D={head_size}")


def test_group_larger_than_one_tile(cuda):
    # 40 members x 4 heads = 160 rows: three 64-row query blocks, the last ragged.
    rng = np.random.default_rng(5)
    suffix = rng.integers(0, 200, size=40)
    b = _batch([1024], [40], suffix, 8, 2, 128, 41)
    _check(cuda, b, "160-row group")


def test_many_prefix_chunks(cuda):
    # 1200 shared pages: more than 64 chunks of 16, so chunks widen to 32 pages.
    rng = np.random.default_rng(6)
    suffix = rng.integers(0, 700, size=3)
    b = _batch([1200 * 16], [3], suffix, 8, 2, 128, 43)
    _check(cuda, b, "1200-page prefix")


def test_whole_sequence_is_prefix(cuda):
    b = _batch([256, 32], [4, 2], [0] * 6, 4, 1, 128, 47)
    _check(cuda, b, "no suffixes")


def test_long_suffix_split_context(cuda):
    # private suffixes beyond one 128-page partition: prefix chunks and several
    # suffix partitions merge in one row.
    b = _batch([320], [3], [5000, 2100, 7], 8, 2, 128, 53)
    _check(cuda, b, "long suffix")


def test_fp32_runs_plain_path(cuda):
    b = _batch([128], [3], [10, 0, 40], 4, 2, 64, 59, dtype="f32")
    _check(cuda, b, "fp32 cascade call")


def test_no_groups_equals_plain(cuda):
    import torch
    b = W.make_batch("plain", [100, 2000, 0, 17], 8, 2, 128, "f16", 61)
    q, k, v = b.values_numpy()
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    a = PA.paged_attention_prefix(qt, kt, vt, bt, sl, [])
    p = PA.paged_attention(qt, kt, vt, bt, sl)
    torch.cuda.synchronize()
    assert torch.equal(a, p)


def test_config4_cascade_matches_plain(cuda):
    """Full-size config 4: the cascade result agrees with the plain kernels'
    to the parity tolerance everywhere, and with the oracle on a subset."""
    import torch
    b = W.config4()
    qt, kt, vt = b.values_torch(cuda)
    bt, sl = b.tables_torch(cuda)
    a = PA.paged_attention_prefix(qt, kt, vt, bt, sl, b.prefix_groups)
    p = PA.paged_attention(qt, kt, vt, bt, sl)
    torch.cuda.synchronize()
    assert PA.device_status() == 0
    check_close(a, p.float().cpu().numpy(), rtol=2e-3, what="cascade vs plain")
    seqs = [0, 1, 127, 128, 200, 255]
    q, k, v, bt2, sl2 = gather_subset(b, seqs, qt, kt, vt)
    ref = O.attention(q, k, v, bt2, sl2, b.num_kv_heads, b.scale)
    check_close(a[seqs], ref, what="cascade vs oracle")


def test_config4_caller_workspace_of_the_queried_size(cuda):
    """A caller workspace of exactly nxt_paged_attention_prefix_workspace_size
    bytes serves a full-size config 4 cascade call (the query is an upper
    bound of whatever prefix chunking the call picks), with the same result
    as the library-owned workspace; a workspace far too small is refused."""
    import torch
    from xllms_b200 import _native
    b = W.config4()
    qt, kt, vt = b.values_torch(cuda)
    bt, sl = b.tables_torch(cuda)
    g = PA.PrefixGroups(b.prefix_groups, b.num_seqs, cuda)
    lib = _native.xpa()
    B, Hq, D, Hkv, bs = b.num_seqs, b.num_heads, b.head_size, b.num_kv_heads, b.block_size
    need = lib.nxt_paged_attention_prefix_workspace_size(B, Hq, D, Hkv, b.max_blocks, bs,
                                                         g.max_prefix_pages)
    assert need > 0

    def call(ws, nbytes):
        out = torch.empty_like(qt)
        rc = lib.nxt_paged_attention_prefix_ex(
            out.data_ptr(), qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), bt.data_ptr(),
            sl.data_ptr(), g.prefix_pages.data_ptr(), g.offsets.data_ptr(), g.members.data_ptr(),
            g.num_groups, g.max_group_size, g.max_prefix_pages, B, Hq, D, Hkv, b.scale,
            b.max_blocks, bs, 2, Hkv * bs * D, bs * D, b.num_blocks, ws, nbytes, None, None)
        return rc, out

    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    rc, out = call(ws.data_ptr(), need)
    assert rc == _native.NXT_PA_OK
    own = PA.paged_attention_prefix(qt, kt, vt, bt, sl, g, num_blocks=b.num_blocks)
    torch.cuda.synchronize()
    assert torch.equal(out, own)
    assert PA.device_status() == 0
    rc, _ = call(ws.data_ptr(), 1024)
    assert rc == _native.NXT_PA_EWORKSPACE


def test_cascade_index_logic_bit_exact(cuda):
    """Indexing through the cascade kernels, exact (plant_hot_keys): for KV
    head 0 each group's hot key lies in its shared prefix (every member must
    return that prefix cell), for KV head 1 in each member's private suffix;
    plus sequences in no group."""
    from _helpers import assert_hot_cells, plant_hot_keys
    prefix, members = [2048, 512], [5, 3]
    suffix = [1, 17, 300, 1000, 16, 40, 513, 2, 70, 900]
    b = _batch(prefix, members, suffix, 8, 2, 128, 93, no_group=2)
    prefix_of = [0] * 5 + [1] * 3 + [-1] * 2
    q, k, v = b.values_numpy()

    def pick(i, h, L):
        g = prefix_of[i]
        plen = prefix[g] if g >= 0 else 0
        if h == 0 and g >= 0:
            return (prefix[g] // 3) + 16 * g  # one position per group
        return plen + (i * 37) % (L - plen)  # this sequence's private tokens

    expect = plant_hot_keys(b, q, k, v, pick,
                            lambda p, s, h: (p % 1024 + 1, p // 1024 + 1, s + 1, h + 1))
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    out = PA.paged_attention_prefix(qt, kt, vt, bt, sl, b.prefix_groups, num_blocks=b.num_blocks)
    assert PA.device_status() == 0
    assert_hot_cells(out, expect)
