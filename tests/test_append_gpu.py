"""KV append (reshape and cache) and the decode step with the append fused in,
against the oracle's scatter and attention."""
import numpy as np
import pytest

from _helpers import check_close, to_device
from oracle import oracle as O
from xllms_b200 import _native
from xllms_b200 import operator_api as PA
from xllms_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,head_size", [("f16", 128), ("f32", 64), ("f16", 34)])
def test_reshape_and_cache_bit_exact(cuda, dtype, head_size):
    import torch
    rng = np.random.default_rng(5)
    nb, hkv, T = 40, 4, 50
    npd = np.float16 if dtype == "f16" else np.float32
    kc = rng.standard_normal((nb, hkv, 16, head_size)).astype(npd)
    vc = rng.standard_normal((nb, hkv, 16, head_size)).astype(npd)
    key = rng.standard_normal((T, hkv, head_size)).astype(npd)
    val = rng.standard_normal((T, hkv, head_size)).astype(npd)
    slots = rng.choice(nb * 16, size=T, replace=False).astype(np.int64)
    slots[[3, 17]] = -1  # padding tokens are skipped
    kt, vt = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    PA.reshape_and_cache(torch.from_numpy(key).to(cuda), torch.from_numpy(val).to(cuda), kt, vt,
                         torch.from_numpy(slots).to(cuda))
    torch.cuda.synchronize()
    O.reshape_and_cache(key, val, kc, vc, slots)
    assert np.array_equal(kt.cpu().numpy(), kc) and np.array_equal(vt.cpu().numpy(), vc)


@pytest.mark.parametrize("dtype,hq,hkv,d", [("f16", 32, 8, 128), ("f32", 12, 12, 64),
                                            ("f16", 16, 2, 256)])
def test_append_fused_decode_step(cuda, dtype, hq, hkv, d):
    import torch
    # lengths include the new token; 17, 33 and 2049 put it at slot 0 of a new page
    lens = [1, 17, 33, 500, 2049, 5000]
    b = W.make_batch("ap", lens, hq, hkv, d, dtype, 61, value_std=0.5)
    q, k, v = b.values_numpy()
    rng = np.random.default_rng(9)
    new_k = rng.standard_normal((b.num_seqs, hkv, d)).astype(k.dtype) * 0.5
    new_v = rng.standard_normal((b.num_seqs, hkv, d)).astype(k.dtype) * 0.5
    slots = np.array([int(b.block_tables[i, (L - 1) // 16]) * 16 + (L - 1) % 16
                      for i, L in enumerate(b.seq_lens)], dtype=np.int64)
    qt, kt, vt, bt, sl = to_device(b, q, k, v, cuda)
    # reference: scatter on the host, then attention
    kr, vr = k.copy(), v.copy()
    O.reshape_and_cache(new_k, new_v, kr, vr, slots)
    ref = O.attention(q, kr, vr, b.block_tables, b.seq_lens, hkv, b.scale)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = PA.paged_attention_append(qt, kt, vt, bt, sl, torch.from_numpy(new_k).to(cuda),
                                    torch.from_numpy(new_v).to(cuda),
                                    torch.from_numpy(slots).to(cuda), device_status=status)
    torch.cuda.synchronize()
    check_close(out, ref, what=f"append {dtype} D={d}")
    assert np.array_equal(kt.cpu().numpy(), kr) and np.array_equal(vt.cpu().numpy(), vr)
    assert int(status.item()) == 0


def test_append_rejects_bad_arguments(cuda):
    import torch
    z = torch.zeros((4, 2, 16, 64), dtype=torch.float16, device=cuda)
    key = torch.zeros((3, 2, 64), dtype=torch.float16, device=cuda)
    slots = torch.zeros(3, dtype=torch.int64, device=cuda)
    # shape mismatches are refused on the host, before any launch
    with pytest.raises(PA.PagedAttentionError):
        PA.reshape_and_cache(key, key, z, z[:, :1].contiguous(), slots)
    with pytest.raises(PA.PagedAttentionError):
        PA.reshape_and_cache(key[:, :1].contiguous(), key[:, :1].contiguous(), z, z, slots)
    # a missing slot mapping is refused by the C ABI
    rc = _native.xpa().nxt_reshape_and_cache(key.data_ptr(), key.data_ptr(), z.data_ptr(),
                                             z.data_ptr(), None, 3, 2, 64, 16, 2, 2 * 16 * 64,
                                             16 * 64, 2 * 64, None)
    assert rc == _native.NXT_PA_EINVAL
