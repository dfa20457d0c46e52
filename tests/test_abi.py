"""The C-ABI boundary without a GPU: libraries load, every declared symbol is
exported with C linkage, argument checks and the plugin's NULL contract."""
import ctypes
import os
import re
import subprocess

import pytest

from xllms_b200 import _native
from xllms_b200 import operator_api as PA

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
DECL = re.compile(r"^\s*(?:void|int|size_t|uint64_t|const\s+char)\s*\*?\s*(nxt_\w+)\s*\(", re.M)


def declared(header):
    with open(os.path.join(INCLUDE, header)) as f:
        return sorted(set(DECL.findall(f.read())))


def test_every_operator_symbol_exported():
    names = declared("operator_api.h")
    assert "nxt_paged_attention" in names and "nxt_paged_attention_v2" in names
    lib = _native.xpa()
    for n in names:
        assert hasattr(lib, n), n
        assert n in _native.SIGNATURES, f"{n} has no ctypes signature"


def test_every_plugin_symbol_exported():
    names = declared("cuda_backend.h")
    assert names == ["nxt_backend_fini", "nxt_backend_init", "nxt_backend_run"]
    lib = _native.plugin()
    for n in names:
        assert hasattr(lib, n), n


def test_plain_c_caller_links_unmangled_symbols(tmp_path):
    """The reference's own CUDA build exports a C++-mangled nxt_paged_attention
    that C callers cannot link. Here a C11 program includes the headers, links
    libxpa.so and makes the reference's zero-size call (tests/test_attention.c:80-100)."""
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include "operator_api.h"
#include "cuda_backend.h"
int main(void) {
    int bt = 0, sl = 0;
    nxt_paged_attention(NULL, NULL, NULL, NULL, &bt, &sl, 0, 0, 0, 0, 0.0f, 0, 0, 0, 0, 0, NULL);
    nxt_paged_attention_v2(NULL, NULL, NULL, NULL, &bt, &sl, 0, 0, 0, 0, 0.0f, 0, 0, 0, 0, 0, NULL);
    nxt_paged_attention_flash(NULL, NULL, NULL, NULL, &bt, &sl, 0, 0, 0, 0, 0.0f, 0, 0, 0, 0, 0, NULL);
    if (nxt_paged_attention_last_error() != NXT_PA_OK) return 1;
    if (nxt_backend_init(NULL) != -1 || nxt_backend_run(NULL, NULL, NULL) != -1 ||
        nxt_backend_fini(NULL) != -1) return 2;
    printf("ok\n");
    return 0;
}
''')
    exe = tmp_path / "caller"
    cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", INCLUDE, str(src), "-o", str(exe),
                    "-L", _native.LIB_DIR, "-lxllm_cuda_backend", "-lxpa",
                    f"-Wl,-rpath,{_native.LIB_DIR}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


def test_zero_size_call_is_a_noop():
    PA.nxt_paged_attention(None, None, None, None, None, None, 0, 0, 0, 0, 0.0, 0, 0, 0, 0, 0)
    assert _native.xpa().nxt_paged_attention_last_error() == _native.NXT_PA_OK


@pytest.mark.parametrize("bad", [
    dict(num_heads=6, num_kv_heads=4),      # heads not a multiple of KV heads
    dict(dtype_size=3),
    dict(head_size=0),
    dict(head_size=512),
    dict(block_size=0),
    dict(num_seqs=-1),
    dict(out=None),
])
def test_invalid_arguments_rejected_before_any_launch(bad):
    args = dict(out=16, query=16, key_cache=16, value_cache=16, block_tables=16, seq_lens=16,
                num_seqs=1, num_heads=8, head_size=64, num_kv_heads=2, scale=0.125,
                max_num_blocks_per_seq=1, block_size=16, dtype_size=2,
                kv_block_stride=2 * 16 * 64, kv_head_stride=16 * 64)
    args.update(bad)
    with pytest.raises(PA.PagedAttentionError) as ei:
        PA.nxt_paged_attention(**args)
    assert ei.value.code == _native.NXT_PA_EINVAL


def _plan_parts(B, Hkv, max_blocks, per_sm=24, nsm=148, part_pages=128):
    """Partition count of one call: the library's planning rule restated
    (partitions halve, down to 4 pages, while the grid holds fewer than
    per_sm items per SM; the SM count is 148 when no device answers)."""
    pp = part_pages
    while pp > 4 and B * Hkv * -(-max_blocks // pp) < per_sm * nsm:
        pp //= 2
    while -(-max_blocks // pp) > 8192:
        pp *= 2
    return -(-max_blocks // pp)


def _partial_bytes(rows_slots, D):
    """part_o [rows][slots][D] fp32, then the (max, sum) pairs from the next
    256-byte boundary."""
    off = -(-(rows_slots * D * 4) // 256) * 256
    return off + rows_slots * 8


@pytest.mark.parametrize("B,Hq,Hkv,D,mb", [(3, 3, 1, 33, 12), (3, 9, 3, 65, 313),
                                           (1, 1, 1, 127, 12), (64, 32, 8, 128, 512)])
def test_workspace_size_pads_the_pair_table_to_an_aligned_offset(B, Hq, Hkv, D, mb):
    """Odd head size x odd query heads x odd partition count puts the end of
    the partial outputs on a 4-byte boundary; the size queries must count the
    padding that starts the (max, sum) pairs on a 256-byte boundary."""
    parts = _plan_parts(B, Hkv, mb)
    assert parts > 1
    lib = _native.xpa()
    got = lib.nxt_paged_attention_workspace_size(B, Hq, D, Hkv, mb, 16, 2)
    assert got == _partial_bytes(B * Hq * parts, D)
    parts8 = _plan_parts(B, Hkv, mb, per_sm=24)
    assert lib.nxt_paged_attention_fp8_workspace_size(B, Hq, D, Hkv, mb, 16) == \
        _partial_bytes(B * Hq * parts8, D)
    # the cascade query adds the prefix chunks' slots (16-page chunks, the floor)
    pre = 32
    assert lib.nxt_paged_attention_prefix_workspace_size(B, Hq, D, Hkv, mb, 16, pre) == \
        _partial_bytes(B * Hq * (parts + -(-pre // 16)), D)


def test_misaligned_caller_workspace_rejected_before_any_launch():
    """A caller workspace that does not start on a 16-byte boundary is refused
    with NXT_PA_EINVAL before anything touches a device."""
    lib = _native.xpa()
    p = ctypes.c_void_p(4096)
    ip = ctypes.cast(p, ctypes.POINTER(ctypes.c_int))
    for ws in (4100, 4104, 4108):
        rc = lib.nxt_paged_attention_ex(p, p, p, p, ip, ip, 3, 3, 33, 1, 0.17, 12, 16, 2,
                                        16 * 33, 16 * 33, 64, ctypes.c_void_p(ws), 1 << 20,
                                        None, None)
        assert rc == _native.NXT_PA_EINVAL


def test_strerror():
    for code in (0, -22, -12, -28, -5, 77):
        assert _native.strerror(code)


def test_plugin_null_contract_without_gpu():
    lib = _native.plugin()
    assert lib.nxt_backend_init(None) == -1
    assert lib.nxt_backend_run(None, None, None) == -1
    assert lib.nxt_backend_fini(None) == -1
    be = PA.NxtBackend()
    assert lib.nxt_backend_run(ctypes.byref(be), ctypes.byref(PA.NxtPagedAttentionInput()),
                               ctypes.c_void_p(16)) == -1       # no backend state yet
    be.state = PA.NXT_BACKEND_STATE_READY
    assert lib.nxt_backend_fini(ctypes.byref(be)) == 0
    assert be.state == PA.NXT_BACKEND_STATE_UNINITIALIZED and not be.backend_state


def test_descriptor_layouts_match_reference_abi():
    # offsets pinned by the reference's tests/mock_cuda_backend.c:22-37 (x86-64)
    assert PA.NxtBackend.state.offset == 88
    assert PA.NxtBackend.backend_state.offset == 112
    assert ctypes.sizeof(PA.NxtBackend) == 120
    # NxtPagedAttentionInput (backends/cuda_backend.h:29-46): 5 pointers, 10 scalars, stream
    assert PA.NxtPagedAttentionInput.num_seqs.offset == 40
    assert PA.NxtPagedAttentionInput.scale.offset == 56
    assert PA.NxtPagedAttentionInput.stream.offset == 80
    assert ctypes.sizeof(PA.NxtPagedAttentionInput) == 88


def test_layout_offsets_in_c(tmp_path):
    src = tmp_path / "off.c"
    src.write_text(r'''
#include <stddef.h>
#include <stdio.h>
#include "cuda_backend.h"
#include "xllm_backend_abi.h"
int main(void) {
    printf("%zu %zu %zu %zu %zu\n", offsetof(struct NxtBackend, state),
           offsetof(struct NxtBackend, backend_state), sizeof(struct NxtBackend),
           offsetof(NxtPagedAttentionInput, stream), sizeof(NxtPagedAttentionInput));
    return 0;
}
''')
    exe = tmp_path / "off"
    cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
    subprocess.run([cc, "-std=c11", "-I", INCLUDE, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["88", "112", "120", "80", "88"]


def test_shard_descriptor_layout():
    from xllms_b200 import sharding as S
    assert ctypes.sizeof(S.NxtPaShard) == 152
    assert S.NxtPaShard.peer_out.offset == 16 and S.NxtPaShard.peer_flags.offset == 80
    assert S.NxtPaShard.mc_out.offset == 144


def test_python_wrappers_refuse_bad_tensors_on_the_host():
    # Every check runs before a pointer reaches the C ABI (no GPU needed).
    torch = pytest.importorskip("torch")
    q = torch.zeros(2, 8, 64, dtype=torch.float16)
    kc = torch.zeros(4, 2, 16, 64, dtype=torch.float16)
    bt = torch.zeros(2, 4, dtype=torch.int32)
    sl = torch.ones(2, dtype=torch.int32)
    cases = [
        lambda: PA.paged_attention(q, kc.float(), kc.float(), bt, sl),          # K/V dtype
        lambda: PA.paged_attention(q, kc, kc, bt.long(), sl),                   # table dtype
        lambda: PA.paged_attention(q, kc, kc, bt, sl.long()),                   # lens dtype
        lambda: PA.paged_attention(q, kc, kc, bt[:1], sl),                      # too few rows
        lambda: PA.paged_attention(q, kc, kc, bt, sl, out=q.float()),           # out dtype
        lambda: PA.paged_attention(q.transpose(0, 1), kc, kc, bt, sl),          # layout
        lambda: PA.paged_attention(q, kc, kc, bt, sl),                          # host tensors
        lambda: PA.paged_attention_fp8(q.float(), kc.to(torch.uint8), kc.to(torch.uint8), bt,
                                       sl, "int8", 1.0, 1.0),                   # query dtype
        lambda: PA.paged_attention_fp8(q, kc, kc, bt, sl, "e4m3", 1.0, 1.0),    # 2-byte pools
        lambda: PA.reshape_and_cache(q[:, :2], q[:, :2], kc, kc,
                                     torch.zeros(2, dtype=torch.int32)),        # slot dtype
        lambda: PA.reshape_and_cache_fp8(q[:, :2].float(), q[:, :2].float(), kc.to(torch.uint8),
                                         kc.to(torch.uint8), torch.zeros(2, dtype=torch.int64),
                                         "e4m3", 1.0, 1.0),                     # key dtype
    ]
    for i, call in enumerate(cases):
        with pytest.raises(PA.PagedAttentionError) as ei:
            call()
        assert ei.value.code == _native.NXT_PA_EINVAL, i


def test_sharded_call_refuses_a_misaligned_multicast_address():
    """The multicast address of the gather buffers takes 16-byte stores: a
    misaligned one is refused with NXT_PA_EINVAL before anything touches a
    device (and so is a shard without peer buffers)."""
    from xllms_b200 import sharding as S
    lib = _native.xpa()
    sh = S.NxtPaShard()
    sh.world_size, sh.rank, sh.total_heads, sh.head_offset = 2, 0, 32, 0
    for r in range(2):
        sh.peer_out[r] = 1 << 20
        sh.peer_flags[r] = (1 << 20) + 4096
    p = ctypes.c_void_p(4096)
    ip = ctypes.cast(p, ctypes.POINTER(ctypes.c_int))
    args = (1, p, p, p, ip, ip, 2, 16, 128, 4, 0.088, 4, 16, 2, 4 * 16 * 128, 16 * 128, 64,
            None, None)
    sh.mc_out = (1 << 21) + 8
    assert lib.nxt_paged_attention_sharded(ctypes.byref(sh), *args) == _native.NXT_PA_EINVAL
    sh.mc_out = None
    sh.peer_out[1] = None
    assert lib.nxt_paged_attention_sharded(ctypes.byref(sh), *args) == _native.NXT_PA_EINVAL
