"""The reference's own C callers drive this repository's libraries.

tests/refc/Makefile compiles, from the xLLMs sources in place, the backend
manager (src/core/backend_manager.c, with scheduler.c) under a small driver,
and the reference's tests/test_attention.c against the reference's own
include/operator_api.h, linking libxpa.so in place of its operators. The
binaries are built here when the reference checkout is present (its path is
BASELINE.json's reference_path) and travel prebuilt otherwise.

CPU: the manager finds the plugin (XLLM_CUDA_BACKEND_PATH, XLLM_BACKEND_DIR),
dlopens it and resolves its three entry points; its init then reports that
no device is usable. test_attention's signature and argument-layout cases
pass. GPU: the manager loads the plugin and runs one seeded paged decode
attention through nxt_backend_run("cuda", &input, out) (checked against the
oracle), and every case of test_attention passes, its real kernel launches
included. The reference's test_backend.c:282-283 / test_backend_load.c case
that hands the plugin a 4-byte int as its descriptor is not run: on a GPU it
would give the kernels stack bytes as device pointers."""
import json
import os
import subprocess

import numpy as np
import pytest

from _helpers import check_close, oracle_out
from xllms_b200 import _native
from xllms_b200 import workloads as W

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFC = os.path.join(ROOT, "tests", "refc")
BUILD = os.path.join(REFC, "_build")
PLUGIN = os.path.join(_native.LIB_DIR, "libxllm_cuda_backend.so")


def _ref_root():
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            path = json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        return None
    return path if path and os.path.isdir(path) else None


@pytest.fixture(scope="module")
def refc():
    ref = _ref_root()
    if ref:
        subprocess.run(["make", "-s", "-C", REFC, f"REF_ROOT={ref}"], check=True)
    exes = {n: os.path.join(BUILD, n) for n in ("manager_driver", "test_attention")}
    if not all(os.path.exists(p) for p in exes.values()):
        pytest.skip("reference C callers neither buildable here nor prebuilt")
    return exes


def _driver(refc, *args, env_extra=None):
    env = dict(os.environ)
    env.pop("XLLM_CUDA_BACKEND_PATH", None)
    env.pop("XLLM_BACKEND_DIR", None)
    env.update(env_extra or {})
    return subprocess.run([refc["manager_driver"], *args], capture_output=True, text=True,
                          env=env, timeout=300, cwd=REFC)


def _gpu():
    import torch
    return torch.cuda.is_available()


@pytest.mark.parametrize("how", ["exact_path", "directory"])
def test_manager_finds_and_dlopens_the_plugin(refc, how):
    env = ({"XLLM_CUDA_BACKEND_PATH": PLUGIN} if how == "exact_path"
           else {"XLLM_BACKEND_DIR": _native.LIB_DIR})
    r = _driver(refc, "discover", env_extra=env)
    assert r.returncode == 0, r.stdout + r.stderr
    if _gpu():
        assert "loaded=1 ready=1" in r.stdout, r.stdout + r.stderr
    else:
        # dlopen and the three dlsym lookups succeeded; init found no device
        assert "loaded=0" in r.stdout
        assert "no usable CUDA device" in r.stderr and "backend_init(cuda) failed" in r.stderr
        assert "dlopen(" not in r.stderr and "no nxt_backend_init" not in r.stderr


def test_manager_without_a_plugin_path_loads_nothing(refc):
    r = _driver(refc, "discover")
    assert r.returncode == 0 and "loaded=0" in r.stdout
    assert "not found" in r.stderr


def test_reference_attention_test_signature_cases(refc):
    r = subprocess.run([refc["test_attention"]], capture_output=True, text=True, timeout=300)
    lines = {ln.split("...")[0].strip(): ln for ln in r.stdout.splitlines() if "..." in ln}
    cpu_cases = [k for k in lines if "cuda_launch" not in k and "head_sizes" not in k]
    assert len(cpu_cases) == 10, r.stdout
    for k in cpu_cases:
        assert lines[k].rstrip().endswith("PASS"), lines[k]


@pytest.mark.gpu
def test_reference_attention_test_passes_on_the_gpu(cuda, refc):
    r = subprocess.run([refc["test_attention"]], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "All tests PASSED." in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,lens,heads,kv_heads,head_size", [
    ("f16", [1, 17, 700, 2100, 0, 4096], 32, 8, 128),   # config-2 shape, split contexts
    ("f32", [37, 128, 255, 512], 12, 12, 64),            # config-1 shape
])
def test_manager_runs_attention_through_the_plugin(cuda, refc, tmp_path, dtype, lens, heads,
                                                   kv_heads, head_size):
    b = W.make_batch("refc", lens, heads, kv_heads, head_size, dtype, 29, value_std=0.5)
    q, k, v = b.values_numpy()
    hdr = np.array([b.num_seqs, b.num_heads, b.head_size, b.num_kv_heads, b.max_blocks,
                    b.block_size, b.dtype_size, b.kv_block_stride, b.kv_head_stride,
                    b.num_blocks], dtype=np.int32)
    prob = tmp_path / "problem.bin"
    with open(prob, "wb") as f:
        for a in (hdr, np.array([b.scale], dtype=np.float32), q, k, v,
                  b.block_tables.astype(np.int32), b.seq_lens.astype(np.int32)):
            f.write(np.ascontiguousarray(a).tobytes())
    out = tmp_path / "out.bin"
    r = _driver(refc, "run", str(prob), str(out), env_extra={"XLLM_CUDA_BACKEND_PATH": PLUGIN})
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
    got = np.fromfile(out, dtype=q.dtype).reshape(q.shape)
    check_close(got, oracle_out(b, q, k, v, f64=True), what=f"manager run {dtype}")
