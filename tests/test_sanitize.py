"""The host C code under AddressSanitizer and UndefinedBehaviorSanitizer
(oracle/Makefile target `sanitize`, program oracle/sanitize_check.c): the CPU
oracle, the backend plugin's C logic, and the reference's own CPU attention
when its sources are present. Any report aborts the program."""
import json
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_host_c_code_is_clean_under_asan_and_ubsan():
    args = ["make", "-s", "-C", os.path.join(ROOT, "oracle"), "sanitize"]
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            ref = json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        ref = ""
    if ref and os.path.isdir(ref):
        args.append(f"REF_ROOT={ref}")
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "sanitize ok" in r.stdout
    if ref and os.path.isdir(ref):
        assert "with the reference's CPU attention" in r.stdout
