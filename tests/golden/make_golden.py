"""Generates the golden fixtures in this folder from the reference's own CPU
attention (examples/run_gpt2.c:46-83 of the xLLMs project, built into
oracle/_ref by `make -C oracle`).

Each fixture stores the generator parameters of a seeded case, the SHA-256 of
the generated inputs (so a change in the generators is caught) and the
reference's output. Inputs are not stored: they are regenerated from the seed.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from xllms_b200 import workloads as W  # noqa: E402

# name -> generator parameters (make_batch arguments, or a named config)
CASES = {
    "c1_gpt2_small_fp32": {"config": "c1"},
    "mha_fp32_edges": {"lens": [0, 1, 15, 16, 17, 33], "num_heads": 4, "num_kv_heads": 4,
                       "head_size": 64, "dtype": "f32", "seed": 201},
    "gqa4_fp16_edges": {"lens": [1, 16, 17, 511, 512, 513], "num_heads": 8, "num_kv_heads": 2,
                        "head_size": 128, "dtype": "f16", "seed": 202, "value_std": 0.5},
    "gqa8_fp16_long": {"lens": [5000, 700], "num_heads": 16, "num_kv_heads": 2,
                       "head_size": 128, "dtype": "f16", "seed": 203},
    "prefix_shared_fp16": {"config": "c4", "num_seqs": 8},
}


def build_case(spec: dict) -> W.PagedBatch:
    spec = dict(spec)
    if "config" in spec:
        name = spec.pop("config")
        return W.CONFIGS[name](**spec)
    lens = spec.pop("lens")
    return W.make_batch("golden", lens, spec.pop("num_heads"), spec.pop("num_kv_heads"),
                        spec.pop("head_size"), spec.pop("dtype"), spec.pop("seed"), **spec)


def input_digest(batch: W.PagedBatch, q, k, v) -> str:
    h = hashlib.sha256()
    for a in (q, k, v, batch.block_tables, batch.seq_lens):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def reference_output(batch: W.PagedBatch, q, k, v) -> np.ndarray:
    kr, vr = O.to_run_gpt2_layout(k, v, batch.num_kv_heads, batch.num_heads, batch.block_size)
    pt = O.per_token_tables(batch.block_tables, batch.seq_lens, batch.block_size)
    return O.reference_attention(q.astype(np.float32), kr, vr, pt, batch.seq_lens,
                                 batch.block_size, threads=1)


def main() -> None:
    for name, spec in CASES.items():
        b = build_case(spec)
        assert abs(b.scale - 1.0 / np.sqrt(b.head_size)) < 1e-12, "run_gpt2 fixes 1/sqrt(D)"
        q, k, v = b.values_numpy()
        out = reference_output(b, q, k, v)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out=out,
                            meta=np.array(json.dumps({"spec": spec,
                                                      "inputs_sha256": input_digest(b, q, k, v)})))
        print(name, out.shape)


if __name__ == "__main__":
    main()
