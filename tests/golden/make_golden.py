"""Generate the golden fixtures in this folder from the CPU oracle.

Run from the repository root:  python tests/golden/make_golden.py

Each fixture fixes a small seeded layer (inputs are regenerated from the
seed by noor_-_bangla_ai_b200/workloads.py and checked against the stored
SHA-256 of their bytes) and stores the oracle's ParallelFFN output, top-k
indices, weights and counts.  The oracle itself is pinned against the
reference's known-answer tests (reference_kat.json, tests/test_oracle.py).
"""
from __future__ import annotations

import hashlib
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

W = importlib.import_module("noor_-_bangla_ai_b200.workloads")
from oracle import oracle as O  # noqa: E402

GOLDEN = {
    "tiny_f32": W.LayerConfig("tiny_f32", 96, 64, 8, 2, 64, 96, W.F32, seed=7, has_shared=True),
    "tiny_f32_e4": W.LayerConfig("tiny_f32_e4", 33, 32, 4, 2, 32, 64, W.F32, seed=8),
    "tiny_bf16": W.LayerConfig("tiny_bf16", 200, 128, 16, 4, 128, 256, W.BF16, seed=9,
                               x_dist="rmsnorm", bias_dist="uniform0.1"),
    "small_bf16_shared": W.LayerConfig("small_bf16_shared", 128, 256, 8, 2, 256, 256, W.BF16, seed=10,
                                       x_dist="rmsnorm", bias_dist="uniform0.1", has_shared=True),
}


def input_digest(w, x) -> str:
    h = hashlib.sha256()
    for a in (x, w.gate, w.bias, w.scales, w.w_gate, w.w_up, w.w_down, w.dense_gate, w.dense_up, w.dense_down,
              w.shared_gate, w.shared_up, w.shared_down):
        if a is not None:
            h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def make(name: str):
    cfg = GOLDEN[name]
    w = W.make_weights(cfg)
    x = W.make_tokens(cfg)
    out, idx, wt, counts = O.parallel_forward(w, x, cfg.top_k)
    return cfg, w, x, dict(out=out, idx=idx, w=wt, counts=counts, digest=np.array(input_digest(w, x)))


if __name__ == "__main__":
    for name in GOLDEN:
        _cfg, _w, _x, fx = make(name)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **fx)
        print(name, fx["out"].shape, fx["counts"].tolist())
