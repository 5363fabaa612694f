"""Small odd-shape cases through the bounds-checked debug build.

Run as a child process with NOOR_MOE_CHECK=1 (tests/test_gpu_check.py), so
that the library loaded is libnoor_moe_check.so: every data-dependent row
index the kernels use is checked against its buffer, and a failed check comes
back from the call as NOOR_MOE_ERR_INVALID.  Each case must pass its checks
and match the CPU oracle within the parity tolerances.  Prints one JSON line.
"""
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    assert os.environ.get("NOOR_MOE_CHECK") == "1", "run with NOOR_MOE_CHECK=1"
    pkg = importlib.import_module("noor_-_bangla_ai_b200")
    from oracle import oracle as O
    from tests import parity
    W = pkg.workloads
    assert pkg.api.LIB_PATH.endswith("libnoor_moe_check.so")
    cases = []
    for T in (1, 2, 127, 129, 1000):
        cases.append((W.LayerConfig(f"b{T}", T, 256, 16, 4, 128, 256, W.BF16, seed=21, x_dist="rmsnorm",
                                    bias_dist="uniform0.1", has_shared=True), 2e-2, True))
        cases.append((W.LayerConfig(f"f{T}", T, 64, 8, 2, 96, 64, W.F32, seed=22, has_shared=True), 1e-5, True))
    cases.append((W.LayerConfig("kE", 300, 256, 8, 8, 256, 256, W.BF16, seed=23, x_dist="rmsnorm"), 2e-2, True))
    cases.append((W.LayerConfig("E128k8", 700, 256, 128, 8, 256, 256, W.BF16, seed=24, x_dist="rmsnorm",
                                bias_dist="uniform0.1"), 2e-2, True))
    cases.append((W.LayerConfig("d384", 333, 384, 16, 2, 128, 384, W.BF16, seed=25, x_dist="rmsnorm"), 2e-2, True))
    cases.append((W.LayerConfig("nodense", 500, 256, 16, 4, 128, 256, W.BF16, seed=26, x_dist="rmsnorm"), 2e-2,
                  False))
    report = []
    for cfg, tol, dense in cases:
        w = W.make_weights(cfg)
        x = W.make_tokens(cfg)
        h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff,
                           has_shared=cfg.has_shared, has_dense=dense, dtype=cfg.dtype, max_tokens=64)
        h.load_weights(w)
        xin = W.bf16_bits(x) if cfg.dtype == W.BF16 else x
        out, idx, wt, counts = h.forward_host(xin)  # raises NoorMoEError if a check failed
        h.sync()
        if cfg.dtype == W.BF16:
            out = (out.astype(np.uint32) << np.uint32(16)).view(np.float32)
        ref = (O.parallel_forward if dense else O.moe_forward)(w, x, cfg.top_k)[0]
        err = parity.rel_l2(out, ref)
        report.append({"case": cfg.name, "rel_l2": err, "ok": bool(err <= tol and counts.sum() == x.shape[0] *
                                                                       min(cfg.top_k, cfg.n_experts))})
        h.close()
    ok = all(r["ok"] for r in report)
    print(json.dumps({"ok": ok, "cases": report}), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
