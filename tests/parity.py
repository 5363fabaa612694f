"""Comparison helpers shared by the parity tests.

Router parity rule: selected experts and per-expert counts must equal the
oracle's exactly, except on score ties.  A (token, rank) mismatch counts as a
tie when the oracle's own f32 scores of the two experts involved differ by at
most `tau`; each test also checks that the largest observed difference
between the GPU's and the oracle's score of an expert both picked is below
tau / 2, so no flip can come from anything but a near-tie.
"""
from __future__ import annotations

import numpy as np

TAU_F32 = 1e-6   # F32 layers: same-order f32 dot, differences only from expf's last place
TAU_BF16 = 1e-5  # BF16 layers: tensor-core dot, f32 accumulation in another order


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def compare_routing(idx_gpu, w_gpu, idx_ref, scores_ref, scales, tau):
    """Returns a dict: tokens that differ, how many are not explained by ties,
    and the largest |s_gpu - s_ref| over picks both sides agree on."""
    idx_gpu = np.asarray(idx_gpu)
    idx_ref = np.asarray(idx_ref)
    T, k = idx_ref.shape
    diff_tok = np.nonzero((idx_gpu != idx_ref).any(axis=1))[0]
    unexplained = []
    for t in diff_tok:
        for r in range(k):
            a, b = int(idx_gpu[t, r]), int(idx_ref[t, r])
            if a == b:
                continue
            if not (0 <= a < scores_ref.shape[1]) or abs(float(scores_ref[t, a]) - float(scores_ref[t, b])) > tau:
                unexplained.append((int(t), r, a, b))
                break
    same = idx_gpu == idx_ref
    s_gpu = np.asarray(w_gpu, np.float64) / np.asarray(scales, np.float64)[np.clip(idx_gpu, 0, len(scales) - 1)]
    s_ref = np.take_along_axis(np.asarray(scores_ref, np.float64), np.clip(idx_ref, 0, scores_ref.shape[1] - 1), 1)
    max_err = float(np.abs(s_gpu - s_ref)[same].max()) if same.any() else 0.0
    return {"tokens_differ": int(diff_tok.size), "unexplained": unexplained, "max_score_err": max_err}


def counts_consistent(counts_gpu, counts_ref, tokens_differ: int, k: int) -> bool:
    """Counts may only differ by the picks of tie-explained tokens."""
    d = np.abs(np.asarray(counts_gpu, np.int64) - np.asarray(counts_ref, np.int64)).sum()
    return int(d) <= 2 * k * tokens_differ
