"""CPU: the oracle against the reference's own known-answer tests, the
independent numpy restatement, and the golden fixtures."""
import json
import os

import numpy as np
import pytest

from tests import parity
from tests.golden import make_golden

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "reference_kat.json")))


def test_matmul_kats(oracle):
    c = KAT["matmul_2x2"]
    assert np.allclose(oracle.matmul(c["a"], c["b"]), c["c"], atol=c["tol"])
    c = KAT["matmul_ones_2x3x4"]
    got = oracle.matmul(np.ones((c["m"], c["k"])), np.ones((c["k"], c["n"])))
    assert np.all(np.abs(got - c["value"]) < c["tol"])
    c = KAT["tiled_matmul_large"]
    rng = np.random.default_rng(0)
    a = (rng.standard_normal((c["m"], c["k"])) * c["std"]).astype(np.float32)
    b = (rng.standard_normal((c["k"], c["n"])) * c["std"]).astype(np.float32)
    got = oracle.matmul(a, b)
    for i in (0, c["m"] // 2, c["m"] - 1):
        for j in (0, c["n"] // 2, c["n"] - 1):
            assert abs(got[i, j] - float(a[i].astype(np.float64) @ b[:, j])) < c["tol"]


def test_matmul_openblas_route_agrees(oracle):
    if not oracle.use_openblas():
        pytest.skip("numpy's OpenBLAS not found")
    try:
        c = KAT["matmul_2x2"]
        assert np.allclose(oracle.matmul(c["a"], c["b"]), c["c"], atol=c["tol"])
        rng = np.random.default_rng(1)
        a = rng.standard_normal((37, 61)).astype(np.float32)
        b = rng.standard_normal((61, 29)).astype(np.float32)
        blas = oracle.matmul(a, b)
    finally:
        oracle.use_plain_loops()
    assert parity.rel_l2(blas, oracle.matmul(a, b)) < 1e-6


def test_elementwise_kats(oracle):
    for x, y, tol in KAT["sigmoid"]["cases"]:
        assert abs(oracle.sigmoid(x) - y) < tol
    for x, y, tol in KAT["silu"]["cases"]:
        assert abs(oracle.silu(x) - y) < tol
    c = KAT["silu_dispatch_bounds"]
    assert abs(oracle.silu(0.0)) < c["zero_tol"]
    for x, lb in c["gt"]:
        assert oracle.silu(x) > lb
    c = KAT["gelu"]
    assert abs(oracle.gelu(0.0)) < c["zero_tol"]
    for x, lb in c["gt"]:
        assert oracle.gelu(x) > lb
    for x, ub in c["lt"]:
        assert oracle.gelu(x) < ub


def test_bf16_kats(oracle, pkg):
    c = KAT["bf16_roundtrip"]
    for v in c["values"]:
        back = oracle.bf16_to_f32(oracle.f32_to_bf16(v))
        err = abs((back - v) / v) if abs(v) > 1e-6 else abs(back - v)
        assert err < c["rel_tol"]
    assert oracle.bf16_to_f32(oracle.f32_to_bf16(0.0)) == 0.0
    nz = np.float32(oracle.bf16_to_f32(oracle.f32_to_bf16(-0.0)))
    assert nz.view(np.uint32) == np.float32(-0.0).view(np.uint32)
    assert np.isinf(oracle.bf16_to_f32(oracle.f32_to_bf16(float("inf"))))
    assert np.isnan(oracle.bf16_to_f32(oracle.f32_to_bf16(float("nan"))))
    # the vectorised generator rounding equals the oracle's scalar RNE
    rng = np.random.default_rng(2)
    v = np.concatenate([rng.standard_normal(10000).astype(np.float32),
                        np.array([1.00390625, 1.01171875, -3.0e38, 1e-40], np.float32)])
    assert np.array_equal(pkg.workloads.bf16_round(v), oracle.round_bf16(v))


def test_rms_norm_kat(oracle, pkg):
    c = KAT["rms_norm"]
    x = np.array(c["x"], np.float32)
    out = oracle.rms_norm(x, np.ones(2, np.float32), c["eps"])
    rms = np.sqrt((out.astype(np.float64) ** 2).mean(axis=1))
    assert np.all(np.abs(rms - 1.0) < c["rms_tol"])
    rng = np.random.default_rng(3)
    y = rng.standard_normal((17, 64)).astype(np.float32)
    assert np.array_equal(pkg.workloads.rms_norm_rows(y, 1e-6), oracle.rms_norm(y, np.ones(64, np.float32), 1e-6))


def _smebu(oracle, c, fractions):
    m = np.zeros(c["n"], np.float32)
    b = np.zeros(c["n"], np.float32)
    for _ in range(c["steps"]):
        oracle.smebu_update(m, b, fractions, c["kappa"], c["beta"], c["lambda"])
    return b


def test_smebu_kats(oracle, pkg):
    c = KAT["smebu_balanced"]
    b = _smebu(oracle, c, np.full(c["n"], 1.0 / c["n"], np.float32))
    assert np.all(np.abs(b) < c["bias_abs_lt"])
    c = KAT["smebu_imbalanced"]
    b = _smebu(oracle, c, np.array(c["fractions"], np.float32))
    assert b[0] < c["b0_lt"] and b[1] > c["b1_gt"] and b[2] > c["b2_gt"]
    c = KAT["smebu_clamped"]
    b = _smebu(oracle, c, np.array(c["fractions"], np.float32))
    assert np.all(np.abs(b) <= c["abs_le"])
    # the host mirror follows the same arithmetic
    s = pkg.SMEBU(c["n"], c["kappa"], c["beta"], c["lambda"])
    m = np.zeros(c["n"], np.float32)
    bo = np.zeros(c["n"], np.float32)
    for _ in range(50):
        s.update(c["fractions"])
        oracle.smebu_update(m, bo, np.array(c["fractions"], np.float32), c["kappa"], c["beta"], c["lambda"])
    assert np.allclose(s.biases, bo, rtol=1e-6, atol=1e-7)


def test_router_structural(oracle):
    rng = np.random.default_rng(4)
    for name in ("router_k_indices", "router_indices_in_range", "router_weights_positive"):
        c = KAT[name]
        gate = (rng.standard_normal((c["d"], c["E"])) * c["init_std"]).astype(np.float32)
        x = (np.full((1, c["d"]), c.get("x_const", 0.0), np.float32) if "x_const" in c
             else rng.standard_normal((1, c["d"])).astype(np.float32))
        idx, w, counts = oracle.route(x, gate, np.zeros(c["E"], np.float32), np.ones(c["E"], np.float32), c["k"])
        assert idx.shape == (1, c["k"])
        assert np.all((idx >= 0) & (idx < c["E"]))
        assert np.all(w > 0)
        assert counts.sum() == c["k"]


def test_router_tie_break_is_stable(oracle):
    """Equal scores keep ascending expert order (stable descending sort, moe.rs:96-97)."""
    d, E = 4, 6
    gate = np.zeros((d, E), np.float32)
    x = np.ones((1, d), np.float32)
    idx, w, _ = oracle.route(x, gate, np.zeros(E, np.float32), np.ones(E, np.float32), 3)
    assert idx.tolist() == [[0, 1, 2]]
    bias = np.array([0, 0, 1, 0, 1, 0], np.float32)
    idx, w, _ = oracle.route(x, gate, bias, np.ones(E, np.float32), 3)
    assert idx.tolist() == [[2, 4, 0]]


def test_utilization_kat(oracle, pkg):
    c = KAT["utilization_tracking"]
    rng = np.random.default_rng(5)
    gate = (rng.standard_normal((c["d"], c["E"])) * c["std"] * 0.5).astype(np.float32)
    x = rng.standard_normal((c["T"], c["d"])).astype(np.float32)
    _, _, counts = oracle.route(x, gate, np.zeros(c["E"], np.float32), np.ones(c["E"], np.float32), c["k"])
    assert counts.sum() == c["total"]
    u = pkg.ExpertUtilization(c["E"])
    u.record_batch(counts, c["T"])
    assert u.total_tokens == c["T"] and sum(u.counts) == c["total"]
    assert u.active_expert_count() >= c["min_active"]
    u.reset()
    assert u.total_tokens == 0 and sum(u.counts) == 0


def test_param_counts(pkg):
    c = KAT["parallel_ffn_param_count"]
    p = pkg.ParallelFFN(c["d"], c["dff"], c["ff"], c["E"], c["k"], c["has_shared"], 0.02)
    assert p.param_count() == c["expected"]
    c = KAT["geglu_param_count"]
    assert pkg.GeGLUFFN(c["d"], c["ff"], 0.02).param_count() == c["expected"]
    c = KAT["swiglu_param_count"]
    assert pkg.SwiGLUFFN(c["d"], c["ff"], 0.02).param_count() == c["expected"]


def test_oracle_matches_numpy_restatement(oracle, pkg):
    W = pkg.workloads
    for cfg in (W.CONFIGS["proxy_tiny"].with_tokens(256), make_golden.GOLDEN["tiny_f32"],
                make_golden.GOLDEN["tiny_bf16"]):
        w = W.make_weights(cfg)
        x = W.make_tokens(cfg)
        out, idx, wt, counts = oracle.parallel_forward(w, x, cfg.top_k)
        ref, ridx, rw = oracle.np_parallel_forward(w, x, cfg.top_k)
        assert parity.rel_l2(out, ref) < 1e-5
        assert (idx != ridx).any(axis=1).sum() <= 1
        assert counts.sum() == cfg.tokens * cfg.top_k


@pytest.mark.parametrize("name", sorted(make_golden.GOLDEN))
def test_golden_fixtures_reproduce(oracle, name):
    _cfg, _w, _x, fx = make_golden.make(name)
    ref = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    assert str(ref["digest"]) == str(fx["digest"])
    for key in ("out", "idx", "w", "counts"):
        assert np.array_equal(ref[key], fx[key]), key


def test_moe_forward_matches_token_loop_definition(oracle, pkg):
    """MoELayer::forward on a batch equals routing + per-pick SwiGLU + weighted
    sum computed from the oracle's pieces (moe.rs:150-165)."""
    cfg = make_golden.GOLDEN["tiny_f32"]
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)[:5]
    out, idx, wt, _ = oracle.moe_forward(w, x, cfg.top_k)
    for t in range(x.shape[0]):
        acc = np.zeros(cfg.d_model, np.float32)
        for r in range(cfg.top_k):
            e = idx[t, r]
            y = oracle.glu_ffn(x[t:t + 1], w.w_gate[e], w.w_up[e], w.w_down[e], 1)[0]
            acc = (acc + wt[t, r] * y).astype(np.float32)
        acc = (acc + oracle.glu_ffn(x[t:t + 1], w.shared_gate, w.shared_up, w.shared_down, 1)[0]).astype(np.float32)
        assert np.array_equal(acc, out[t])
