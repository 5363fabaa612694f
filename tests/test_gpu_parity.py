"""Parity of the CUDA path (through the C ABI) against the CPU oracle.

Tolerances (written here, checked below):
  F32 layers   output rel-L2 <= 1e-5, router picks exact except ties (TAU_F32)
  BF16 layers  output rel-L2 <= 2e-2, router picks exact except ties (TAU_BF16)
At the full sizes of the Edge-like, skewed and Pro-like layers the oracle runs
on a sample of tokens (the layer is token-wise, so those output rows are exact
references) and the router on every token; size-independent properties
(permutation equivariance, batch splitting, count sums) cover the rest.
"""
import json
import os

import numpy as np
import pytest

from tests import parity
from tests.golden import make_golden

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_BF16 = 2e-2
HERE = os.path.dirname(os.path.abspath(__file__))


def _io(cfg, pkg, x):
    return pkg.workloads.bf16_bits(x) if cfg.dtype == pkg.workloads.BF16 else np.ascontiguousarray(x, np.float32)


def _back(cfg, pkg, y):
    if cfg.dtype == pkg.workloads.BF16:
        return (y.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return y


def _handle(pkg, cfg, w, tokens, has_dense=True):
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff,
                       has_shared=cfg.has_shared, has_dense=has_dense, dtype=cfg.dtype, max_tokens=tokens)
    h.load_weights(w)
    return h


def _tau(cfg, pkg):
    return parity.TAU_BF16 if cfg.dtype == pkg.workloads.BF16 else parity.TAU_F32


def _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts):
    ridx, rw, rcounts, rscores = oracle.route(x, w.gate, w.bias, w.scales, cfg.top_k, want_scores=True)
    tau = _tau(cfg, pkg)
    rep = parity.compare_routing(idx, wt, ridx, rscores, w.scales, tau)
    assert rep["unexplained"] == [], rep
    assert rep["max_score_err"] <= tau / 2, rep
    assert rep["tokens_differ"] <= max(2, x.shape[0] // 500), rep
    assert parity.counts_consistent(counts, rcounts, rep["tokens_differ"], idx.shape[1]), (counts, rcounts)
    assert int(counts.sum()) == x.shape[0] * idx.shape[1]
    return ridx, rep


# ------------------------------------------------------------ matmul boundary

def test_matmul_known_answers(pkg):
    kat = json.load(open(os.path.join(HERE, "golden", "reference_kat.json")))
    c = kat["matmul_2x2"]
    got = pkg.matmul_f32(np.array(c["a"], np.float32), np.array(c["b"], np.float32))
    assert np.allclose(got, np.array(c["c"]), atol=c["tol"])
    c = kat["matmul_ones_2x3x4"]
    got = pkg.matmul_f32(np.ones((c["m"], c["k"]), np.float32), np.ones((c["k"], c["n"]), np.float32))
    assert np.all(np.abs(got - c["value"]) < c["tol"])
    c = kat["matmul_dispatch_large"]
    a = (np.arange(c["m"] * c["k"], dtype=np.float32) * np.float32(c["a_step"])).reshape(c["m"], c["k"])
    b = (np.arange(c["k"] * c["n"], dtype=np.float32) * np.float32(c["b_step"])).reshape(c["k"], c["n"])
    got = pkg.matmul_f32(a, b)
    exp = np.float32(0)
    for i in range(c["k"]):
        exp += a[0, i] * b[i, 0]
    assert abs(got[0, 0] - exp) < c["tol"]
    c = kat["tiled_matmul_large"]
    rng = np.random.default_rng(0)
    a = (rng.standard_normal((c["m"], c["k"])) * c["std"]).astype(np.float32)
    b = (rng.standard_normal((c["k"], c["n"])) * c["std"]).astype(np.float32)
    got = pkg.matmul_f32(a, b)
    for i in (0, c["m"] // 2, c["m"] - 1):
        for j in (0, c["n"] // 2, c["n"] - 1):
            assert abs(got[i, j] - float(np.dot(a[i].astype(np.float64), b[:, j]))) < c["tol"]


def test_matmul_matches_oracle_ragged(pkg, oracle):
    rng = np.random.default_rng(1)
    for (m, k, n) in [(1, 1, 1), (3, 5, 7), (65, 33, 129), (200, 300, 100)]:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        assert parity.rel_l2(pkg.matmul_f32(a, b), oracle.matmul(a, b)) < 1e-6


# ------------------------------------------------------------ golden fixtures

@pytest.mark.parametrize("name", sorted(make_golden.GOLDEN))
def test_golden_fixture(pkg, oracle, name):
    cfg = make_golden.GOLDEN[name]
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)
    fx = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    assert str(fx["digest"]) == make_golden.input_digest(w, x), "seeded inputs changed"
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    out = _back(cfg, pkg, out)
    tol = TOL_BF16 if cfg.dtype == pkg.workloads.BF16 else TOL_F32
    assert parity.rel_l2(out, fx["out"]) <= tol
    _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts)
    h.close()


# ------------------------------------------------------------ full configs

def test_proxy_tiny_full(pkg, oracle):
    cfg = pkg.workloads.CONFIGS["proxy_tiny"]
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    ref, ridx, rw, rcounts = oracle.parallel_forward(w, x, cfg.top_k)
    assert parity.rel_l2(out, ref) <= TOL_F32
    _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts)
    # MoELayer::forward alone (no dense branch, no 1/sqrt 2)
    hm = _handle(pkg, cfg, w, cfg.tokens, has_dense=False)
    out_m, _, _, _ = hm.forward_host(_io(cfg, pkg, x[:256]))
    ref_m, _, _, _ = oracle.moe_forward(w, x[:256], cfg.top_k)
    assert parity.rel_l2(out_m, ref_m) <= TOL_F32
    h.close()
    hm.close()


def _sampled_rows(T, n, seed=0):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(T, size=min(n, T), replace=False))


@pytest.mark.parametrize("name,tokens,sample", [("edge", None, 48), ("edge_skewed", None, 32), ("pro", None, 32),
                                                ("max_layer", None, 32)])
def test_bf16_config_sampled(pkg, oracle, name, tokens, sample):
    """Every config at its full size: the router on every token against the
    oracle, sampled output rows against the oracle's forward of those rows.
    max_layer (E = 128, k = 8) sits at the BF16 router's limits: 128 TMEM
    columns read in four 32-column loads, and the largest top-k."""
    cfg = pkg.workloads.CONFIGS[name]
    if tokens is not None:
        cfg = cfg.with_tokens(tokens)
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    out = _back(cfg, pkg, out)
    ridx, rep = _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts)
    rows = _sampled_rows(cfg.tokens, sample)
    oracle.use_openblas()
    try:
        ref, _, _, _ = oracle.parallel_forward(w, x[rows], cfg.top_k)
    finally:
        oracle.use_plain_loops()
    assert parity.rel_l2(out[rows], ref) <= TOL_BF16
    assert np.isfinite(out).all()
    if name == "edge_skewed":
        share = np.isin(idx, w.hot_experts).mean()
        assert 0.55 <= share <= 0.65, share
    h.close()


# ------------------------------------------------------------ properties at full size

def test_edge_permutation_and_split(pkg):
    cfg = pkg.workloads.CONFIGS["edge"]
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)
    xb = _io(cfg, pkg, x)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(xb)
    perm = np.random.default_rng(3).permutation(cfg.tokens)
    out_p, idx_p, wt_p, counts_p = h.forward_host(np.ascontiguousarray(xb[perm]))
    assert np.array_equal(out_p, out[perm])          # token-wise layer: bit-exact
    assert np.array_equal(idx_p, idx[perm])
    assert np.array_equal(counts_p, counts)
    cut = 5000
    o1, _, _, c1 = h.forward_host(np.ascontiguousarray(xb[:cut]))
    o2, _, _, c2 = h.forward_host(np.ascontiguousarray(xb[cut:]))
    assert np.array_equal(np.concatenate([o1, o2]), out)
    assert np.array_equal(c1 + c2, counts)
    h.close()


@pytest.mark.parametrize("name,tokens", [("edge", 6000), ("max_layer", 3000)])
def test_repeat_calls_bit_identical(pkg, name, tokens):
    """The router's blocks claim their rows of each expert's segment with
    atomics, so the row order inside a segment changes from call to call;
    every row is computed on its own and returns to its token through the row
    map, so outputs, picks and counts must not change at all."""
    cfg = pkg.workloads.CONFIGS[name].with_tokens(tokens)
    w = pkg.workloads.make_weights(cfg)
    xb = _io(cfg, pkg, pkg.workloads.make_tokens(cfg))
    h = _handle(pkg, cfg, w, cfg.tokens)
    first = h.forward_host(xb)
    for _ in range(3):
        again = h.forward_host(xb)
        for a, b in zip(first, again):
            assert np.array_equal(a, b)
    h.close()


def test_device_mode_matches_host_mode(pkg):
    import torch
    cfg = pkg.workloads.CONFIGS["edge"].with_tokens(3000)
    w = pkg.workloads.make_weights(cfg)
    x = pkg.workloads.make_tokens(cfg)
    xb = _io(cfg, pkg, x)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out_h, idx_h, wt_h, cnt_h = h.forward_host(xb)
    xd = torch.from_numpy(xb.view(np.int16)).cuda()
    od = torch.empty_like(xd)
    idx_d = torch.empty((cfg.tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    w_d = torch.empty((cfg.tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    c_d = torch.empty(cfg.n_experts, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream()
    h.forward_device(xd.data_ptr(), od.data_ptr(), cfg.tokens, s.cuda_stream, idx_d.data_ptr(), w_d.data_ptr(),
                     c_d.data_ptr())
    h.sync(s.cuda_stream)
    assert np.array_equal(od.cpu().numpy().view(np.uint16), out_h)
    assert np.array_equal(idx_d.cpu().numpy(), idx_h)
    assert np.array_equal(c_d.cpu().numpy(), cnt_h)
    h.close()


# ------------------------------------------------------------ edge cases

@pytest.mark.parametrize("T", [1, 2, 127, 129, 1000])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_ragged_token_counts(pkg, oracle, T, dt):
    W = pkg.workloads
    if dt == "f32":
        cfg = W.LayerConfig("r32", T, 64, 8, 2, 96, 64, W.F32, seed=11, has_shared=True)
        tol = TOL_F32
    else:
        cfg = W.LayerConfig("r16", T, 256, 16, 4, 128, 256, W.BF16, seed=12, x_dist="rmsnorm",
                            bias_dist="uniform0.1", has_shared=True)
        tol = TOL_BF16
    w = W.make_weights(cfg)
    x = W.make_tokens(cfg)
    h = _handle(pkg, cfg, w, 64)   # workspace grows on demand
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    ref, _, _, _ = oracle.parallel_forward(w, x, cfg.top_k)
    assert parity.rel_l2(_back(cfg, pkg, out), ref) <= tol
    _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts)
    h.close()


def test_zero_tokens(pkg):
    W = pkg.workloads
    cfg = W.LayerConfig("z", 0, 128, 8, 2, 128, 128, W.BF16, seed=1)
    w = W.make_weights(cfg)
    h = _handle(pkg, cfg, w, 128)
    out, idx, wt, counts = h.forward_host(np.zeros((0, 128), np.uint16))
    assert out.shape == (0, 128) and counts.sum() == 0
    h.close()


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_empty_and_hot_experts(pkg, oracle, dt):
    """Experts that receive no tokens, and one expert that receives every token."""
    W = pkg.workloads
    dtype = W.F32 if dt == "f32" else W.BF16
    cfg = W.LayerConfig("hot", 700, 128, 16, 2, 128, 128, dtype, seed=13, x_dist="rmsnorm")
    w = W.make_weights(cfg)
    w.bias = np.full(cfg.n_experts, -50.0, np.float32)
    w.bias[5] = 50.0     # every token picks expert 5 first
    w.bias[9] = 0.0      # and expert 9 second; 14 experts stay empty
    x = W.make_tokens(cfg)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    assert counts[5] == cfg.tokens and counts[9] == cfg.tokens and counts.sum() == 2 * cfg.tokens
    ref, ridx, _, _ = oracle.parallel_forward(w, x, cfg.top_k)
    assert np.array_equal(idx, ridx)
    assert parity.rel_l2(_back(cfg, pkg, out), ref) <= (TOL_BF16 if dt == "bf16" else TOL_F32)
    h.close()


def test_top_k_equals_experts(pkg, oracle):
    W = pkg.workloads
    cfg = W.LayerConfig("kE", 300, 64, 8, 8, 64, 64, W.F32, seed=14)
    w = W.make_weights(cfg)
    x = W.make_tokens(cfg)
    h = _handle(pkg, cfg, w, cfg.tokens)
    out, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
    ref, ridx, _, _ = oracle.parallel_forward(w, x, cfg.top_k)
    assert parity.rel_l2(out, ref) <= TOL_F32
    assert np.all(counts == cfg.tokens)
    h.close()


def test_set_bias_reroutes(pkg, oracle):
    """SMEBU's apply_to_router path: a new bias changes the routing exactly as
    the oracle predicts."""
    W = pkg.workloads
    cfg = W.CONFIGS["proxy_tiny"].with_tokens(512)
    w = W.make_weights(cfg)
    x = W.make_tokens(cfg)
    h = _handle(pkg, cfg, w, cfg.tokens)
    new_bias = np.linspace(-0.5, 0.5, cfg.n_experts).astype(np.float32)
    h.set_bias(new_bias)
    idx, wt, counts = h.route_host(_io(cfg, pkg, x))
    w.bias = new_bias
    _check_routing(pkg, oracle, cfg, w, x, idx, wt, counts)
    h.close()


def test_errors_are_status_codes(pkg):
    api = pkg.api
    with pytest.raises(api.NoorMoEError) as e:
        api.Handle(100, 8, 2, 128, 128, dtype=api.DTYPE_BF16)  # d_model not a multiple of 128
    assert e.value.code == 7
    with pytest.raises(api.NoorMoEError) as e:
        api.Handle(128, 6, 2, 128, 128, dtype=api.DTYPE_BF16, world_size=4, rank=0)  # E % G != 0
    assert e.value.code == 1
    h = api.Handle(128, 8, 2, 128, 128, dtype=api.DTYPE_BF16)
    with pytest.raises(api.NoorMoEError) as e:
        h.forward_host(np.zeros((4, 128), np.uint16))
    assert e.value.code == 5
    h.close()


# ------------------------------------------------------------ reference structural tests, through the mirror

def test_reference_router_tests(pkg):
    kat = json.load(open(os.path.join(HERE, "golden", "reference_kat.json")))
    rng = np.random.default_rng(5)
    c = kat["router_k_indices"]
    moe = pkg.MoELayer(c["d"], 32, c["E"], c["k"], False, c["init_std"] * 2, rng=rng)
    r = moe.router.route(np.full(c["d"], c["x_const"], np.float32))
    assert len(r.indices) == c["k"] and len(r.weights) == c["k"]
    c = kat["router_indices_in_range"]
    moe = pkg.MoELayer(c["d"], 32, c["E"], c["k"], False, c["init_std"] * 2, rng=rng)
    r = moe.router.route(rng.standard_normal(c["d"]).astype(np.float32))
    assert all(0 <= i < c["E"] for i in r.indices)
    c = kat["router_weights_positive"]
    moe = pkg.MoELayer(c["d"], 32, c["E"], c["k"], False, c["init_std"] * 2, rng=rng)
    r = moe.router.route(rng.standard_normal(c["d"]).astype(np.float32))
    assert all(v > 0 for v in r.weights)


def test_reference_layer_tests(pkg):
    kat = json.load(open(os.path.join(HERE, "golden", "reference_kat.json")))
    rng = np.random.default_rng(6)
    c = kat["moe_layer_shape"]
    moe = pkg.MoELayer(c["d"], c["ff"], c["E"], c["k"], c["has_shared"], c["std"], rng=rng)
    assert moe.forward(rng.standard_normal((c["T"], c["d"])).astype(np.float32)).shape == (c["T"], c["d"])
    c = kat["utilization_tracking"]
    moe = pkg.MoELayer(c["d"], c["ff"], c["E"], c["k"], c["has_shared"], c["std"], rng=rng)
    moe.forward(rng.standard_normal((c["T"], c["d"])).astype(np.float32))
    assert moe.utilization.total_tokens == c["T"]
    assert sum(moe.utilization.counts) == c["total"]
    assert moe.utilization.active_expert_count() >= c["min_active"]
    c = kat["parallel_ffn_shape"]
    p = pkg.ParallelFFN(c["d"], c["dff"], c["ff"], c["E"], c["k"], c["has_shared"], c["std"], rng=rng)
    assert p.forward(rng.standard_normal((c["T"], c["d"])).astype(np.float32)).shape == (c["T"], c["d"])
    c = kat["parallel_ffn_scaling"]
    p = pkg.ParallelFFN(c["d"], c["dff"], c["ff"], c["E"], c["k"], c["has_shared"], c["std"], rng=rng)
    x = (rng.standard_normal((c["T"], c["d"])) * c["x_std"]).astype(np.float32)
    out = p.forward(x)
    assert float((out ** 2).mean()) < float((x ** 2).mean()) * c["var_ratio_lt"]
