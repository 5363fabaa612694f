"""Expert utilization and the SMEBU bias update on the device, against the
oracle's ExpertUtilization / SMEBU::update (smebu.rs:36-48).

Tolerances (written here, checked below):
  utilization counts and tokens     exact
  momentum                          exact (f32 mul/add/div rounded as the reference)
  bias = kappa * tanh(m / kappa)    within 4 ulp of the oracle (CUDA tanhf vs glibc tanhf)
  routing with the new bias         exact picks except ties (the router parity rule)
"""
import numpy as np
import pytest

from tests import parity

pytestmark = pytest.mark.gpu


def _io(cfg, pkg, x):
    return pkg.workloads.bf16_bits(x) if cfg.dtype == pkg.workloads.BF16 else np.ascontiguousarray(x, np.float32)


def _ulp_close(a, b, ulps):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    spacing = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32))
    return bool(np.all(np.abs(a.astype(np.float64) - b.astype(np.float64)) <= ulps * spacing.astype(np.float64)))


@pytest.mark.parametrize("name", ["proxy_tiny", "edge"])
def test_utilization_and_smebu_match_oracle(pkg, oracle, name):
    W = pkg.workloads
    cfg = W.CONFIGS[name].with_tokens(1000)
    w = W.make_weights(cfg)
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                       max_tokens=1024)
    h.load_weights(w)
    kappa, beta, lam = 5.0, 0.9, 0.05
    m_ref = np.zeros(cfg.n_experts, np.float32)
    b_ref = np.zeros(cfg.n_experts, np.float32)
    bias = w.bias.copy()
    for step in range(3):
        total = np.zeros(cfg.n_experts, np.int64)
        tokens = 0
        for part, T in enumerate((1000, 337)):  # two forwards per step, ragged
            x = W.make_tokens(cfg, seed_offset=17 * step + part + 1, tokens=T)
            _, idx, wt, counts = h.forward_host(_io(cfg, pkg, x))
            # the device routed with `bias`: the oracle agrees up to ties
            ridx, _, rcounts, rscores = oracle.route(x, w.gate, bias, w.scales, cfg.top_k, want_scores=True)
            tau = parity.TAU_BF16 if cfg.dtype == W.BF16 else parity.TAU_F32
            rep = parity.compare_routing(idx, wt, ridx, rscores, w.scales, tau)
            assert rep["unexplained"] == [], rep
            total += counts
            tokens += T
        c, t = h.utilization()
        assert np.array_equal(c, total) and t == tokens
        # ExpertUtilization::fractions, then SMEBU::update in the oracle
        fr = (total.astype(np.float32) / np.float32(tokens)).astype(np.float32)
        oracle.smebu_update(m_ref, b_ref, fr, kappa, beta, lam)
        h.smebu_update(kappa, beta, lam)
        m_dev = h.smebu_momentum()
        b_dev = h.get_bias()
        assert np.array_equal(m_dev, m_ref), (m_dev, m_ref)
        assert _ulp_close(b_dev, b_ref, 4), (b_dev, b_ref)
        c2, t2 = h.utilization()
        assert t2 == 0 and not c2.any()  # the update resets the utilization
        bias = b_dev
    h.close()


def test_utilization_reset_and_route_only(pkg):
    W = pkg.workloads
    cfg = W.CONFIGS["edge"].with_tokens(256)
    w = W.make_weights(cfg)
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                       max_tokens=256)
    h.load_weights(w)
    x = _io(cfg, pkg, W.make_tokens(cfg))
    h.route_host(x)  # MoERouter::route does not record
    c, t = h.utilization()
    assert t == 0 and not c.any()
    _, _, _, counts = h.forward_host(x)
    c, t = h.utilization(reset=True)
    assert np.array_equal(c, counts) and t == cfg.tokens
    c, t = h.utilization()
    assert t == 0 and not c.any()
    # no recorded tokens: fractions are all zero (ExpertUtilization::fractions)
    h.smebu_update(5.0, 0.9, 0.01)
    m = h.smebu_momentum()
    ft = np.float32(1.0) / np.float32(cfg.n_experts)
    assert np.array_equal(m, np.full(cfg.n_experts, np.float32(0.01) * ft, np.float32))
    prev = h.smebu_momentum(set_to=np.zeros(cfg.n_experts, np.float32))
    assert np.array_equal(prev, m) and not h.smebu_momentum().any()
    h.close()
