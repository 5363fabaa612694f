"""The MoE block's FFN sublayer with its sandwich norm (block.rs:87-90,
norm.rs:31-60) through noor_moe_ffn_sublayer_forward, against the oracle's
composition of rms_norm (tensor.rs:462-490) and ParallelFFN::forward.

Tolerances (written here, checked below):
  F32 layers   output rel-L2 <= 1e-5
  BF16 layers  output rel-L2 <= 2e-2
  routing of the normalised input: exact picks except ties (the router rule)
"""
import numpy as np
import pytest

from tests import parity

pytestmark = pytest.mark.gpu

TOL = {0: 1e-5, 1: 2e-2}  # by dtype: F32, BF16


def _io(cfg, pkg, x):
    return pkg.workloads.bf16_bits(x) if cfg.dtype == pkg.workloads.BF16 else np.ascontiguousarray(x, np.float32)


def _back(cfg, pkg, y):
    if cfg.dtype == pkg.workloads.BF16:
        return (y.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return y


@pytest.mark.parametrize("name,tokens,layer_idx", [("proxy_tiny", 300, 0), ("edge", 512, 3), ("edge", 129, 15)])
def test_sublayer_matches_oracle(pkg, oracle, name, tokens, layer_idx):
    W = pkg.workloads
    cfg = W.CONFIGS[name].with_tokens(tokens)
    w = W.make_weights(cfg)
    rng = np.random.default_rng(11 + layer_idx)
    pre_w = (1.0 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32)
    post_w = (1.0 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32)
    eps = 1e-6
    ds = float(np.float32(1.0) / np.sqrt(np.float32(layer_idx + 1)))
    # the residual stream: not normalised, a few times larger than unit RMS
    x = (3.0 * W.make_tokens(cfg)).astype(np.float32)
    if cfg.dtype == W.BF16:
        x = W.bf16_round(x)
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                       max_tokens=tokens)
    h.load_weights(w)
    with pytest.raises(pkg.api.NoorMoEError):
        h.ffn_sublayer_host(_io(cfg, pkg, x))  # before set_sandwich
    h.set_sandwich(pre_w, post_w, eps, ds)
    out, idx, wt, counts = h.ffn_sublayer_host(_io(cfg, pkg, x))
    ref, ridx, rwt, rcounts, xn = oracle.ffn_sublayer_forward(w, x, cfg.top_k, pre_w, post_w, eps, ds,
                                                              cfg.dtype == W.BF16)
    _, _, _, rscores = oracle.route(xn, w.gate, w.bias, w.scales, cfg.top_k, want_scores=True)
    tau = parity.TAU_BF16 if cfg.dtype == W.BF16 else parity.TAU_F32
    rep = parity.compare_routing(idx, wt, ridx, rscores, w.scales, tau)
    assert rep["unexplained"] == [], rep
    got = _back(cfg, pkg, out)
    err = parity.rel_l2(got, ref)
    assert err <= TOL[cfg.dtype], err
    assert int(counts.sum()) == tokens * idx.shape[1]
    h.close()


def test_sublayer_mirror_api(pkg):
    """The mirror classes: SandwichNorm + ParallelFFN through ffn_sublayer_forward."""
    rng = np.random.default_rng(3)
    pffn = pkg.ParallelFFN(256, 512, 256, 8, 2, False, 0.02, dtype=pkg.api.DTYPE_BF16, rng=rng)
    norm = pkg.SandwichNorm(256, 1e-6, layer_idx=1)
    assert norm.depth_scale == np.float32(1.0) / np.sqrt(np.float32(2.0))
    hid = rng.standard_normal((64, 256)).astype(np.float32)
    out = pkg.ffn_sublayer_forward(pffn, norm, hid)
    assert out.shape == hid.shape and np.isfinite(out).all()
    assert pffn.moe.utilization.total_tokens == 64
