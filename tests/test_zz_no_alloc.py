"""GPU: noor_moe_route_static, the routing entry point that allocates nothing.

Some callers cannot call cudaMalloc: code recording a CUDA graph (allocation
is not allowed while a stream is captured) and hosts that hand all device
memory to their own pool at start-up.  noor_moe_route_static serves them by
running the router out of one fixed device array in the library.  This file
checks, through the C ABI, that two calls in a row give the same picks,
weights and counts as the handle-based noor_moe_route and as the CPU oracle's
router (picks and counts exact up to score ties, the parity tests' rule),
that no count comes back as -1 (the entry point's in-band report of a device
wait that gave up), that the free device memory does not change, and that a
batch too big for the array is refused.  It is named so that pytest collects
it last.
"""
import numpy as np
import pytest

from tests import parity

pytestmark = pytest.mark.gpu


def _setup(pkg, cfg):
    import torch
    W = pkg.workloads
    w = W.make_weights(cfg)
    x = W.make_tokens(cfg)
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                       max_tokens=cfg.tokens)
    h.load_weights(w)
    dev = torch.device("cuda", 0)
    if cfg.dtype == W.BF16:
        xd = torch.from_numpy(W.bf16_bits(x).view(np.int16)).to(dev)
        epad = (cfg.n_experts + 7) // 8 * 8
        gt = np.zeros((epad, cfg.d_model), np.uint16)
        gt[:cfg.n_experts] = W.bf16_bits(np.ascontiguousarray(w.gate.T))
        gate = torch.from_numpy(gt.view(np.int16)).to(dev)
    else:
        xd = torch.from_numpy(x).to(dev)
        gate = torch.from_numpy(w.gate).to(dev)
    bias = torch.from_numpy(w.bias).to(dev)
    scales = torch.from_numpy(w.scales).to(dev)
    return w, x, h, xd, gate, bias, scales


def _route_static(pkg, cfg, xd, gate, bias, scales, T):
    """Calls the entry point with outputs allocated beforehand, and returns
    the free device memory seen just before and just after the call."""
    import torch
    k = min(cfg.top_k, cfg.n_experts)
    idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    wt = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    counts = torch.full((cfg.n_experts,), -7, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream()
    s.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    pkg.api.route_static(xd.data_ptr(), gate.data_ptr(), bias.data_ptr(), scales.data_ptr(), T, cfg.d_model,
                         cfg.n_experts, cfg.top_k, cfg.dtype, idx.data_ptr(), wt.data_ptr(), counts.data_ptr(),
                         s.cuda_stream)
    s.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    return idx.cpu().numpy(), wt.cpu().numpy(), counts.cpu().numpy(), (free_before, free_after)


def _check_oracle(pkg, oracle, cfg, w, x, idx, wt, counts):
    """Picks, weights and counts against the oracle's router on the same tokens."""
    W = pkg.workloads
    ridx, _rw, rcounts, rscores = oracle.route(x, w.gate, w.bias, w.scales, cfg.top_k, want_scores=True)
    tau = parity.TAU_BF16 if cfg.dtype == W.BF16 else parity.TAU_F32
    rep = parity.compare_routing(idx, wt, ridx, rscores, w.scales, tau)
    assert rep["unexplained"] == [], rep
    assert rep["max_score_err"] <= tau / 2, rep
    assert rep["tokens_differ"] <= max(2, x.shape[0] // 500), rep
    assert parity.counts_consistent(counts, rcounts, rep["tokens_differ"], idx.shape[1]), (counts, rcounts)


@pytest.mark.parametrize("name", ["edge", "proxy_tiny"])
def test_route_static_matches_route_twice(pkg, oracle, name):
    import torch
    W = pkg.workloads
    cfg = W.CONFIGS[name].with_tokens(3000)
    w, x, h, xd, gate, bias, scales = _setup(pkg, cfg)
    xin = W.bf16_bits(x) if cfg.dtype == W.BF16 else x
    # the routing tolerance of the parity tests: picks and counts exact, weights
    # within half the tie threshold
    tol = (parity.TAU_BF16 if cfg.dtype == W.BF16 else parity.TAU_F32) / 2
    # first call: all 3000 tokens
    idx_ref, w_ref, c_ref = h.route_host(xin)
    idx, wt, counts, mem1 = _route_static(pkg, cfg, xd, gate, bias, scales, cfg.tokens)
    assert (counts >= 0).all(), counts  # -1 would report a device wait that gave up
    assert np.array_equal(idx, idx_ref)
    np.testing.assert_allclose(wt, w_ref, rtol=0, atol=tol)
    assert np.array_equal(counts, c_ref)
    _check_oracle(pkg, oracle, cfg, w, x, idx, wt, counts)
    # second call right after, on a shorter batch: the array still holds the
    # first call's contents and must not leak into the result
    lo, hi = 1000, 1777
    idx_ref2, w_ref2, c_ref2 = h.route_host(np.ascontiguousarray(xin[lo:hi]))
    idx2, wt2, counts2, mem2 = _route_static(pkg, cfg, xd[lo:hi].contiguous(), gate, bias, scales, hi - lo)
    assert (counts2 >= 0).all(), counts2
    assert np.array_equal(idx2, idx_ref2)
    np.testing.assert_allclose(wt2, w_ref2, rtol=0, atol=tol)
    assert np.array_equal(counts2, c_ref2)
    _check_oracle(pkg, oracle, cfg, w, x[lo:hi], idx2, wt2, counts2)
    assert int(counts2.sum()) == (hi - lo) * min(cfg.top_k, cfg.n_experts)
    assert mem1[0] == mem1[1] and mem2[0] == mem2[1]  # no device allocation inside the call
    h.close()


def test_route_static_rejects_oversized_batch(pkg):
    import torch
    W = pkg.workloads
    cfg = W.CONFIGS["edge"].with_tokens(64)
    _w, _x, h, xd, gate, bias, scales = _setup(pkg, cfg)
    T = 1000000  # needs more than the fixed 8 MiB scratch; refused before any launch
    with pytest.raises(pkg.api.NoorMoEError) as e:
        pkg.api.route_static(xd.data_ptr(), gate.data_ptr(), bias.data_ptr(), scales.data_ptr(), T, cfg.d_model,
                             cfg.n_experts, cfg.top_k, cfg.dtype, xd.data_ptr(), xd.data_ptr(), xd.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    assert e.value.code == 1 and "scratch" in str(e.value)
    h.close()
