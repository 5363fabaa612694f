"""Seeded synthetic MoE-layer workloads.

The reference measures on no public dataset, so every workload here is
synthetic: a counter-based Philox stream (numpy) draws the inputs and weights
in a fixed order from the listed seed, and the same f32 arrays feed the CUDA
library and the CPU oracle.  For BF16 layers the weights and activations are
rounded to BF16 with the reference's round-to-nearest-even
(crates/noor-core/src/tensor.rs:23-28) before either side sees them, so both
compute on identical values.

Layer shapes follow the reference's `[moe]` config block
(crates/noor-core/src/config.rs:32-39) and `ParallelFFN::new`
(crates/noor-core/src/layers/parallel_ffn.rs:14-27).  Weights use the
reference's row-major layouts: router gate [d, E] (moe.rs:7), expert and
dense w_gate / w_up [d, ff] and w_down [ff, d] (ffn.rs:5-12, 43-50).
"""
from __future__ import annotations

import dataclasses
import math
import os
from concurrent.futures import ThreadPoolExecutor
from typing import Optional

import numpy as np

F32 = 0
BF16 = 1
ACT_GELU_TANH = 0
ACT_SILU = 1


@dataclasses.dataclass(frozen=True)
class LayerConfig:
    name: str
    tokens: int
    d_model: int
    n_experts: int
    top_k: int
    expert_ff: int
    dense_ff: int
    dtype: int
    seed: int
    x_dist: str = "normal"          # "normal" (N(0,1)) or "rmsnorm" (rows with RMS 1)
    bias_dist: str = "zero"         # "zero" or "uniform0.1" (U(-0.1, 0.1))
    has_shared: bool = False
    hot_share: Optional[float] = None  # skewed routing: share of assignments to the hot experts
    hot_fraction: float = 0.25         # fraction of experts that are hot
    weight_std: float = 0.02
    # Large layers: every expert matrix, dense matrix and 4096-row block of x
    # has its own Philox stream (the base stream jumped), so the draws run on
    # all host cores and do not depend on each other's order.
    threaded_draw: bool = False

    def with_tokens(self, tokens: int) -> "LayerConfig":
        return dataclasses.replace(self, tokens=tokens)

    def flops_per_token(self) -> dict:
        d, E, k, ff, dff = self.d_model, self.n_experts, self.top_k, self.expert_ff, self.dense_ff
        out = {
            "router": 2 * d * E,
            "experts": 6 * k * d * ff,
            "dense": 6 * d * dff,
            "shared": 6 * d * ff if self.has_shared else 0,
        }
        out["total"] = sum(out.values())
        return out


CONFIGS = {
    # proxy_tiny MoE layer, FP32, CPU-runnable.
    "proxy_tiny": LayerConfig("proxy_tiny", 2048, 256, 8, 2, 512, 512, F32, seed=0),
    # Edge-like, BF16 weights and activations, FP32 accumulate.
    "edge": LayerConfig("edge", 16384, 2048, 32, 4, 1024, 2048, BF16, seed=0,
                        x_dist="rmsnorm", bias_dist="uniform0.1"),
    # Edge-like with skewed routing: 25% of experts receive 60% of assignments.
    "edge_skewed": LayerConfig("edge_skewed", 65536, 2048, 32, 4, 1024, 2048, BF16, seed=0,
                               x_dist="rmsnorm", bias_dist="uniform0.1", hot_share=0.60),
    # Pro-like, expert-parallel across 1/2/4/8 GPUs.
    "pro": LayerConfig("pro", 131072, 3072, 64, 6, 1536, 3072, BF16, seed=1,
                       x_dist="rmsnorm", bias_dist="uniform0.1", threaded_draw=True),
    # The MoE layer of the Max-like stack (one of its 16 blocks): batch 8 x
    # seq 4096 tokens, d_model 4096, 128 experts top-8.
    "max_layer": LayerConfig("max_layer", 32768, 4096, 128, 8, 1536, 4096, BF16, seed=2,
                             x_dist="rmsnorm", bias_dist="uniform0.1", threaded_draw=True),
}

TOKEN_BLOCK = 4096  # rows of x per Philox stream under threaded_draw


def _pool_map(fn, items):
    items = list(items)
    with ThreadPoolExecutor(max_workers=max(1, min(len(items), os.cpu_count() or 1))) as ex:
        return list(ex.map(fn, items))


def _stream(seed: int, i: int) -> np.random.Generator:
    """Stream i of the threaded draws: the base Philox stream jumped i + 1 times."""
    return np.random.Generator(np.random.Philox(seed).jumped(i + 1))


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round f32 values to the nearest BF16 (ties to even), returned as f32.

    Vectorised form of `f32_to_bf16` then `bf16_to_f32`
    (crates/noor-core/src/tensor.rs:23-33)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32)
    bias = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    r = ((bits + bias) >> np.uint32(16)).astype(np.uint32) << np.uint32(16)
    return r.view(np.float32)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """BF16 bit patterns (uint16) of f32 values, RNE as tensor.rs:23-28."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32)
    bias = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((bits + bias) >> np.uint32(16)).astype(np.uint16)


def rms_norm_rows(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """`rms_norm` with unit weight (tensor.rs:462-490): f64 accumulation,
    each element computed as (x as f64 / rms) as f32."""
    x64 = x.astype(np.float64)
    rms = np.sqrt((x64 * x64).sum(axis=1, keepdims=True) / x.shape[1] + eps)
    return (x64 / rms).astype(np.float32)


@dataclasses.dataclass
class LayerWeights:
    """One ParallelFFN layer in the reference's layouts (all f32, C-contiguous)."""
    gate: np.ndarray          # [d, E]
    bias: np.ndarray          # [E]
    scales: np.ndarray        # [E]
    w_gate: np.ndarray        # [E, d, ff]
    w_up: np.ndarray          # [E, d, ff]
    w_down: np.ndarray        # [E, ff, d]
    dense_gate: np.ndarray    # [d, dff]
    dense_up: np.ndarray      # [d, dff]
    dense_down: np.ndarray    # [dff, d]
    shared_gate: Optional[np.ndarray] = None  # [d, ff]
    shared_up: Optional[np.ndarray] = None
    shared_down: Optional[np.ndarray] = None
    hot_experts: Optional[np.ndarray] = None
    hot_alpha: Optional[float] = None
    hot_share_achieved: Optional[float] = None


def _normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    out = rng.standard_normal(size=shape, dtype=np.float32)
    out *= np.float32(std)
    return out


def _topk_share(x: np.ndarray, gate: np.ndarray, bias: np.ndarray, k: int, hot: np.ndarray) -> float:
    s = x @ gate + bias[None, :]
    top = np.argsort(-s, axis=1, kind="stable")[:, :k]
    return float(np.isin(top, hot).mean())


def _fill_normal(out: np.ndarray, rng: np.random.Generator, std: float, bf16: bool) -> None:
    rng.standard_normal(out=out, dtype=np.float32)
    out *= np.float32(std)
    if bf16:
        out[...] = bf16_round(out)


def make_weights(cfg: LayerConfig, rng: Optional[np.random.Generator] = None) -> LayerWeights:
    """Draw the layer's weights.  Order of draws: router gate, bias, experts
    (gate, up, down per expert), shared expert, dense branch.  Under
    cfg.threaded_draw the gate and bias come from the base stream and every
    larger matrix from its own stream: expert e's gate, up and down from
    streams 3e, 3e+1, 3e+2, then the dense and shared matrices."""
    if rng is None:
        rng = np.random.Generator(np.random.Philox(cfg.seed))
    d, E, ff, dff, std = cfg.d_model, cfg.n_experts, cfg.expert_ff, cfg.dense_ff, cfg.weight_std
    gate = _normal(rng, (d, E), std)
    if cfg.bias_dist == "zero":
        bias = np.zeros(E, np.float32)
    else:
        bias = rng.uniform(-0.1, 0.1, size=E).astype(np.float32)
    scales = np.ones(E, np.float32)
    w_gate = np.empty((E, d, ff), np.float32)
    w_up = np.empty((E, d, ff), np.float32)
    w_down = np.empty((E, ff, d), np.float32)
    sg = su = sd = None
    if cfg.threaded_draw:
        bf = cfg.dtype == BF16
        dg, du, dd = (np.empty((d, dff), np.float32), np.empty((d, dff), np.float32),
                      np.empty((dff, d), np.float32))
        jobs = []
        for e in range(E):
            jobs += [(w_gate[e], 3 * e), (w_up[e], 3 * e + 1), (w_down[e], 3 * e + 2)]
        jobs += [(dg, 3 * E), (du, 3 * E + 1), (dd, 3 * E + 2)]
        if cfg.has_shared:
            sg, su, sd = np.empty((d, ff), np.float32), np.empty((d, ff), np.float32), np.empty((ff, d), np.float32)
            jobs += [(sg, 3 * E + 3), (su, 3 * E + 4), (sd, 3 * E + 5)]
        _pool_map(lambda j: _fill_normal(j[0], _stream(cfg.seed, j[1]), std, bf), jobs)
        rounded = {"w_gate", "w_up", "w_down", "dense_gate", "dense_up", "dense_down", "shared_gate",
                   "shared_up", "shared_down"} if bf else set()
    else:
        for e in range(E):
            w_gate[e] = _normal(rng, (d, ff), std)
            w_up[e] = _normal(rng, (d, ff), std)
            w_down[e] = _normal(rng, (ff, d), std)
        if cfg.has_shared:
            sg, su, sd = _normal(rng, (d, ff), std), _normal(rng, (d, ff), std), _normal(rng, (ff, d), std)
        dg, du, dd = _normal(rng, (d, dff), std), _normal(rng, (d, dff), std), _normal(rng, (dff, d), std)
        rounded = set()
    w = LayerWeights(gate, bias, scales, w_gate, w_up, w_down, dg, du, dd, sg, su, sd)
    if cfg.hot_share is not None:
        _skew_router(cfg, w)
    if cfg.dtype == BF16:
        for f in ("gate", "w_gate", "w_up", "w_down", "dense_gate", "dense_up", "dense_down",
                  "shared_gate", "shared_up", "shared_down"):
            v = getattr(w, f)
            if v is not None and f not in rounded:
                setattr(w, f, bf16_round(v))
    return w


def _skew_router(cfg: LayerConfig, w: LayerWeights) -> None:
    """Scale the gate columns of the hot experts (every 1/hot_fraction-th
    expert) by alpha, found by bisection on a 4096-token sample so that the hot
    experts take `hot_share` of all top-k assignments."""
    E = cfg.n_experts
    step = int(round(1.0 / cfg.hot_fraction))
    hot = np.arange(0, E, step)
    x = make_tokens(cfg.with_tokens(4096), seed_offset=1000)
    xs = bf16_round(x) if cfg.dtype == BF16 else x
    lo, hi = 1.0, 64.0
    base = w.gate.copy()
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        g = base.copy()
        g[:, hot] *= np.float32(mid)
        if cfg.dtype == BF16:
            g = bf16_round(g)
        share = _topk_share(xs, g, w.bias, cfg.top_k, hot)
        if share < cfg.hot_share:
            lo = mid
        else:
            hi = mid
    alpha = 0.5 * (lo + hi)
    g = base.copy()
    g[:, hot] *= np.float32(alpha)
    w.gate = g
    w.hot_experts = hot
    w.hot_alpha = float(alpha)
    w.hot_share_achieved = _topk_share(xs, bf16_round(g) if cfg.dtype == BF16 else g, w.bias,
                                       cfg.top_k, hot)


def _token_rows(cfg: LayerConfig, x: np.ndarray) -> np.ndarray:
    if cfg.x_dist == "rmsnorm":
        x = rms_norm_rows(x)
    if cfg.dtype == BF16:
        x = bf16_round(x)
    return x


def make_tokens(cfg: LayerConfig, seed_offset: int = 1, tokens: Optional[int] = None) -> np.ndarray:
    """Draw x [T, d] (f32; BF16-rounded for BF16 layers) from its own Philox
    stream (seed + seed_offset), so token count does not change the weights.
    Under cfg.threaded_draw every TOKEN_BLOCK rows come from their own stream
    (drawn on all host cores); the first n rows are the same for any T >= n
    either way."""
    T = cfg.tokens if tokens is None else tokens
    if cfg.threaded_draw:
        x = np.empty((T, cfg.d_model), np.float32)

        def block(b):
            r0, r1 = b * TOKEN_BLOCK, min(T, (b + 1) * TOKEN_BLOCK)
            part = _stream(cfg.seed + seed_offset, b).standard_normal(size=(TOKEN_BLOCK, cfg.d_model),
                                                                      dtype=np.float32)[: r1 - r0]
            x[r0:r1] = _token_rows(cfg, part)

        _pool_map(block, range((T + TOKEN_BLOCK - 1) // TOKEN_BLOCK))
        return x
    rng = np.random.Generator(np.random.Philox(cfg.seed + seed_offset))
    x = rng.standard_normal(size=(T, cfg.d_model), dtype=np.float32)
    return np.ascontiguousarray(_token_rows(cfg, x))


def algorithmic_bytes(cfg: LayerConfig, tokens: int) -> dict:
    """Bytes each HBM-bound kernel must move per launch over `tokens` tokens
    (b = bytes per activation element)."""
    b = 4 if cfg.dtype == F32 else 2
    d, E, k = cfg.d_model, cfg.n_experts, cfg.top_k
    T = tokens
    return {
        # BF16 router (one kernel): x once, gate once, (index, weight) per
        # pick, the E counts
        "router": T * d * b + d * E * b + T * k * 8 + 8 * E,
        # x once, router gate once, f32 scores written
        "router_scores": T * d * b + d * E * b + T * E * 4,
        # scores read; index, weight and rank per pick written
        "router_topk": T * E * 4 + T * k * 12,
        # x once, k copies written, dst index per pick
        "permute": T * d * b + T * k * d * b + 8 * T * k,
        # k expert rows gathered, out written, (index, weight) per pick
        "combine": T * k * d * b + T * d * b + 8 * T * k,
        # sandwich norm: pre reads h and writes the normalised input; post
        # reads the layer output and the residual and writes the sublayer output
        "norm_pre": 2 * T * d * b,
        "norm_post": 3 * T * d * b,
    }


def inv_sqrt2() -> np.float32:
    return np.float32(1.0) / np.float32(math.sqrt(2.0))
