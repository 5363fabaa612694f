"""ctypes front end of the CPU oracle, plus an independent numpy restatement.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the library.  See noor_oracle.c for the
reference lines each function restates (crates/noor-core/src/layers/moe.rs,
ffn.rs, parallel_ffn.rs, tensor.rs; crates/noor-train/src/optim/smebu.rs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libnoor_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


class _Layer(ctypes.Structure):
    _fields_ = [
        ("d_model", _i64), ("n_experts", _i64), ("top_k", _i64), ("expert_ff", _i64),
        ("dense_ff", _i64),
        ("gate", _f32p), ("bias", _f32p), ("scales", _f32p),
        ("w_gate", _f32p), ("w_up", _f32p), ("w_down", _f32p),
        ("shared_gate", _f32p), ("shared_up", _f32p), ("shared_down", _f32p),
        ("dense_gate", _f32p), ("dense_up", _f32p), ("dense_down", _f32p),
    ]


def build() -> str:
    """Compile libnoor_oracle.so with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
                os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "noor_oracle.c"))):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.noor_oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.noor_oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.noor_oracle_bf16_to_f32.restype = ctypes.c_float
        L.noor_oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.noor_oracle_round_bf16.argtypes = [_f32p, _i64]
        for name in ("sigmoid", "silu", "gelu"):
            fn = getattr(L, "noor_oracle_" + name)
            fn.restype = ctypes.c_float
            fn.argtypes = [ctypes.c_float]
        L.noor_oracle_use_openblas.restype = ctypes.c_int
        L.noor_oracle_use_openblas.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.noor_oracle_matmul.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64]
        L.noor_oracle_route.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                        _i32p, _f32p, _i64p, _f32p]
        L.noor_oracle_scores_f64.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64, _f64p, _f64p]
        L.noor_oracle_glu_ffn.argtypes = [_f32p, _i64, _i64, _i64, _f32p, _f32p, _f32p,
                                          ctypes.c_int, _f32p]
        L.noor_oracle_moe_forward.argtypes = [ctypes.POINTER(_Layer), _f32p, _i64, _f32p, _i32p,
                                              _f32p, _i64p]
        L.noor_oracle_parallel_forward.argtypes = L.noor_oracle_moe_forward.argtypes
        L.noor_oracle_rms_norm.argtypes = [_f32p, _f32p, _i64, _i64, ctypes.c_double, _f32p]
        L.noor_oracle_smebu_update.argtypes = [_f32p, _f32p, _f32p, _i64, ctypes.c_float,
                                               ctypes.c_float, ctypes.c_float]
        _lib = L
    return _lib


def _p(a: Optional[np.ndarray], t=_f32p):
    if a is None:
        return ctypes.cast(None, t)
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- scalar ops

def f32_to_bf16(x: float) -> int:
    return int(lib().noor_oracle_f32_to_bf16(x))


def bf16_to_f32(h: int) -> float:
    return float(lib().noor_oracle_bf16_to_f32(h))


def round_bf16(a) -> np.ndarray:
    a = _f32(a).copy()
    lib().noor_oracle_round_bf16(_p(a), a.size)
    return a


def sigmoid(x: float) -> float:
    return float(lib().noor_oracle_sigmoid(x))


def silu(x: float) -> float:
    return float(lib().noor_oracle_silu(x))


def gelu(x: float) -> float:
    return float(lib().noor_oracle_gelu(x))


def use_openblas(threads: int = 0) -> bool:
    """Route oracle matmuls through numpy's bundled ILP64 OpenBLAS sgemm (the
    reference's cblas route, kernels.rs:151-163).  Returns False if absent."""
    libs = os.path.join(os.path.dirname(np.__file__) + ".libs")
    if not os.path.isdir(libs):
        libs = os.path.join(os.path.dirname(os.path.dirname(np.__file__)), "numpy.libs")
    cands = [f for f in os.listdir(libs) if f.startswith("libscipy_openblas64_")] if os.path.isdir(libs) else []
    if not cands:
        return False
    rc = lib().noor_oracle_use_openblas(os.path.join(libs, cands[0]).encode(), threads)
    return rc == 0


def use_plain_loops() -> None:
    lib().noor_oracle_use_openblas(None, 0)


# ---------------------------------------------------------------- layer ops

def matmul(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), np.float32)
    lib().noor_oracle_matmul(_p(a), _p(b), _p(c), m, k, n)
    return c


def route(x, gate, bias, scales, k: int, want_scores: bool = False):
    """Batched MoERouter::route (moe.rs:79-107) + ExpertUtilization::record.
    Returns idx [T,k] int32, w [T,k] f32, counts [E] int64 (and scores [T,E])."""
    x, gate, bias, scales = _f32(x), _f32(gate), _f32(bias), _f32(scales)
    T, d = x.shape
    E = gate.shape[1]
    kk = min(k, E)
    idx = np.empty((T, kk), np.int32)
    w = np.empty((T, kk), np.float32)
    counts = np.zeros(E, np.int64)
    scores = np.empty((T, E), np.float32) if want_scores else None
    lib().noor_oracle_route(_p(x), _p(gate), _p(bias), _p(scales), T, d, E, k, _p(idx, _i32p),
                            _p(w), _p(counts, _i64p), _p(scores))
    if want_scores:
        return idx, w, counts, scores
    return idx, w, counts


def scores_f64(x, gate, bias):
    """Router scores with f64 accumulation and the absolute-sum bound."""
    x, gate, bias = _f32(x), _f32(gate), _f32(bias)
    T, d = x.shape
    E = gate.shape[1]
    s = np.empty((T, E), np.float64)
    ab = np.empty((T, E), np.float64)
    lib().noor_oracle_scores_f64(_p(x), _p(gate), _p(bias), T, d, E, _p(s, _f64p), _p(ab, _f64p))
    return s, ab


def glu_ffn(x, w_gate, w_up, w_down, act: int) -> np.ndarray:
    """act 0 = GeGLUFFN::forward (ffn.rs:24-34), 1 = SwiGLUFFN::forward (ffn.rs:62-68)."""
    x, w_gate, w_up, w_down = _f32(x), _f32(w_gate), _f32(w_up), _f32(w_down)
    m, d = x.shape
    ff = w_gate.shape[1]
    out = np.empty((m, d), np.float32)
    lib().noor_oracle_glu_ffn(_p(x), m, d, ff, _p(w_gate), _p(w_up), _p(w_down), act, _p(out))
    return out


def _layer_struct(w, top_k: int):
    d, E = w.gate.shape
    ff = w.w_gate.shape[2]
    dff = w.dense_gate.shape[1]
    keep = [w.gate, w.bias, w.scales, w.w_gate, w.w_up, w.w_down, w.dense_gate, w.dense_up,
            w.dense_down, w.shared_gate, w.shared_up, w.shared_down]
    for a in keep:
        if a is not None:
            assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    L = _Layer(d, E, top_k, ff, dff, _p(w.gate), _p(w.bias), _p(w.scales), _p(w.w_gate),
               _p(w.w_up), _p(w.w_down), _p(w.shared_gate), _p(w.shared_up), _p(w.shared_down),
               _p(w.dense_gate), _p(w.dense_up), _p(w.dense_down))
    return L, keep


def moe_forward(w, x, top_k: int):
    """MoELayer::forward (moe.rs:145-177).  Returns out [T,d], idx, w, counts."""
    x = _f32(x)
    T, d = x.shape
    L, _keep = _layer_struct(w, top_k)
    kk = min(top_k, w.gate.shape[1])
    out = np.empty((T, d), np.float32)
    idx = np.empty((T, kk), np.int32)
    wt = np.empty((T, kk), np.float32)
    counts = np.zeros(w.gate.shape[1], np.int64)
    lib().noor_oracle_moe_forward(ctypes.byref(L), _p(x), T, _p(out), _p(idx, _i32p), _p(wt),
                                  _p(counts, _i64p))
    return out, idx, wt, counts


def parallel_forward(w, x, top_k: int):
    """ParallelFFN::forward (parallel_ffn.rs:30-36): (dense + moe) / sqrt(2)."""
    x = _f32(x)
    T, d = x.shape
    L, _keep = _layer_struct(w, top_k)
    kk = min(top_k, w.gate.shape[1])
    out = np.empty((T, d), np.float32)
    idx = np.empty((T, kk), np.int32)
    wt = np.empty((T, kk), np.float32)
    counts = np.zeros(w.gate.shape[1], np.int64)
    lib().noor_oracle_parallel_forward(ctypes.byref(L), _p(x), T, _p(out), _p(idx, _i32p), _p(wt),
                                       _p(counts, _i64p))
    return out, idx, wt, counts


def rms_norm(a, weight, eps: float) -> np.ndarray:
    a, weight = _f32(a), _f32(weight)
    out = np.empty_like(a)
    dim = a.shape[-1]
    lib().noor_oracle_rms_norm(_p(a), _p(weight), a.size // dim, dim, eps, _p(out))
    return out


def ffn_sublayer_forward(w, x, top_k: int, pre_w, post_w, eps: float, depth_scale: float, bf16_storage: bool):
    """The MoE block's FFN sublayer (block.rs:87-90): normed = rms_norm(h,
    pre) * depth_scale (norm.rs:51-54); ffn = ParallelFFN(normed); out = h +
    rms_norm(ffn, post) * depth_scale (norm.rs:57-60, tensor.rs:280-288).
    With bf16_storage the normalised input is rounded to BF16, as a BF16
    layer stores its input.  Returns out, idx, w, counts of the layer."""
    x = _f32(x)
    ds = np.float32(depth_scale)
    xn = (rms_norm(x, pre_w, eps) * ds).astype(np.float32)
    if bf16_storage:
        u = xn.view(np.uint32).astype(np.uint64)
        u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16  # RNE to BF16 (tensor.rs:23-28; finite values)
        xn = (u.astype(np.uint32) << np.uint32(16)).view(np.float32)
    ffn, idx, wt, counts = parallel_forward(w, xn, top_k)
    out = (x + (rms_norm(ffn, post_w, eps) * ds).astype(np.float32)).astype(np.float32)
    return out, idx, wt, counts, xn


def smebu_update(momentum, biases, fractions, kappa: float, beta: float, lam: float):
    """SMEBU::update (smebu.rs:36-48), in place on momentum and biases."""
    assert momentum.dtype == np.float32 and biases.dtype == np.float32
    fr = _f32(fractions)
    lib().noor_oracle_smebu_update(_p(momentum), _p(biases), _p(fr), momentum.size, kappa, beta, lam)


# ------------------------------------------------- independent numpy mirror

def np_parallel_forward(w, x, top_k: int):
    """Second, vectorised restatement of ParallelFFN::forward in numpy (f64
    accumulation), used only to cross-check the C oracle within tolerance."""
    x64 = np.asarray(x, np.float64)
    g = x64 @ w.gate.astype(np.float64) + w.bias.astype(np.float64)[None, :]
    s = 1.0 / (1.0 + np.exp(-g))
    order = np.argsort(-s, axis=1, kind="stable")[:, :top_k]
    wt = np.take_along_axis(s, order, axis=1) * w.scales.astype(np.float64)[order]
    T, d = x64.shape
    moe = np.zeros((T, d))
    for e in range(w.gate.shape[1]):
        rows, slot = np.nonzero(order == e)
        if rows.size == 0:
            continue
        xe = x64[rows]
        gg = xe @ w.w_gate[e].astype(np.float64)
        uu = xe @ w.w_up[e].astype(np.float64)
        h = gg / (1.0 + np.exp(-gg)) * uu
        moe[rows] += wt[rows, slot][:, None] * (h @ w.w_down[e].astype(np.float64))
    if w.shared_gate is not None:
        gg = x64 @ w.shared_gate.astype(np.float64)
        uu = x64 @ w.shared_up.astype(np.float64)
        moe += (gg / (1.0 + np.exp(-gg)) * uu) @ w.shared_down.astype(np.float64)
    gg = x64 @ w.dense_gate.astype(np.float64)
    uu = x64 @ w.dense_up.astype(np.float64)
    c = np.sqrt(2.0 / np.pi)
    ge = 0.5 * gg * (1.0 + np.tanh(c * (gg + 0.044715 * gg ** 3)))
    dense = (ge * uu) @ w.dense_down.astype(np.float64)
    return (dense + moe) / np.sqrt(2.0), order.astype(np.int32), wt


# ------------------------------------------------- the decoder stack around the layer
# RoPE::apply (rope.rs:49-90), GQAAttention::forward without a KV cache
# (attention.rs:67-191), MoEBlock::forward (block.rs:74-97) and the model
# forward (model.rs:127-207), restated in f32 with the reference's operation
# order.  Rust's f32 cos / sin / exp call libm's cosf / sinf / expf, which
# these use too.  Loops are plain Python: small configurations only.

_libm = None


def _m():
    global _libm
    if _libm is None:
        _libm = ctypes.CDLL("libm.so.6")
        for f in ("cosf", "sinf", "expf"):
            getattr(_libm, f).argtypes = [ctypes.c_float]
            getattr(_libm, f).restype = ctypes.c_float
    return _libm


def rope_inv_freq(head_dim: int, theta: float, fraction: Optional[float] = None):
    """RoPE::new / new_proportional (rope.rs:17-45)."""
    rotate_dim = head_dim if fraction is None else max(2, (int(head_dim * fraction) // 2) * 2)
    inv = np.array([np.float32(1.0) / np.float32(theta ** (2.0 * i / rotate_dim))
                    for i in range(rotate_dim // 2)], np.float32)
    return inv, rotate_dim


def rope_apply(x, inv_freq, rotate_dim: int, seq_offset: int = 0) -> np.ndarray:
    """RoPE::apply (rope.rs:49-90) on x (..., seq, head_dim), f32."""
    x = _f32(x)
    out = x.copy()
    m = _m()
    for s in range(x.shape[-2]):
        pos = np.float32(seq_offset + s)
        for i in range(rotate_dim // 2):
            ang = np.float32(pos * inv_freq[i])
            c, sn = np.float32(m.cosf(float(ang))), np.float32(m.sinf(float(ang)))
            x0, x1 = x[..., s, 2 * i], x[..., s, 2 * i + 1]
            out[..., s, 2 * i] = (x0 * c).astype(np.float32) - (x1 * sn).astype(np.float32)
            out[..., s, 2 * i + 1] = (x0 * sn).astype(np.float32) + (x1 * c).astype(np.float32)
    return out


def gqa_attention(x, wq, wk, wv, wo, n_heads: int, n_kv_heads: int, head_dim: int, sliding_window: int,
                  inv_freq, rotate_dim: int):
    """GQAAttention::forward (attention.rs:67-191), one sequence, no cache.
    Returns (output [seq, d], max_attn_logit)."""
    x = _f32(x)
    S = x.shape[0]
    nh, nkv, hd = n_heads, n_kv_heads, head_dim
    q = matmul(x, wq).reshape(S, nh, hd).transpose(1, 0, 2).copy()
    k = matmul(x, wk).reshape(S, nkv, hd).transpose(1, 0, 2).copy()
    v = matmul(x, wv).reshape(S, nkv, hd).transpose(1, 0, 2).copy()
    q = rope_apply(q, inv_freq, rotate_dim)
    k = rope_apply(k, inv_freq, rotate_dim)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    out = np.zeros((nh, S, hd), np.float32)
    max_logit = np.float32(-np.inf)
    m = _m()
    group = nh // nkv
    for qh in range(nh):
        kv = qh // group
        for sq in range(S):
            scores = np.full(S, -np.inf, np.float32)
            for sk in range(S):
                if sk > sq or (sliding_window > 0 and sq > sk + sliding_window):
                    continue
                dot = np.float32(0.0)
                for dd in range(hd):
                    dot = np.float32(dot + np.float32(q[qh, sq, dd] * k[kv, sk, dd]))
                scores[sk] = np.float32(dot * scale)
                max_logit = max(max_logit, scores[sk])
            max_s = scores.max()
            p = np.array([0.0 if s_ == -np.inf else m.expf(float(np.float32(s_ - max_s))) for s_ in scores],
                         np.float32)
            tot = np.float32(0.0)
            for p_ in p:
                tot = np.float32(tot + p_)
            if tot > 0:
                p = (p / tot).astype(np.float32)
            for dd in range(hd):
                val = np.float32(0.0)
                for sk in range(S):
                    if p[sk] > 0:
                        val = np.float32(val + np.float32(p[sk] * v[kv, sk, dd]))
                out[qh, sq, dd] = val
    attn = out.transpose(1, 0, 2).reshape(S, nh * hd).copy()
    return matmul(attn, wo), float(max_logit)


def _bf16_storage(a):
    u = _f32(a).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16  # RNE (tensor.rs:23-28), finite values
    return (u.astype(np.uint32) << np.uint32(16)).view(np.float32)


def moe_block_forward(blk, x, eps: float, inv_freq, rotate_dim: int, bf16_storage: bool):
    """MoEBlock::forward (block.rs:74-97).  blk: dict with the attention
    weights / head counts / window, the four norm weights, depth_scale, the
    layer's LayerWeights `w` and top_k.  With bf16_storage the residual
    stream is rounded to BF16 after each sublayer, as a BF16 layer stores
    it."""
    ds = np.float32(blk["depth_scale"])
    normed = (rms_norm(x, blk["attn_pre"], eps) * ds).astype(np.float32)
    a, ml = gqa_attention(normed, blk["wq"], blk["wk"], blk["wv"], blk["wo"], blk["n_heads"], blk["n_kv_heads"],
                          blk["head_dim"], blk["window"], inv_freq, rotate_dim)
    a = (rms_norm(a, blk["attn_post"], eps) * ds).astype(np.float32)
    h = (_f32(x) + a).astype(np.float32)
    if bf16_storage:
        h = _bf16_storage(h)
    out, _idx, _wt, counts, _xn = ffn_sublayer_forward(blk["w"], h, blk["top_k"], blk["ffn_pre"], blk["ffn_post"],
                                                        eps, float(ds), bf16_storage)
    if bf16_storage:
        out = _bf16_storage(out)
    return out, ml, counts


def stack_forward(embedding, blocks, final_norm, output_proj, token_ids, eps: float, ropes, bf16_storage: bool):
    """The model forward (model.rs:127-207) over MoE blocks: embedding lookup
    (embedding.rs:19-35), the blocks (ropes[i] = (inv_freq, rotate_dim) of
    layer i), the final RMSNorm and the output projection.  Returns (logits,
    max_attn_logit)."""
    h = _f32(embedding)[np.asarray(token_ids)]
    if bf16_storage:
        h = _bf16_storage(h)
    ml = -np.inf
    for blk, (inv, rd) in zip(blocks, ropes):
        h, m_, _ = moe_block_forward(blk, h, eps, inv, rd, bf16_storage)
        ml = max(ml, m_)
    h = rms_norm(h, final_norm, eps)
    return matmul(h, output_proj), ml
