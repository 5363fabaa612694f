"""The MoE decoder stack around the layer: Noor's MoEBlock and NoorModel forward
(crates/noor-core/src/layers/block.rs:74-97, model.rs:127-207) with the names
and parameter layouts of the reference.

NOT THE HOT PATH.  The attention sublayer is a stand-in built from PyTorch
operations (the projections are torch matmuls, attention is
torch.nn.functional.scaled_dot_product_attention with an explicit causal /
sliding-window mask); it follows GQAAttention::forward (attention.rs:67-191)
and RoPE::apply (rope.rs:49-90) but is not a B200 kernel of this library.  The
FFN sublayer of every block -- sandwich norm, router, experts, dense branch,
combine, residual -- is one call of the library's noor_moe_ffn_sublayer_forward.

Tensors live on one CUDA device; BF16 layers keep the residual stream in
bfloat16 between sublayers, F32 layers in float32.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import api


def rope_inv_freq(head_dim: int, theta: float, fraction: Optional[float] = None) -> Tuple[np.ndarray, int]:
    """RoPE::new / new_proportional (rope.rs:17-45): inverse frequencies (f32)
    of the rotated pairs and the number of rotated dims."""
    if fraction is None:
        rotate_dim = head_dim
    else:
        rotate_dim = max(2, (int(head_dim * fraction) // 2) * 2)
    half = rotate_dim // 2
    inv = np.array([np.float32(1.0) / np.float32(theta ** (2.0 * i / rotate_dim)) for i in range(half)], np.float32)
    return inv, rotate_dim


class RoPE:
    """rope.rs:5-90.  Pairs (2i, 2i+1) of the first rotate_dim dims are rotated
    by angle = position * inv_freq[i] (f32); the rest pass unchanged."""

    def __init__(self, head_dim: int, theta: float, fraction: Optional[float] = None):
        self.inv_freq, self.rotate_dim = rope_inv_freq(head_dim, theta, fraction)
        self.head_dim = head_dim

    def apply(self, x, seq_offset: int = 0):
        """x: torch tensor (..., seq, head_dim); the rotation is computed in f32."""
        import torch
        seq = x.shape[-2]
        half = self.rotate_dim // 2
        pos = torch.arange(seq_offset, seq_offset + seq, device=x.device, dtype=torch.float32)
        inv = torch.from_numpy(self.inv_freq).to(x.device)
        ang = pos[:, None] * inv[None, :]  # f32 products, as the reference's pos * inv_freq[i]
        cos, sin = torch.cos(ang), torch.sin(ang)
        xf = x.float()
        x0 = xf[..., 0:2 * half:2]
        x1 = xf[..., 1:2 * half:2]
        out = xf.clone()
        out[..., 0:2 * half:2] = x0 * cos - x1 * sin
        out[..., 1:2 * half:2] = x0 * sin + x1 * cos
        return out.to(x.dtype)


class GQAAttention:
    """attention.rs:24-191 (no KV cache): grouped-query attention, q head h
    uses kv head h // (n_heads / n_kv_heads); causal, optionally limited to a
    sliding window of keys at most `sliding_window` positions back."""

    def __init__(self, d_model: int, n_heads: int, n_kv_heads: int, head_dim: int, sliding_window: int,
                 init_std: float, rng=None):
        rng = rng or np.random.default_rng()
        r = lambda shape: (rng.standard_normal(shape) * init_std).astype(np.float32)
        self.wq = r((d_model, n_heads * head_dim))
        self.wk = r((d_model, n_kv_heads * head_dim))
        self.wv = r((d_model, n_kv_heads * head_dim))
        self.wo = r((n_heads * head_dim, d_model))
        self.n_heads, self.n_kv_heads, self.head_dim = n_heads, n_kv_heads, head_dim
        self.sliding_window = sliding_window
        self._dev = {}

    def _w(self, name, device, dtype):
        key = (name, str(device), dtype)
        if key not in self._dev:
            import torch
            self._dev[key] = torch.from_numpy(getattr(self, name)).to(device=device, dtype=dtype)
        return self._dev[key]

    def forward(self, x, rope: RoPE, want_max_logit: bool = True):
        """x: (seq, d_model) torch tensor.  Returns (output in x's dtype,
        max_attn_logit).  Computed in f32 whatever x's dtype, as the
        reference does."""
        import torch
        import torch.nn.functional as F
        S = x.shape[0]
        nh, nkv, hd = self.n_heads, self.n_kv_heads, self.head_dim
        dt, dev = torch.float32, x.device
        out_dtype = x.dtype
        x = x.float()
        q = (x @ self._w("wq", dev, dt)).view(S, nh, hd).transpose(0, 1)
        k = (x @ self._w("wk", dev, dt)).view(S, nkv, hd).transpose(0, 1)
        v = (x @ self._w("wv", dev, dt)).view(S, nkv, hd).transpose(0, 1)
        q, k = rope.apply(q), rope.apply(k)
        g = nh // nkv
        k = k.repeat_interleave(g, dim=0)
        v = v.repeat_interleave(g, dim=0)
        i = torch.arange(S, device=dev)
        allowed = i[None, :] <= i[:, None]  # key position <= query position
        if self.sliding_window > 0:
            allowed &= i[:, None] <= i[None, :] + self.sliding_window
        scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))  # 1.0 / (hd as f32).sqrt()
        o = F.scaled_dot_product_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), attn_mask=allowed,
                                           scale=scale).squeeze(0)
        max_logit = float("-inf")
        if want_max_logit:  # the largest unmasked scaled score, in blocks of queries
            for q0 in range(0, S, 512):
                s = (q[:, q0:q0 + 512].float() @ k.float().transpose(1, 2)) * scale
                s = s.masked_fill(~allowed[q0:q0 + 512][None], float("-inf"))
                max_logit = max(max_logit, float(s.max().item()))
        out = o.transpose(0, 1).reshape(S, nh * hd) @ self._w("wo", dev, dt)
        return out.to(out_dtype), max_logit

    def param_count(self) -> int:
        return self.wq.size + self.wk.size + self.wv.size + self.wo.size


def _rms_norm_torch(x, w, eps: float, depth_scale: float):
    """rms_norm (tensor.rs:462-490) then Tensor::scale, in f32 on the device."""
    import torch
    xf = x.float()
    rms = torch.sqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return ((xf / rms) * w * depth_scale).to(x.dtype)


class MoEBlock:
    """block.rs:10-97: sandwich-normed attention and sandwich-normed
    ParallelFFN, each with a residual.  The FFN half runs in the library."""

    def __init__(self, d_model: int, n_heads: int, n_kv_heads: int, head_dim: int, dense_ffn_dim: int,
                 expert_ffn_dim: int, n_experts: int, n_active_experts: int, has_shared_expert: bool,
                 sliding_window: int, layer_idx: int, is_global: bool, eps: float, init_std: float,
                 dtype: int = api.DTYPE_BF16, device: int = 0, rng=None):
        rng = rng or np.random.default_rng()
        window = 0 if is_global else sliding_window
        depth_init = init_std / math.sqrt(2.0 * (layer_idx + 1))
        self.attn_norm = api.SandwichNorm(d_model, eps, layer_idx)
        self.attention = GQAAttention(d_model, n_heads, n_kv_heads, head_dim, window, depth_init, rng)
        self.ffn_norm = api.SandwichNorm(d_model, eps, layer_idx)
        self.parallel_ffn = api.ParallelFFN(d_model, dense_ffn_dim, expert_ffn_dim, n_experts, n_active_experts,
                                            has_shared_expert, depth_init, dtype=dtype, device=device, rng=rng)
        self.layer_idx, self.is_global = layer_idx, is_global
        self._sandwich_set = False

    def forward(self, x, rope: RoPE, want_max_logit: bool = True):
        """x: (seq, d_model) torch tensor on the layer's device.  Returns
        (hidden, max_attn_logit)."""
        import torch
        an = self.attn_norm
        normed = _rms_norm_torch(x, self._norm_w(an.pre_norm, x), an.pre_norm.eps, float(an.depth_scale))
        attn_out, max_logit = self.attention.forward(normed, rope, want_max_logit)
        attn_out = _rms_norm_torch(attn_out, self._norm_w(an.post_norm, x), an.post_norm.eps, float(an.depth_scale))
        h = (x.float() + attn_out.float()).to(x.dtype)  # tensor::add, in f32
        moe = self.parallel_ffn.moe
        dev = moe._device_handle()
        fn = self.ffn_norm
        if not self._sandwich_set:
            dev.set_sandwich(fn.pre_norm.weight, fn.post_norm.weight, fn.pre_norm.eps, float(fn.depth_scale))
            self._sandwich_set = True
        h = h.contiguous()
        out = torch.empty_like(h)
        counts = torch.empty(len(moe.experts), dtype=torch.int64, device=h.device)
        stream = torch.cuda.current_stream(h.device).cuda_stream
        dev.ffn_sublayer_device(h.data_ptr(), out.data_ptr(), h.shape[0], stream, counts_ptr=counts.data_ptr())
        moe.utilization.record_batch(counts.cpu().numpy(), h.shape[0])
        return out, max_logit

    def _norm_w(self, norm: "api.RMSNorm", like):
        import torch
        return torch.from_numpy(norm.weight).to(like.device)

    def param_count(self) -> int:
        return self.attention.param_count() + self.parallel_ffn.param_count() + 4 * self.attention.wq.shape[0]


class NoorStack:
    """model.rs:10-207 for a stack of MoE blocks: embedding -> blocks (global
    layers, every global_every_n-th, attend to the whole prefix with p-RoPE;
    the others to a sliding window with standard RoPE) -> final RMSNorm ->
    output projection."""

    def __init__(self, vocab_size: int, d_model: int, n_layers: int, n_heads: int, n_kv_heads: int,
                 head_dim: int, dense_ffn_dim: int, expert_ffn_dim: int, n_experts: int, n_active_experts: int,
                 has_shared_expert: bool = False, sliding_window: int = 0, global_every_n: int = 0,
                 rope_theta: float = 10000.0, prope_theta: float = 1_000_000.0, prope_fraction: float = 0.0,
                 eps: float = 1e-6, init_std: float = 0.02, dtype: int = api.DTYPE_BF16, device: int = 0,
                 rng=None):
        rng = rng or np.random.default_rng()
        self.embedding = (rng.standard_normal((vocab_size, d_model)) * init_std).astype(np.float32)
        self.blocks: List[MoEBlock] = []
        for i in range(n_layers):
            is_global = global_every_n > 0 and (i + 1) % global_every_n == 0
            self.blocks.append(MoEBlock(d_model, n_heads, n_kv_heads, head_dim, dense_ffn_dim, expert_ffn_dim,
                                        n_experts, n_active_experts, has_shared_expert, sliding_window, i,
                                        is_global, eps, init_std, dtype, device, rng))
        self.final_norm = api.RMSNorm(d_model, eps)
        self.output_proj = (rng.standard_normal((d_model, vocab_size)) * init_std).astype(np.float32)
        self.rope = RoPE(head_dim, rope_theta)
        self.prope = (RoPE(head_dim, prope_theta, prope_fraction)
                      if global_every_n > 0 and prope_fraction > 0.0 else None)
        self.dtype, self.device = dtype, device

    def forward(self, token_ids: Sequence[int], want_max_logit: bool = True):
        """Returns (logits [seq, vocab] f32 torch tensor, max_attn_logit,
        per-layer expert utilization fractions); the utilization is reset
        after each read, as model.rs:180-183."""
        import torch
        dev = torch.device("cuda", self.device)
        tdt = torch.bfloat16 if self.dtype == api.DTYPE_BF16 else torch.float32
        ids = torch.as_tensor(np.asarray(token_ids, np.int64), device=dev)
        if int(ids.max()) >= self.embedding.shape[0] or int(ids.min()) < 0:
            raise ValueError("token id out of vocab range")
        h = torch.from_numpy(self.embedding).to(dev)[ids].to(tdt)
        max_logit = float("-inf")
        util = []
        for b in self.blocks:
            rope = self.prope if (b.is_global and self.prope is not None) else self.rope
            h, ml = b.forward(h, rope, want_max_logit)
            max_logit = max(max_logit, ml)
            util.append(b.parallel_ffn.moe.utilization.fractions())
            b.parallel_ffn.moe.utilization.reset()
        w = torch.from_numpy(self.final_norm.weight).to(dev)
        h = _rms_norm_torch(h, w, self.final_norm.eps, 1.0)
        logits = h.float() @ torch.from_numpy(self.output_proj).to(dev)
        return logits, max_logit, util
