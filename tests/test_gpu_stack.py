"""A small MoE decoder stack (noor_-_bangla_ai_b200/stack.py: embedding,
MoE blocks with the attention stand-in and the library's FFN sublayer, final
norm, output projection) against the oracle's model forward (model.rs:127-207,
block.rs:74-97, attention.rs:67-191, rope.rs:49-90).

Tolerances (written here, checked below):
  F32 stack   logits rel-L2 <= 1e-4  (two layers; the attention stand-in
                                      differs from the reference's serial f32
                                      loops in the last bits)
  BF16 stack  logits rel-L2 <= 2e-2  (BF16 weights and residual stream, as
                                      mirrored in the oracle)
  max attention logit within 1e-3 relative; per-layer counts sum to T*k
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _blocks_for_oracle(pkg, st, bf16):
    W = pkg.workloads
    rb = (lambda a: W.bf16_round(np.asarray(a, np.float32))) if bf16 else (lambda a: np.asarray(a, np.float32))
    out, ropes = [], []
    for b in st.blocks:
        w = b.parallel_ffn.moe._weights()
        for f in ("gate", "w_gate", "w_up", "w_down", "dense_gate", "dense_up", "dense_down"):
            setattr(w, f, rb(getattr(w, f)))  # the device stores the layer's weights in its dtype
        a = b.attention
        out.append({"wq": a.wq, "wk": a.wk, "wv": a.wv, "wo": a.wo, "n_heads": a.n_heads, "n_kv_heads": a.n_kv_heads,
                    "head_dim": a.head_dim, "window": a.sliding_window, "attn_pre": b.attn_norm.pre_norm.weight,
                    "attn_post": b.attn_norm.post_norm.weight, "ffn_pre": b.ffn_norm.pre_norm.weight,
                    "ffn_post": b.ffn_norm.post_norm.weight, "depth_scale": float(b.attn_norm.depth_scale), "w": w,
                    "top_k": b.parallel_ffn.moe.router.n_active})
        r = st.prope if (b.is_global and st.prope is not None) else st.rope
        ropes.append((r.inv_freq, r.rotate_dim))
    return out, ropes


@pytest.mark.parametrize("dtype_name,tol", [("f32", 1e-4), ("bf16", 2e-2)])
def test_stack_matches_oracle(pkg, oracle, dtype_name, tol):
    api = pkg.api
    dtype = api.DTYPE_BF16 if dtype_name == "bf16" else api.DTYPE_F32
    rng = np.random.default_rng(7)
    st = pkg.stack.NoorStack(vocab_size=97, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64,
                             dense_ffn_dim=512, expert_ffn_dim=256, n_experts=8, n_active_experts=2,
                             sliding_window=8, global_every_n=2, prope_fraction=0.25, dtype=dtype, rng=rng)
    assert [b.is_global for b in st.blocks] == [False, True]
    assert st.blocks[0].attention.sliding_window == 8 and st.blocks[1].attention.sliding_window == 0
    ids = np.random.default_rng(3).integers(0, 97, size=40)
    logits, ml, util = st.forward(ids)
    blocks, ropes = _blocks_for_oracle(pkg, st, dtype == api.DTYPE_BF16)
    ref, rml = oracle.stack_forward(st.embedding, blocks, st.final_norm.weight, st.output_proj, ids, 1e-6, ropes,
                                    dtype == api.DTYPE_BF16)
    got = logits.cpu().numpy()
    err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err <= tol, err
    assert abs(ml - rml) <= 1e-3 * max(1.0, abs(rml)), (ml, rml)
    for f in util:  # ExpertUtilization::fractions sums to k
        assert abs(sum(f) - 2.0) < 1e-5
    for b in st.blocks:
        b.parallel_ffn.moe.invalidate()


def test_reference_block_tests(pkg):
    """block.rs:198-212 and 273-281 through the mirror: a small F32 MoE block
    (shared expert on) keeps the shape, and its max attention logit is finite."""
    api = pkg.api
    rng = np.random.default_rng(11)
    blk = pkg.stack.MoEBlock(32, 4, 2, 8, 64, 32, 4, 2, True, 16, 0, False, 1e-6, 0.02, dtype=api.DTYPE_F32,
                             rng=rng)
    rope = pkg.stack.RoPE(8, 10000.0)
    x = torch.randn(4, 32, device="cuda")
    out, ml = blk.forward(x, rope)
    assert tuple(out.shape) == (4, 32) and torch.isfinite(out).all()
    blk2 = pkg.stack.MoEBlock(16, 2, 1, 8, 32, 16, 4, 2, False, 0, 0, False, 1e-6, 0.5, dtype=api.DTYPE_F32,
                              rng=rng)
    out2, ml2 = blk2.forward(torch.randn(3, 16, device="cuda"), rope)
    assert np.isfinite(ml2) and tuple(out2.shape) == (3, 16)
    for b in (blk, blk2):
        b.parallel_ffn.moe.invalidate()
