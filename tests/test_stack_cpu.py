"""The decoder stack's attention stand-in (noor_-_bangla_ai_b200/stack.py,
PyTorch on the CPU here) against the oracle's restatement of RoPE::apply and
GQAAttention::forward, plus the reference's own RoPE and attention tests
(rope.rs:92-167, attention.rs:230-300) ported to the stand-in.

Tolerances: attention output rel-L2 <= 1e-5 and max logit within 1e-5
(f32 against f32; torch's cos/sin and softmax order differ from libm's and
the reference's serial loops in the last bits)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _stand_in(pkg, d, nh, nkv, hd, window, fraction, seed):
    S = pkg.stack
    rng = np.random.default_rng(seed)
    att = S.GQAAttention(d, nh, nkv, hd, window, 0.3, rng)
    rope = S.RoPE(hd, 10000.0 if fraction is None else 1_000_000.0, fraction)
    return att, rope


@pytest.mark.parametrize("nh,nkv,hd,window,fraction", [(4, 2, 8, 0, None), (4, 4, 8, 3, None), (4, 1, 16, 0, 0.25),
                                                       (2, 1, 8, 2, None)])
def test_attention_stand_in_matches_oracle(pkg, oracle, nh, nkv, hd, window, fraction):
    d, S = 32, 12
    att, rope = _stand_in(pkg, d, nh, nkv, hd, window, fraction, seed=nh * 10 + hd)
    x = np.random.default_rng(1).standard_normal((S, d)).astype(np.float32)
    out, ml = att.forward(torch.from_numpy(x), rope)
    inv, rd = oracle.rope_inv_freq(hd, 10000.0 if fraction is None else 1_000_000.0, fraction)
    assert np.array_equal(inv, rope.inv_freq) and rd == rope.rotate_dim
    ref, rml = oracle.gqa_attention(x, att.wq, att.wk, att.wv, att.wo, nh, nkv, hd, window, inv, rd)
    err = float(np.linalg.norm(out.numpy() - ref) / np.linalg.norm(ref))
    assert err <= 1e-5, err
    assert abs(ml - rml) <= 1e-5 * max(1.0, abs(rml)), (ml, rml)


def test_rope_reference_tests(pkg):
    S = pkg.stack
    rope = S.RoPE(64, 10000.0)
    x = torch.randn(2, 8, 64)
    r = rope.apply(x, 0)
    assert r.shape == x.shape
    mag = lambda t: torch.sqrt(t[..., 0::2] ** 2 + t[..., 1::2] ** 2)
    assert torch.all((mag(r) - mag(x)).abs() < 1e-4)              # preserves magnitude
    one = torch.ones(1, 1, 64)
    r0, r1, r100 = rope.apply(one, 0), rope.apply(one, 1), rope.apply(one, 100)
    assert not torch.equal(r0, r1) and not torch.equal(r1, r100)  # different offsets differ
    rope4 = S.RoPE(4, 10000.0)
    x4 = torch.tensor([[[1.0, 2.0, 3.0, 4.0]]])
    assert torch.all((rope4.apply(x4, 0) - x4).abs() < 1e-5)     # position 0 is the identity
    prope = S.RoPE(8, 1_000_000.0, 0.25)
    assert prope.rotate_dim == 2
    x8 = torch.arange(1.0, 9.0).view(1, 1, 8)
    r8 = prope.apply(x8, 5)
    assert torch.equal(r8[..., 2:], x8[..., 2:])                  # dims past rotate_dim untouched
    assert (r8[..., :2] - x8[..., :2]).abs().max() > 1e-6


def test_attention_reference_tests(pkg):
    S = pkg.stack
    rng = np.random.default_rng(0)
    rope = S.RoPE(8, 10000.0)
    # causal: position 0 does not see a change at position 3
    att = S.GQAAttention(16, 2, 1, 8, 0, 0.5, rng)
    x = torch.zeros(4, 16)
    x[0] = 1.0
    x2 = x.clone()
    x2[3] = 99.0
    o1, _ = att.forward(x, rope)
    o2, _ = att.forward(x2, rope)
    assert torch.all((o1[0] - o2[0]).abs() < 1e-5)
    # sliding window 2: position 5 does not see position 0
    att = S.GQAAttention(16, 2, 1, 8, 2, 0.5, rng)
    x = torch.ones(8, 16)
    x2 = x.clone()
    x2[0] = 99.0
    o1, _ = att.forward(x, rope)
    o2, _ = att.forward(x2, rope)
    assert torch.all((o1[5] - o2[5]).abs() < 1e-4)
    # GQA shapes and a finite max logit
    att = S.GQAAttention(32, 4, 2, 8, 0, 0.1, rng)
    assert att.n_heads // att.n_kv_heads == 2
    o, ml = att.forward(torch.randn(4, 32), rope)
    assert o.shape == (4, 32) and np.isfinite(ml)
