"""noor_moe_load_gguf: a MoE block read from a Noor GGUF checkpoint must give
exactly the layer that noor_moe_load_weights builds from the same arrays
(bit-identical outputs), for F32 and F16 files, with and without the
sandwich norm."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cfg(pkg):
    W = pkg.workloads
    return W.LayerConfig("gguf_small", 300, 256, 8, 2, 256, 512, W.BF16, seed=4)


def _handle(pkg, cfg):
    return pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                          max_tokens=cfg.tokens)


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_gguf_layer_equals_loaded_arrays(pkg, tmp_path, dtype):
    W, G = pkg.workloads, pkg.gguf
    cfg = _cfg(pkg)
    w = W.make_weights(cfg)
    layer = 3
    path = str(tmp_path / f"ckpt_{dtype}.gguf")
    G.save_gguf(path, G.moe_block_tensors(layer, w), {"model.name": G.GGUFValue("String", "noor-test")},
                dtype=dtype)
    if dtype == "f16":  # what the file holds, as f32
        for f in ("gate", "bias", "scales", "w_gate", "w_up", "w_down", "dense_gate", "dense_up", "dense_down"):
            setattr(w, f, getattr(w, f).astype(np.float16).astype(np.float32))
    x = W.bf16_bits(W.make_tokens(cfg))
    a = _handle(pkg, cfg)
    a.load_gguf(path, layer)
    b = _handle(pkg, cfg)
    b.load_weights(w)
    oa, ia, wa, ca = a.forward_host(x)
    ob, ib, wb, cb = b.forward_host(x)
    assert np.array_equal(oa, ob) and np.array_equal(ia, ib) and np.array_equal(wa, wb) and np.array_equal(ca, cb)
    with pytest.raises(pkg.api.NoorMoEError):
        a.load_gguf(path, layer + 1)  # no such block
    a.close()
    b.close()


def test_gguf_sandwich_norm(pkg, tmp_path):
    W, G = pkg.workloads, pkg.gguf
    cfg = _cfg(pkg)
    w = W.make_weights(cfg)
    rng = np.random.default_rng(1)
    pre = (1 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32)
    post = (1 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32)
    layer = 2
    path = str(tmp_path / "ckpt_norm.gguf")
    G.save_gguf(path, G.moe_block_tensors(layer, w, pre, post), {})
    x = W.bf16_bits(3.0 * W.make_tokens(cfg))
    a = _handle(pkg, cfg)
    a.load_gguf(path, layer, norm_eps=1e-6)
    b = _handle(pkg, cfg)
    b.load_weights(w)
    b.set_sandwich(pre, post, 1e-6, float(np.float32(1.0) / np.sqrt(np.float32(layer + 1))))
    oa = a.ffn_sublayer_host(x)[0]
    ob = b.ffn_sublayer_host(x)[0]
    assert np.array_equal(oa, ob)
    a.close()
    b.close()


def test_gguf_wrong_shape_is_refused(pkg, tmp_path):
    W, G = pkg.workloads, pkg.gguf
    cfg = _cfg(pkg)
    w = W.make_weights(cfg)
    t = G.moe_block_tensors(0, w)
    t["blocks.0.moe.experts.5.w_down"] = t["blocks.0.moe.experts.5.w_down"][:, :-8].copy()  # [ff, d-8], not [ff, d]
    path = str(tmp_path / "bad_shape.gguf")
    G.save_gguf(path, t, {})
    a = _handle(pkg, cfg)
    with pytest.raises(pkg.api.NoorMoEError) as e:
        a.load_gguf(path, 0)
    assert e.value.code == 1 and "experts.5.w_down" in str(e.value)
    a.close()
