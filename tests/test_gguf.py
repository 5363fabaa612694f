"""GGUF checkpoints on the host (no GPU): the reference's own round-trip
tests (gguf.rs:398-440) against save_gguf / load_gguf, and the library's C
parser (noor_gguf_tensor_info / noor_gguf_read_f32, the reader behind
noor_moe_load_gguf) against the same files: shapes, dtypes, the exact F16
conversion of every half bit pattern, and malformed files refused."""
import os
import struct

import numpy as np
import pytest


def test_save_load_roundtrip(pkg, tmp_path):
    G = pkg.gguf
    path = str(tmp_path / "roundtrip.gguf")
    tensors = {"weight_a": np.array([[1.0, 2.0], [3.0, 4.0]], np.float32),
               "weight_b": np.array([5.0, 6.0, 7.0], np.float32)}
    meta = {"model.name": G.GGUFValue("String", "noor-test"), "model.layers": G.GGUFValue("U32", 16),
            "training.lr": G.GGUFValue("F64", 3e-4)}
    G.save_gguf(path, tensors, meta)
    m, t = G.load_gguf(path)
    assert m["model.name"] == G.GGUFValue("String", "noor-test")
    assert m["model.layers"] == G.GGUFValue("U32", 16)
    assert t["weight_a"].shape == (2, 2) and t["weight_a"].tolist() == [[1.0, 2.0], [3.0, 4.0]]
    assert t["weight_b"].shape == (3,) and t["weight_b"].tolist() == [5.0, 6.0, 7.0]
    # the library's parser sees the same tensors
    assert pkg.api.gguf_tensor_info(path, "weight_a") == ([2, 2], 0)
    assert pkg.api.gguf_read_f32(path, "weight_b").tolist() == [5.0, 6.0, 7.0]


def test_save_load_large_tensor(pkg, tmp_path):
    G = pkg.gguf
    path = str(tmp_path / "large.gguf")
    data = (np.arange(4096, dtype=np.float32) * np.float32(0.001)).reshape(64, 64)
    G.save_gguf(path, {"big": data}, {})
    _, t = G.load_gguf(path)
    assert t["big"].shape == (64, 64)
    assert np.all(np.abs(t["big"] - data) < 1e-7)
    assert np.array_equal(pkg.api.gguf_read_f32(path, "big"), data)


def test_all_metadata_types_and_many_tensors(pkg, tmp_path):
    G = pkg.gguf
    path = str(tmp_path / "meta.gguf")
    meta = {"a": G.GGUFValue("U32", 7), "b": G.GGUFValue("I32", -3), "c": G.GGUFValue("F32", 1.5),
            "d": G.GGUFValue("Bool", True), "e": G.GGUFValue("String", "x" * 100), "f": G.GGUFValue("F64", 2.25),
            "g": G.GGUFValue("U64", 1 << 40)}
    rng = np.random.default_rng(0)
    tensors = {f"t{i}": rng.standard_normal((i + 1, 3)).astype(np.float32) for i in range(17)}
    G.save_gguf(path, tensors, meta)
    m, t = G.load_gguf(path)
    assert m == meta
    for k, v in tensors.items():
        assert np.array_equal(t[k], v)
        assert pkg.api.gguf_tensor_info(path, k) == (list(v.shape), 0)
        assert np.array_equal(pkg.api.gguf_read_f32(path, k), v)


def test_f16_conversion_is_exact_for_every_half(pkg, tmp_path):
    """F16 tensors: the library's half-to-single conversion (tensor.rs:60-80)
    against numpy's, for all 65536 bit patterns (NaN payloads included)."""
    G = pkg.gguf
    path = str(tmp_path / "f16.gguf")
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    G.save_gguf(path, {"h": halves.astype(np.float32)}, {}, dtype="f16")
    assert pkg.api.gguf_tensor_info(path, "h") == ([65536], 1)
    got = pkg.api.gguf_read_f32(path, "h")
    want = halves.astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_malformed_files_are_refused(pkg, tmp_path):
    G = pkg.gguf
    good = str(tmp_path / "good.gguf")
    G.save_gguf(good, {"w": np.ones((8, 8), np.float32)}, {"k": G.GGUFValue("String", "v")})
    blob = open(good, "rb").read()
    cases = {
        "truncated": blob[: len(blob) - 8],
        "header_only": blob[:20],
        "not_gguf": b"GGML" + blob[4:],
        "version2": blob[:4] + struct.pack("<I", 2) + blob[8:],
        "bad_value_type": None,
    }
    # metadata value type 9 (not one of Noor's codes)
    i = blob.index(b"k") + 1
    cases["bad_value_type"] = blob[:i] + struct.pack("<I", 9) + blob[i + 4:]
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.gguf")
        open(p, "wb").write(data)
        with pytest.raises(pkg.api.NoorMoEError) as e:
            pkg.api.gguf_tensor_info(p, "w")
        assert e.value.code == 1, name
    with pytest.raises(pkg.api.NoorMoEError):
        pkg.api.gguf_tensor_info(good, "missing")
    with pytest.raises(pkg.api.NoorMoEError):
        pkg.api.gguf_tensor_info(str(tmp_path / "does_not_exist.gguf"), "w")
