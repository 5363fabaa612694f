"""Noor's GGUF v3 checkpoint format on the host: save_gguf / load_gguf with the
names, value types and layout of crates/noor-core/src/gguf.rs (save_gguf
:68-150, load_gguf :153-233, value codes :323-347).

The device loader is the C ABI's noor_moe_load_gguf (Handle.load_gguf),
which reads a MoE block's tensors from the same files straight into the
layer's device layout.  save_gguf writes F32 tensors as the reference does;
`dtype="f16"` writes F16 tensors, which the reference's reader (and the
device loader) also accept.
"""
from __future__ import annotations

import struct
from typing import Dict, Tuple

import numpy as np

MAGIC = 0x46475547  # "GGUF" little-endian
VERSION = 3
ALIGNMENT = 32
TYPE_F32, TYPE_F16 = 0, 1

# metadata value types (gguf.rs:323-347)
V_U32, V_I32, V_F32, V_BOOL, V_STRING, V_F64, V_U64 = range(7)


class GGUFValue:
    """A typed metadata value (gguf.rs:21-30): kind is one of U32, I32, F32,
    F64, Bool, String, U64."""

    CODES = {"U32": V_U32, "I32": V_I32, "F32": V_F32, "Bool": V_BOOL, "String": V_STRING, "F64": V_F64,
             "U64": V_U64}

    def __init__(self, kind: str, value):
        if kind not in self.CODES:
            raise ValueError(f"unknown GGUF value kind {kind}")
        self.kind = kind
        self.value = value

    def __eq__(self, other):
        return isinstance(other, GGUFValue) and self.kind == other.kind and self.value == other.value

    def __repr__(self):
        return f"GGUFValue.{self.kind}({self.value!r})"


def _align(off: int) -> int:
    return (off + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


def _w_string(out: bytearray, s: str) -> None:
    b = s.encode()
    out += struct.pack("<Q", len(b)) + b


def _w_value(out: bytearray, v: GGUFValue) -> None:
    code = GGUFValue.CODES[v.kind]
    out += struct.pack("<I", code)
    if code == V_U32:
        out += struct.pack("<I", v.value)
    elif code == V_I32:
        out += struct.pack("<i", v.value)
    elif code == V_F32:
        out += struct.pack("<f", v.value)
    elif code == V_BOOL:
        out += struct.pack("<B", 1 if v.value else 0)
    elif code == V_STRING:
        _w_string(out, v.value)
    elif code == V_F64:
        out += struct.pack("<d", v.value)
    else:
        out += struct.pack("<Q", v.value)


def save_gguf(path: str, tensors: Dict[str, np.ndarray], metadata: Dict[str, GGUFValue],
              dtype: str = "f32") -> None:
    """save_gguf (gguf.rs:68-150): header, metadata, tensor infos in sorted
    name order, data aligned to 32 bytes.  dtype "f32" (the reference) or
    "f16"."""
    if dtype not in ("f32", "f16"):
        raise ValueError("dtype must be f32 or f16")
    ttype = TYPE_F32 if dtype == "f32" else TYPE_F16
    esize = 4 if dtype == "f32" else 2
    out = bytearray()
    out += struct.pack("<IIQQ", MAGIC, VERSION, len(tensors), len(metadata))
    for k, v in metadata.items():
        _w_string(out, k)
        _w_value(out, v)
    names = sorted(tensors)
    off = 0
    infos = []
    for n in names:
        t = np.asarray(tensors[n])
        infos.append((n, t.shape, off))
        off = _align(off + t.size * esize)
    for n, shape, o in infos:
        _w_string(out, n)
        out += struct.pack("<I", len(shape))
        for dim in shape:
            out += struct.pack("<Q", dim)
        out += struct.pack("<IQ", ttype, o)
    out += b"\0" * (_align(len(out)) - len(out))
    data_start = len(out)
    for n, _shape, o in infos:
        assert len(out) - data_start == o
        t = np.ascontiguousarray(tensors[n], np.float32 if dtype == "f32" else np.float16)
        out += t.astype("<f4" if dtype == "f32" else "<f2").tobytes()
        out += b"\0" * (_align(len(out) - data_start) - (len(out) - data_start))
    with open(path, "wb") as f:
        f.write(out)


def load_gguf(path: str) -> Tuple[Dict[str, GGUFValue], Dict[str, np.ndarray]]:
    """load_gguf (gguf.rs:153-233): (metadata, tensors as f32 arrays)."""
    data = open(path, "rb").read()
    pos = 0

    def take(fmt):
        nonlocal pos
        n = struct.calcsize(fmt)
        if pos + n > len(data):
            raise ValueError("truncated GGUF file")
        v = struct.unpack_from(fmt, data, pos)
        pos += n
        return v if len(v) > 1 else v[0]

    def string():
        nonlocal pos
        n = take("<Q")
        if pos + n > len(data):
            raise ValueError("truncated GGUF file")
        s = data[pos:pos + n].decode()
        pos += n
        return s

    magic, version, n_tensors, n_meta = take("<IIQQ")
    if magic != MAGIC:
        raise ValueError("Not a GGUF file")
    if version != VERSION:
        raise ValueError(f"Unsupported GGUF version: {version}")
    meta: Dict[str, GGUFValue] = {}
    kinds = {v: k for k, v in GGUFValue.CODES.items()}
    for _ in range(n_meta):
        key = string()
        code = take("<I")
        if code not in kinds:
            raise ValueError(f"Unknown value type: {code}")
        fmt = {V_U32: "<I", V_I32: "<i", V_F32: "<f", V_BOOL: "<B", V_F64: "<d", V_U64: "<Q"}.get(code)
        val = string() if code == V_STRING else take(fmt)
        meta[key] = GGUFValue(kinds[code], bool(val) if code == V_BOOL else val)
    infos = []
    for _ in range(n_tensors):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        ttype, off = take("<IQ")
        if ttype not in (TYPE_F32, TYPE_F16):
            raise ValueError(f"Unknown dtype: {ttype}")
        infos.append((name, dims, ttype, off))
    start = _align(pos)
    tensors: Dict[str, np.ndarray] = {}
    for name, dims, ttype, off in infos:
        n = int(np.prod(dims)) if dims else 1
        dt = np.dtype("<f4") if ttype == TYPE_F32 else np.dtype("<f2")
        a = np.frombuffer(data, dt, count=n, offset=start + off)
        tensors[name] = a.astype(np.float32).reshape(dims)
    return meta, tensors


def moe_block_tensors(layer: int, w, pre_norm=None, post_norm=None) -> Dict[str, np.ndarray]:
    """The tensors of MoE block `layer` under the names collect_model_tensors
    gives them (gguf.rs:262-280), from a workloads.LayerWeights."""
    p = f"blocks.{layer}."
    t = {p + "moe.router.gate": w.gate, p + "moe.router.biases": w.bias, p + "moe.router.scales": w.scales}
    for e in range(w.w_gate.shape[0]):
        t[p + f"moe.experts.{e}.w_gate"] = w.w_gate[e]
        t[p + f"moe.experts.{e}.w_up"] = w.w_up[e]
        t[p + f"moe.experts.{e}.w_down"] = w.w_down[e]
    if getattr(w, "shared_gate", None) is not None:
        t[p + "moe.shared.w_gate"], t[p + "moe.shared.w_up"], t[p + "moe.shared.w_down"] = (
            w.shared_gate, w.shared_up, w.shared_down)
    if getattr(w, "dense_gate", None) is not None:
        t[p + "dense.w_gate"], t[p + "dense.w_up"], t[p + "dense.w_down"] = w.dense_gate, w.dense_up, w.dense_down
    if pre_norm is not None:
        t[p + "ffn_norm.pre.weight"] = pre_norm
        t[p + "ffn_norm.post.weight"] = post_norm
    return t

