"""ctypes binding of libnoor_moe.so and the host-side mirror of noor-core's
MoE layer API.

The classes below keep the names, fields and call shapes of the reference
(crates/noor-core/src/layers/moe.rs, ffn.rs, parallel_ffn.rs and
crates/noor-train/src/optim/smebu.rs) so code written against the Rust API
reads the same; `forward` hands the whole layer to the CUDA library in one
call through the C ABI declared in include/noor_moe.h.

There is no CPU fallback: if the shared library is missing or no CUDA device
is present, the calls raise.
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import List, Optional, Sequence

import numpy as np

from . import workloads as _w

_HERE = os.path.dirname(os.path.abspath(__file__))
# NOOR_MOE_CHECK=1 loads the bounds-checked debug build (build.py --check).
LIB_PATH = os.path.join(_HERE, "libnoor_moe_check.so" if os.environ.get("NOOR_MOE_CHECK") == "1"
                        else "libnoor_moe.so")

NOOR_MOE_OK = 0
ERR_NAMES = {1: "INVALID", 2: "CUDA", 3: "NCCL", 4: "OOM", 5: "STATE", 6: "TIMEOUT", 7: "UNSUPPORTED"}

DTYPE_F32 = _w.F32
DTYPE_BF16 = _w.BF16
ACT_GELU_TANH = _w.ACT_GELU_TANH
ACT_SILU = _w.ACT_SILU

# Every symbol include/noor_moe.h declares.
EXPORTED_SYMBOLS = (
    "noor_moe_create", "noor_moe_load_weights", "noor_moe_set_bias", "noor_moe_forward",
    "noor_moe_route", "noor_matmul_f32", "noor_moe_last_error", "noor_moe_sync", "noor_moe_destroy",
    "noor_moe_comm_id_size", "noor_moe_comm_get_id", "noor_moe_comm_init_rank",
    "noor_moe_comm_destroy", "noor_moe_profile_begin", "noor_moe_profile_end",
    "noor_moe_launch_count", "noor_moe_ep_plan", "noor_moe_route_static", "noor_moe_ep_transport",
    "noor_moe_utilization", "noor_moe_smebu_update", "noor_moe_smebu_momentum", "noor_moe_get_bias",
    "noor_moe_ffn_sublayer_forward", "noor_moe_set_sandwich", "noor_moe_load_gguf", "noor_gguf_tensor_info",
    "noor_gguf_read_f32", "noor_moe_peer_plan",
)

EP_TRANSPORTS = {0: "none", 1: "nccl", 2: "peer"}


class NoorMoEError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"noor_moe error {code} ({ERR_NAMES.get(code, '?')}): {msg}")
        self.code = code


class Desc(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("expert_ff", ctypes.c_int32), ("dense_ff", ctypes.c_int32), ("has_shared", ctypes.c_int32),
        ("has_dense", ctypes.c_int32), ("dtype", ctypes.c_int32), ("dense_act", ctypes.c_int32),
        ("device", ctypes.c_int32), ("world_size", ctypes.c_int32), ("rank", ctypes.c_int32),
        ("max_tokens", ctypes.c_int64),
    ]


_lib = None
_vp = ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)
_fpp = ctypes.POINTER(_fp)
_i64 = ctypes.c_int64


def lib() -> ctypes.CDLL:
    """Load libnoor_moe.so (built in-tree by build.py).  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    L = ctypes.CDLL(LIB_PATH)
    L.noor_moe_create.argtypes = [ctypes.POINTER(Desc), _vp, ctypes.POINTER(_vp)]
    L.noor_moe_load_weights.argtypes = [_vp, _fp, _fp, _fp, _fpp, _fpp, _fpp, _fpp, _fpp]
    L.noor_moe_set_bias.argtypes = [_vp, _fp]
    L.noor_moe_forward.argtypes = [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]
    L.noor_moe_route.argtypes = [_vp, _vp, _i64, _vp, _vp, _vp, _vp]
    L.noor_matmul_f32.argtypes = [_fp, _fp, _fp, _i64, _i64, _i64]
    L.noor_moe_last_error.restype = ctypes.c_char_p
    L.noor_moe_last_error.argtypes = []
    L.noor_moe_sync.argtypes = [_vp, _vp]
    L.noor_moe_destroy.argtypes = [_vp]
    L.noor_moe_destroy.restype = None
    L.noor_moe_comm_id_size.argtypes = []
    L.noor_moe_comm_get_id.argtypes = [_vp]
    L.noor_moe_comm_init_rank.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]
    L.noor_moe_comm_destroy.argtypes = [_vp]
    L.noor_moe_profile_begin.argtypes = [_vp, ctypes.c_int]
    L.noor_moe_profile_end.argtypes = [_vp, ctypes.c_char_p, _fp, ctypes.POINTER(ctypes.c_int32),
                                       ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    L.noor_moe_launch_count.argtypes = [_vp]
    L.noor_moe_launch_count.restype = ctypes.c_int64
    L.noor_moe_ep_transport.argtypes = [_vp]
    L.noor_moe_ep_transport.restype = ctypes.c_int
    L.noor_moe_utilization.argtypes = [_vp, _vp, _vp, ctypes.c_int, _vp]
    L.noor_moe_smebu_update.argtypes = [_vp, ctypes.c_float, ctypes.c_float, ctypes.c_float, _vp]
    L.noor_moe_smebu_momentum.argtypes = [_vp, _vp, _vp]
    L.noor_moe_get_bias.argtypes = [_vp, _vp]
    L.noor_moe_ffn_sublayer_forward.argtypes = [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]
    L.noor_moe_set_sandwich.argtypes = [_vp, _vp, _vp, ctypes.c_double, ctypes.c_float]
    L.noor_moe_load_gguf.argtypes = [_vp, ctypes.c_char_p, ctypes.c_int32, ctypes.c_double]
    L.noor_gguf_tensor_info.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _vp, _vp, _vp]
    L.noor_gguf_read_f32.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _vp, _i64]
    L.noor_moe_peer_plan.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int] + [_vp] * 7
    L.noor_moe_route_static.argtypes = [_vp, _vp, _vp, _vp, _i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, _vp, _vp, _vp, _vp]
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != NOOR_MOE_OK:
        raise NoorMoEError(rc, lib().noor_moe_last_error().decode(errors="replace"))


def _fptr(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.cast(None, _fp)
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def gguf_tensor_info(path: str, name: str):
    """(dims, dtype) of one tensor of a GGUF file, parsed by the library (host only)."""
    dims = np.zeros(8, np.int64)
    nd = ctypes.c_int32(0)
    dt = ctypes.c_int32(0)
    check(lib().noor_gguf_tensor_info(os.fsencode(path), name.encode(), _ptr(dims), ctypes.byref(nd),
                                      ctypes.byref(dt)))
    return [int(v) for v in dims[:nd.value]], int(dt.value)


def gguf_read_f32(path: str, name: str) -> np.ndarray:
    """One tensor of a GGUF file as f32, read by the library (host only)."""
    dims, _ = gguf_tensor_info(path, name)
    out = np.empty(int(np.prod(dims)) if dims else 1, np.float32)
    check(lib().noor_gguf_read_f32(os.fsencode(path), name.encode(), _ptr(out), out.size))
    return out.reshape(dims)


def peer_plan(cnt: np.ndarray, me: int, BM: int) -> dict:
    """Rank `me`'s plan under the peer-memory exchange from the count matrix
    cnt [G, E] -- the device's arithmetic, run on the host."""
    cnt = np.ascontiguousarray(cnt, np.int64)
    G, E = cnt.shape
    out = {k: np.zeros(E + 1 if k in ("grp_row", "grp_mtile") else E, np.int32)
           for k in ("grp_row", "grp_mtile", "grp_widx", "grp_orank", "grp_oshift", "dest_base")}
    out["counts_glob"] = np.zeros(E, np.int64)
    check(lib().noor_moe_peer_plan(_ptr(cnt), G, E, me, BM, _ptr(out["grp_row"]), _ptr(out["grp_mtile"]),
                                   _ptr(out["grp_widx"]), _ptr(out["grp_orank"]), _ptr(out["grp_oshift"]),
                                   _ptr(out["dest_base"]), _ptr(out["counts_glob"])))
    return out


def matmul_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The matmul boundary (kernels.rs:141-163): C = A.B, f32, on the GPU."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"matmul inner dimensions must match: {k} vs {k2}")
    c = np.empty((m, n), np.float32)
    check(lib().noor_matmul_f32(_fptr(a), _fptr(b), _fptr(c), m, k, n))
    return c


# ------------------------------------------------------------------ handle


class Handle:
    """Owns one noor_moe_handle (one layer on one device)."""

    def __init__(self, d_model: int, n_experts: int, top_k: int, expert_ff: int, dense_ff: int = 0,
                 has_shared: bool = False, has_dense: bool = True, dtype: int = DTYPE_BF16,
                 dense_act: int = ACT_GELU_TANH, device: int = 0, world_size: int = 1, rank: int = 0,
                 max_tokens: int = 0, comm: Optional[int] = None):
        self.desc = Desc(d_model, n_experts, top_k, expert_ff, dense_ff, int(has_shared), int(has_dense),
                         dtype, dense_act, device, world_size, rank, max_tokens)
        self.k = min(top_k, n_experts)
        self._h = ctypes.c_void_p()
        check(lib().noor_moe_create(ctypes.byref(self.desc), ctypes.c_void_p(comm) if comm else None,
                                    ctypes.byref(self._h)))

    @property
    def ptr(self):
        return self._h

    def close(self):
        if self._h:
            lib().noor_moe_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_weights(self, w: "_w.LayerWeights") -> None:
        E = self.desc.n_experts
        arr = lambda xs: (_fp * len(xs))(*[_fptr(x) for x in xs])
        wg = arr([np.ascontiguousarray(w.w_gate[e]) for e in range(E)])
        wu = arr([np.ascontiguousarray(w.w_up[e]) for e in range(E)])
        wd = arr([np.ascontiguousarray(w.w_down[e]) for e in range(E)])
        shared = arr([w.shared_gate, w.shared_up, w.shared_down]) if w.shared_gate is not None else None
        dense = arr([w.dense_gate, w.dense_up, w.dense_down]) if w.dense_gate is not None else None
        check(lib().noor_moe_load_weights(self._h, _fptr(w.gate), _fptr(w.bias), _fptr(w.scales), wg, wu, wd,
                                          shared, dense))

    def set_bias(self, bias: np.ndarray) -> None:
        check(lib().noor_moe_set_bias(self._h, _fptr(np.ascontiguousarray(bias, np.float32))))

    # host-pointer (synchronous) calls: x is f32 for F32 layers, uint16 BF16 bits for BF16 layers
    def forward_host(self, x: np.ndarray, want_route: bool = True):
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.k), np.int32) if want_route else None
        wt = np.empty((T, self.k), np.float32) if want_route else None
        counts = np.empty(self.desc.n_experts, np.int64)
        check(lib().noor_moe_forward(self._h, _ptr(x), _ptr(out), T, _ptr(idx), _ptr(wt), _ptr(counts), None))
        return out, idx, wt, counts

    def route_host(self, x: np.ndarray):
        T = x.shape[0]
        idx = np.empty((T, self.k), np.int32)
        wt = np.empty((T, self.k), np.float32)
        counts = np.empty(self.desc.n_experts, np.int64)
        check(lib().noor_moe_route(self._h, _ptr(x), T, _ptr(idx), _ptr(wt), _ptr(counts), None))
        return idx, wt, counts

    # device-pointer (asynchronous) calls on a CUDA stream
    def forward_device(self, x_ptr: int, out_ptr: int, T: int, stream: int, idx_ptr: int = 0, w_ptr: int = 0,
                       counts_ptr: int = 0) -> None:
        check(lib().noor_moe_forward(self._h, x_ptr, out_ptr, T, idx_ptr or None, w_ptr or None,
                                     counts_ptr or None, stream))

    def route_device(self, x_ptr: int, T: int, idx_ptr: int, w_ptr: int, counts_ptr: int, stream: int) -> None:
        check(lib().noor_moe_route(self._h, x_ptr, T, idx_ptr, w_ptr, counts_ptr or None, stream))

    def sync(self, stream: int = 0) -> None:
        check(lib().noor_moe_sync(self._h, stream or None))

    def launch_count(self) -> int:
        return int(lib().noor_moe_launch_count(self._h))

    def load_gguf(self, path: str, layer: int, norm_eps: float = -1.0) -> None:
        """Load MoE block `layer` of a Noor GGUF checkpoint into the device
        (and its sandwich norm when norm_eps >= 0)."""
        check(lib().noor_moe_load_gguf(self._h, os.fsencode(path), int(layer), float(norm_eps)))

    def set_sandwich(self, pre_w: np.ndarray, post_w: np.ndarray, eps: float, depth_scale: float) -> None:
        pre = np.ascontiguousarray(pre_w, np.float32)
        post = np.ascontiguousarray(post_w, np.float32)
        check(lib().noor_moe_set_sandwich(self._h, _ptr(pre), _ptr(post), float(eps), float(depth_scale)))

    def ffn_sublayer_host(self, x: np.ndarray, want_route: bool = True):
        """out = x + post(F(pre(x))) (block.rs:87-90); host arrays in and out."""
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.k), np.int32) if want_route else None
        wt = np.empty((T, self.k), np.float32) if want_route else None
        counts = np.empty(self.desc.n_experts, np.int64)
        check(lib().noor_moe_ffn_sublayer_forward(self._h, _ptr(x), _ptr(out), T, _ptr(idx), _ptr(wt),
                                                  _ptr(counts), None))
        return out, idx, wt, counts

    def ffn_sublayer_device(self, x_ptr: int, out_ptr: int, T: int, stream: int, counts_ptr: int = 0) -> None:
        check(lib().noor_moe_ffn_sublayer_forward(self._h, x_ptr, out_ptr, T, None, None, counts_ptr or None,
                                                  stream))

    def utilization(self, reset: bool = False, stream: int = 0):
        """(counts [E] int64, tokens) recorded on the device since the last reset."""
        counts = np.empty(self.desc.n_experts, np.int64)
        tokens = ctypes.c_int64(0)
        check(lib().noor_moe_utilization(self._h, _ptr(counts), ctypes.byref(tokens), int(reset), stream or None))
        return counts, int(tokens.value)

    def smebu_update(self, kappa: float, beta: float, lam: float, stream: int = 0) -> None:
        """SMEBU::update + apply_to_router on the device from the recorded utilization."""
        check(lib().noor_moe_smebu_update(self._h, kappa, beta, lam, stream or None))

    def smebu_momentum(self, set_to: Optional[np.ndarray] = None) -> np.ndarray:
        m = np.empty(self.desc.n_experts, np.float32)
        src = None if set_to is None else np.ascontiguousarray(set_to, np.float32)
        check(lib().noor_moe_smebu_momentum(self._h, _ptr(m), _ptr(src)))
        return m

    def get_bias(self) -> np.ndarray:
        b = np.empty(self.desc.n_experts, np.float32)
        check(lib().noor_moe_get_bias(self._h, _ptr(b)))
        return b

    @property
    def ep_transport(self) -> str:
        """How the ranks exchange rows: "none" (one GPU), "nccl" or "peer"."""
        return EP_TRANSPORTS.get(int(lib().noor_moe_ep_transport(self._h)), "?")

    def profile_begin(self, max_launches: int) -> None:
        check(lib().noor_moe_profile_begin(self._h, max_launches))

    def profile_end(self) -> dict:
        n_slots = 32
        names = ctypes.create_string_buffer(32 * n_slots)
        tot = (ctypes.c_float * n_slots)()
        cnt = (ctypes.c_int32 * n_slots)()
        n = ctypes.c_int()
        check(lib().noor_moe_profile_end(self._h, names, tot, cnt, n_slots, ctypes.byref(n)))
        out = {}
        raw = names.raw
        for i in range(n.value):
            nm = raw[32 * i:32 * (i + 1)].split(b"\0", 1)[0].decode()
            out[nm] = {"total_ms": float(tot[i]), "launches": int(cnt[i])}
        return out


def route_static(x_ptr: int, gate_ptr: int, bias_ptr: int, scales_ptr: int, T: int, d: int, E: int, top_k: int,
                 dtype: int, idx_ptr: int, w_ptr: int, counts_ptr: int, stream: int) -> None:
    """noor_moe_route_static: routing with the library's fixed scratch, no
    handle and no device allocation (device pointers, enqueued on `stream`)."""
    check(lib().noor_moe_route_static(x_ptr, gate_ptr, bias_ptr, scales_ptr, T, d, E, top_k, dtype, idx_ptr,
                                      w_ptr, counts_ptr, stream or None))


def comm_get_id() -> bytes:
    n = lib().noor_moe_comm_id_size()
    buf = ctypes.create_string_buffer(n)
    check(lib().noor_moe_comm_get_id(buf))
    return buf.raw


def comm_init_rank(uid: bytes, world_size: int, rank: int, device: int) -> int:
    comm = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(uid, len(uid))
    check(lib().noor_moe_comm_init_rank(buf, world_size, rank, device, ctypes.byref(comm)))
    return comm.value


def comm_destroy(comm: int) -> None:
    check(lib().noor_moe_comm_destroy(ctypes.c_void_p(comm)))


# ------------------------------------------------- mirror of the layer API


class RouteResult:
    """moe.rs:17-22."""

    def __init__(self, indices: List[int], weights: List[float]):
        self.indices = indices
        self.weights = weights


class ExpertUtilization:
    """moe.rs:25-65: per-layer counters fed by the router's histogram."""

    def __init__(self, n_experts: int):
        self.counts = [0] * n_experts
        self.total_tokens = 0

    def record(self, indices: Sequence[int]) -> None:
        self.total_tokens += 1
        for i in indices:
            self.counts[i] += 1

    def record_batch(self, counts: np.ndarray, tokens: int) -> None:
        self.total_tokens += int(tokens)
        for e, c in enumerate(np.asarray(counts).tolist()):
            self.counts[e] += int(c)

    def fractions(self) -> List[float]:
        if self.total_tokens == 0:
            return [0.0] * len(self.counts)
        return [float(np.float32(c) / np.float32(self.total_tokens)) for c in self.counts]

    def active_expert_count(self) -> int:
        return sum(1 for f in self.fractions() if f > 0.01)

    def reset(self) -> None:
        self.counts = [0] * len(self.counts)
        self.total_tokens = 0


def _randn(shape, std, rng) -> np.ndarray:
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


class SwiGLUFFN:
    """ffn.rs:43-68 (weights only; the forward runs inside the layer call)."""

    def __init__(self, d_model: int, d_ffn: int, init_std: float, rng=None):
        rng = rng or np.random.default_rng()
        self.w_gate = _randn((d_model, d_ffn), init_std, rng)
        self.w_up = _randn((d_model, d_ffn), init_std, rng)
        self.w_down = _randn((d_ffn, d_model), init_std, rng)

    def param_count(self) -> int:
        return self.w_gate.size + self.w_up.size + self.w_down.size


class GeGLUFFN(SwiGLUFFN):
    """ffn.rs:5-34: the dense branch (GELU on the gate projection)."""


class MoERouter:
    """moe.rs:5-14, 67-107."""

    def __init__(self, d_model: int, n_experts: int, n_active: int, init_std: float, rng=None):
        rng = rng or np.random.default_rng()
        self.gate = _randn((d_model, n_experts), init_std, rng)
        self.expert_biases = np.zeros(n_experts, np.float32)
        self.expert_scales = np.ones(n_experts, np.float32)
        self.n_experts = n_experts
        self.n_active = n_active
        self._layer: Optional["MoELayer"] = None

    def route(self, x: np.ndarray) -> RouteResult:
        """Route one token (x: [d_model]) on the GPU through noor_moe_route."""
        if self._layer is None:
            raise RuntimeError("MoERouter.route needs the router to belong to a MoELayer")
        h = self._layer._device_handle()
        xx = self._layer._to_dtype(np.asarray(x, np.float32).reshape(1, -1))
        idx, wt, _ = h.route_host(xx)
        return RouteResult([int(i) for i in idx[0]], [float(v) for v in wt[0]])


class MoELayer:
    """moe.rs:110-190.  `forward` runs the whole layer on the GPU."""

    def __init__(self, d_model: int, expert_ffn_dim: int, n_experts: int, n_active: int, has_shared: bool,
                 init_std: float, dtype: int = DTYPE_F32, device: int = 0, rng=None):
        rng = rng or np.random.default_rng()
        self.experts = [SwiGLUFFN(d_model, expert_ffn_dim, init_std, rng) for _ in range(n_experts)]
        self.shared_expert = SwiGLUFFN(d_model, expert_ffn_dim, init_std, rng) if has_shared else None
        self.router = MoERouter(d_model, n_experts, n_active, init_std * 0.5, rng)
        self.router._layer = self
        self.utilization = ExpertUtilization(n_experts)
        self.d_model = d_model
        self.expert_ffn_dim = expert_ffn_dim
        self.dtype = dtype
        self.device = device
        self._handle: Optional[Handle] = None
        self._dense: Optional[GeGLUFFN] = None  # set by ParallelFFN
        self._dense_act = ACT_GELU_TANH
        self._uploaded_bias: Optional[np.ndarray] = None

    # weights -> LayerWeights in the reference layouts
    def _weights(self) -> "_w.LayerWeights":
        E = len(self.experts)
        stack = lambda f: np.ascontiguousarray(np.stack([getattr(e, f) for e in self.experts]), np.float32)
        w = _w.LayerWeights(
            gate=np.ascontiguousarray(self.router.gate, np.float32),
            bias=np.ascontiguousarray(self.router.expert_biases, np.float32),
            scales=np.ascontiguousarray(self.router.expert_scales, np.float32),
            w_gate=stack("w_gate"), w_up=stack("w_up"), w_down=stack("w_down"),
            dense_gate=None, dense_up=None, dense_down=None)
        if self.shared_expert is not None:
            w.shared_gate, w.shared_up, w.shared_down = (self.shared_expert.w_gate, self.shared_expert.w_up,
                                                         self.shared_expert.w_down)
        if self._dense is not None:
            w.dense_gate, w.dense_up, w.dense_down = self._dense.w_gate, self._dense.w_up, self._dense.w_down
        assert w.gate.shape[1] == E
        return w

    def invalidate(self) -> None:
        """Re-upload weights on the next forward (call after editing them)."""
        if self._handle is not None:
            self._handle.close()
        self._handle = None

    def _device_handle(self) -> Handle:
        if self._handle is None:
            dense = self._dense
            h = Handle(self.d_model, len(self.experts), self.router.n_active, self.expert_ffn_dim,
                       dense_ff=dense.w_gate.shape[1] if dense is not None else 0,
                       has_shared=self.shared_expert is not None, has_dense=dense is not None,
                       dtype=self.dtype, dense_act=self._dense_act, device=self.device)
            h.load_weights(self._weights())
            self._handle = h
            self._uploaded_bias = self.router.expert_biases.copy()
        elif not np.array_equal(self._uploaded_bias, self.router.expert_biases):
            self._handle.set_bias(self.router.expert_biases)  # SMEBU apply_to_router path
            self._uploaded_bias = self.router.expert_biases.copy()
        return self._handle

    def _to_dtype(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        return _w.bf16_bits(x) if self.dtype == DTYPE_BF16 else x

    def _from_dtype(self, y: np.ndarray) -> np.ndarray:
        if self.dtype == DTYPE_BF16:
            return (y.astype(np.uint32) << np.uint32(16)).view(np.float32)
        return y

    def _run(self, x: np.ndarray) -> np.ndarray:
        x = np.asarray(x, np.float32)
        if x.ndim != 2 or x.shape[1] != self.d_model:
            raise ValueError(f"expected x of shape (seq_len, {self.d_model}), got {x.shape}")
        h = self._device_handle()
        out, _idx, _wt, counts = h.forward_host(self._to_dtype(x))
        self.utilization.record_batch(counts, x.shape[0])
        return self._from_dtype(out)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """MoELayer::forward (moe.rs:145-177): (seq_len, d_model) -> (seq_len, d_model)."""
        if self._dense is not None:
            raise RuntimeError("this MoELayer belongs to a ParallelFFN; call ParallelFFN.forward")
        return self._run(x)

    def param_count(self) -> int:
        expert = sum(e.param_count() for e in self.experts)
        shared = self.shared_expert.param_count() if self.shared_expert is not None else 0
        router = self.router.gate.size + self.router.expert_biases.size + self.router.expert_scales.size
        return expert + shared + router


class ParallelFFN:
    """parallel_ffn.rs:6-40: (dense(x) + moe(x)) / sqrt(2), one GPU call."""

    def __init__(self, d_model: int, dense_ffn_dim: int, expert_ffn_dim: int, n_experts: int, n_active: int,
                 has_shared: bool, init_std: float, dtype: int = DTYPE_F32, device: int = 0, rng=None):
        rng = rng or np.random.default_rng()
        self.dense = GeGLUFFN(d_model, dense_ffn_dim, init_std, rng)
        self.moe = MoELayer(d_model, expert_ffn_dim, n_experts, n_active, has_shared, init_std, dtype, device, rng)
        self.moe._dense = self.dense

    def forward(self, x: np.ndarray) -> np.ndarray:
        return self.moe._run(x)

    def param_count(self) -> int:
        return self.dense.param_count() + self.moe.param_count()


class RMSNorm:
    """norm.rs:3-28: x / sqrt(mean(x^2) + eps) * weight (weight ones at init)."""

    def __init__(self, d_model: int, eps: float):
        self.weight = np.ones(d_model, np.float32)
        self.eps = float(eps)


class SandwichNorm:
    """norm.rs:31-60: pre/post RMSNorm around a sublayer, both scaled by
    depth_scale = 1/sqrt(layer_idx + 1) (f32)."""

    def __init__(self, d_model: int, eps: float, layer_idx: int):
        self.pre_norm = RMSNorm(d_model, eps)
        self.post_norm = RMSNorm(d_model, eps)
        self.depth_scale = np.float32(1.0) / np.sqrt(np.float32(layer_idx + 1))


def ffn_sublayer_forward(pffn: "ParallelFFN", norm: SandwichNorm, h: np.ndarray) -> np.ndarray:
    """The FFN half of MoEBlock::forward (block.rs:87-90):
    h + post(ParallelFFN(pre(h))), in one GPU call."""
    moe = pffn.moe
    x = np.asarray(h, np.float32)
    if x.ndim != 2 or x.shape[1] != moe.d_model:
        raise ValueError(f"expected h of shape (seq_len, {moe.d_model}), got {x.shape}")
    dev = moe._device_handle()
    dev.set_sandwich(norm.pre_norm.weight, norm.post_norm.weight, norm.pre_norm.eps, float(norm.depth_scale))
    out, _idx, _wt, counts = dev.ffn_sublayer_host(moe._to_dtype(x))
    moe.utilization.record_batch(counts, x.shape[0])
    return moe._from_dtype(out)


class SMEBU:
    """smebu.rs:7-62: momentum expert-bias update (host, E-sized, once per step)."""

    def __init__(self, n_experts: int, kappa: float, beta: float, lam: float):
        self.momentum = np.zeros(n_experts, np.float32)
        self.biases = np.zeros(n_experts, np.float32)
        self.kappa = np.float32(kappa)
        self.beta = np.float32(beta)
        self.lam = np.float32(lam)
        self.n_experts = n_experts

    def update(self, fractions: Sequence[float]) -> None:
        fr = np.asarray(fractions, np.float32)
        assert fr.size == self.n_experts
        f_target = np.float32(1.0) / np.float32(self.n_experts)
        self.momentum = (self.beta * self.momentum + self.lam * (f_target - fr)).astype(np.float32)
        self.biases = (self.kappa * np.tanh(self.momentum / self.kappa)).astype(np.float32)

    def apply_to_router(self, router: MoERouter) -> None:
        assert router.expert_biases.size == self.n_experts
        router.expert_biases[:] = self.biases
