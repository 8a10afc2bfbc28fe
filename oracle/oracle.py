"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle.

`liboracle.so` is the C restatement of the reference MoE (moe_oracle.c);
`_ref/libref_moe.so` is the reference's own fp32 MixtureOfExperts
(src/model/feed_forward.cpp:36-78) compiled from its sources by
oracle/Makefile. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import this module. The product library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "liboracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libref_moe.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i64 = ctypes.c_int64


class OracleLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", _i64), ("experts", _i64), ("top_k", _i64), ("ffn", _i64), ("shared_ffn", _i64),
        ("renormalize", ctypes.c_int32),
        ("router", _f32p), ("router_bias", _f32p), ("gate", _f32p), ("up", _f32p), ("down", _f32p),
        ("shared_gate", _f32p), ("shared_up", _f32p), ("shared_down", _f32p),
    ]


def build() -> None:
    """Builds liboracle.so (and _ref/ when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.oracle_moe_forward.argtypes = [ctypes.POINTER(OracleLayer), _f32p, _i64, _f32p, _i32p, _f32p, _f32p,
                                            _f32p, _f32p, ctypes.c_int]
        _lib.oracle_moe_forward.restype = ctypes.c_int
        _lib.oracle_linear.argtypes = [_f32p, _i64, _i64, _f32p, _i64, _f32p, _f32p, ctypes.c_int]
        _lib.oracle_quantize_q8.argtypes = [_f32p, _i64, _i64, _i64, _i8p, _f32p]
        _lib.oracle_quantize_q8.restype = ctypes.c_int
        _lib.oracle_dequantize_q8.argtypes = [_i8p, _f32p, _i64, _i64, _i64, _f32p]
        _lib.oracle_round_bf16.argtypes = [_f32p, _i64]
        _lib.oracle_synth_stream.argtypes = [ctypes.c_uint64] * 3
        _lib.oracle_synth_stream.restype = ctypes.c_uint64
        _lib.oracle_synth_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, _i64, _i64, _f32p,
                                           ctypes.c_int]
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


def ref():
    global _ref
    if _ref is None:
        _ref = ctypes.CDLL(_REF_PATH)
        _ref.ref_moe_create.argtypes = [_i64] * 5 + [_f32p] * 7
        _ref.ref_moe_create.restype = ctypes.c_void_p
        _ref.ref_moe_run.argtypes = [ctypes.c_void_p, _f32p, _i64, _f32p]
        _ref.ref_moe_run.restype = ctypes.c_int
        _ref.ref_moe_destroy.argtypes = [ctypes.c_void_p]
        _ref.ref_last_error.restype = ctypes.c_char_p
        _ref.ref_set_threads.argtypes = [ctypes.c_int]
        _ref.ref_get_threads.restype = ctypes.c_uint
        _ref.ref_rms_norm.argtypes = [_f32p, _i64, _i64, _f32p, ctypes.c_float]
        _ref.ref_rms_norm.restype = ctypes.c_int
        _ref.ref_attention_head.argtypes = [_f32p, _i64, _f32p, _i64, _i64, _f32p, _i64, _f32p, ctypes.c_float,
                                            _f32p]
        _ref.ref_attention_head.restype = ctypes.c_int
        _i64p = ctypes.POINTER(ctypes.c_int64)
        _ref.ref_page_rope.argtypes = [_f32p, _i64, _i64, _i64, ctypes.c_double, ctypes.c_double, _i64, _i64, _i64p,
                                       _i64p, _f32p]
        _ref.ref_page_rope.restype = ctypes.c_int
    return _ref


def _p(a, t=_f32p):
    return None if a is None else a.ctypes.data_as(t)


def _c(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


# Tensor kinds of the synthetic streams (one stream per tensor per layer).
KIND_ROUTER, KIND_GATE, KIND_UP, KIND_DOWN, KIND_SGATE, KIND_SUP, KIND_SDOWN, KIND_X = 1, 2, 3, 4, 5, 6, 7, 8


def synth(seed: int, layer: int, kind: int, index: int, n: int, sigma: float, offset: int = 0,
          threads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    L = lib()
    L.oracle_synth_fill(seed, L.oracle_synth_stream(layer, kind, index), sigma, offset, n, _p(out), threads)
    return out


def round_bf16(a: np.ndarray) -> np.ndarray:
    a = np.array(a, dtype=np.float32, copy=True)
    lib().oracle_round_bf16(_p(a), a.size)
    return a


def quantize_q8(w: np.ndarray, group: int | None = None):
    w = _c(w)
    rows, cols = w.shape
    group = cols if group is None else group
    q = np.empty((rows, cols), dtype=np.int8)
    s = np.empty((rows, cols // group), dtype=np.float32)
    if lib().oracle_quantize_q8(_p(w), rows, cols, group, _p(q, _i8p), _p(s)) != 0:
        raise ValueError("quantize_q8: group must divide the row width")
    return q, s


def dequantize_q8(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    rows, cols = q.shape
    group = cols // s.shape[1]
    w = np.empty((rows, cols), dtype=np.float32)
    lib().oracle_dequantize_q8(_p(np.ascontiguousarray(q), _i8p), _p(_c(s)), rows, cols, group, _p(w))
    return w


@dataclass
class MoeWeights:
    """One MoE layer's fp32 weights in the reference's stacked layout."""
    router: np.ndarray              # [E, H]
    gate: np.ndarray                # [E*F, H]
    up: np.ndarray                  # [E*F, H]
    down: np.ndarray                # [E*H, F]
    shared_gate: np.ndarray         # [S, H]
    shared_up: np.ndarray           # [S, H]
    shared_down: np.ndarray         # [H, S]
    router_bias: np.ndarray | None = None

    @property
    def hidden(self):
        return self.router.shape[1]

    @property
    def experts(self):
        return self.router.shape[0]

    @property
    def ffn(self):
        return self.gate.shape[0] // self.experts

    @property
    def shared_ffn(self):
        return self.shared_gate.shape[0]


@dataclass
class MoeResult:
    y: np.ndarray
    ids: np.ndarray
    weights: np.ndarray
    logits: np.ndarray
    margin: np.ndarray
    order_margin: np.ndarray


def moe_forward(w: MoeWeights, x: np.ndarray, top_k: int, renormalize: bool, threads: int = 0) -> MoeResult:
    """The restated reference MoE (moe_oracle.c) on fp32 weights."""
    x = _c(x)
    T, H = x.shape
    E = w.experts
    arrays = [_c(a) for a in (w.router, w.router_bias, w.gate, w.up, w.down, w.shared_gate, w.shared_up,
                              w.shared_down)]
    layer = OracleLayer(H, E, top_k, w.ffn, w.shared_ffn, int(renormalize), *[_p(a) for a in arrays])
    y = np.empty((T, H), np.float32)
    ids = np.empty((T, top_k), np.int32)
    wts = np.empty((T, top_k), np.float32)
    logits = np.empty((T, E), np.float32)
    margin = np.empty(T, np.float32)
    om = np.empty(T, np.float32)
    rc = lib().oracle_moe_forward(ctypes.byref(layer), _p(x), T, _p(y), _p(ids, _i32p), _p(wts), _p(logits),
                                  _p(margin), _p(om), threads)
    if rc != 0:
        raise ValueError("oracle_moe_forward: bad argument")
    return MoeResult(y, ids, wts, logits, margin, om)


def linear(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None, threads: int = 0) -> np.ndarray:
    """y [m, n] = x [m, k] . w [n, k]^T (+ bias) in the reference's dot order
    (src/backend/reference/ops.cpp:25-38, :91-109): oracle_linear."""
    x, w = _c(x), _c(w)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float32)
    b = None if bias is None else _c(bias)
    lib().oracle_linear(_p(x), m, k, _p(w), n, None if b is None else _p(b), _p(y), threads)
    return y


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float) -> np.ndarray:
    """The decoder's pre-feed-forward RMSNorm, restated from
    src/backend/reference/ops.cpp:129-141: per row, ss = the sum in index order
    of double(v) * v (np.cumsum adds in order), inv = float(1 / sqrt(ss / H +
    eps)) in double, then weight * (v * inv) in float. weight None = ones."""
    x = _c(x)
    H = x.shape[-1]
    w = np.ones(H, np.float32) if weight is None else _c(weight)
    v = x.astype(np.float64)
    ss = np.cumsum(v * v, axis=-1)[..., -1]
    inv = (1.0 / np.sqrt(ss / np.float64(H) + np.float64(np.float32(eps)))).astype(np.float32)
    return (w * (x * inv[..., None]).astype(np.float32)).astype(np.float32)


def ref_rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float) -> np.ndarray:
    """The reference's own rms_norm (oracle/_ref)."""
    out = np.array(_c(x), copy=True)
    w = np.ones(out.shape[-1], np.float32) if weight is None else _c(weight)
    if ref().ref_rms_norm(_p(out), out.shape[0], out.shape[1], _p(w), eps) != 0:
        raise RuntimeError(ref().ref_last_error().decode())
    return out


class RefMoe:
    """The reference's own MixtureOfExperts::forward (renorm off, no bias)."""

    def __init__(self, w: MoeWeights, top_k: int):
        if w.router_bias is not None:
            raise ValueError("the reference gate has no bias")
        self._keep = [_c(a) for a in (w.router, w.gate, w.up, w.down, w.shared_gate, w.shared_up, w.shared_down)]
        self.hidden = w.hidden
        self.h = ref().ref_moe_create(w.hidden, w.experts, top_k, w.ffn, w.shared_ffn,
                                      *[_p(a) for a in self._keep])
        if not self.h:
            raise RuntimeError(ref().ref_last_error().decode())

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = _c(x)
        y = np.empty_like(x)
        if ref().ref_moe_run(self.h, _p(x), x.shape[0], _p(y)) != 0:
            raise RuntimeError(ref().ref_last_error().decode())
        return y

    def close(self):
        if self.h:
            ref().ref_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def set_ref_threads(n: int) -> None:
    ref().ref_set_threads(n)


def ref_attention_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """The reference's own attention_head (ops.cpp:219-251), no bias."""
    q, k, v = _c(q), _c(k), _c(v)
    out = np.empty((q.shape[0], v.shape[1]), np.float32)
    if ref().ref_attention_head(_p(q), q.shape[0], _p(k), k.shape[0], q.shape[1], _p(v), v.shape[1], None, scale,
                                _p(out)) != 0:
        raise RuntimeError(ref().ref_last_error().decode())
    return out


def ref_page_rope(x: np.ndarray, dim: int, tok_theta: float, page_theta: float, page_pairs: int, page_mod: int,
                  tok: np.ndarray, page: np.ndarray):
    """The reference's own PageRope::apply on x [rows, width] in place
    (page_rope.cpp:8-56); returns (rotated x, its frequency table)."""
    out = np.array(_c(x), copy=True)
    inv = np.empty(dim // 2, np.float32)
    t = np.ascontiguousarray(tok, np.int64)
    pg = np.ascontiguousarray(page, np.int64)
    i64p = ctypes.POINTER(ctypes.c_int64)
    if ref().ref_page_rope(_p(out), out.shape[0], out.shape[1], dim, tok_theta, page_theta, page_pairs, page_mod,
                           t.ctypes.data_as(i64p), pg.ctypes.data_as(i64p), _p(inv)) != 0:
        raise RuntimeError(ref().ref_last_error().decode())
    return out, inv
