"""Python binding of the C ABI in include/uocr_moe.h and include/uocr_decoder.h
(ctypes over libuocr_moe.so).

This is the host-side mirror tests and bench.py call: torch supplies device
memory and streams; every computation happens in libuocr_moe.so's sm_100a
kernels. There is no fallback: if the library is missing the import of
`lib()` raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libuocr_moe.so")

UOCR_OK = 0
STATUS_NAMES = {0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED", 3: "CUDA", 4: "OUT_OF_MEMORY", 5: "DEVICE",
                6: "TIMEOUT", 7: "COMM"}
WEIGHT_BF16, WEIGHT_INT8 = 0, 1
MEMORY_HOST, MEMORY_DEVICE = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
PLAN_NO_GRAPHS = 1
PLAN_EP_STRIDED = 4
PLAN_PRE_NORM = 8
DECODER_CUDA_CORE_ATTENTION = 1
EP_HANDLE_BYTES = 256

# Synthetic tensor kinds (one generator stream per tensor per layer).
KIND_ROUTER, KIND_GATE, KIND_UP, KIND_DOWN, KIND_SGATE, KIND_SUP, KIND_SDOWN, KIND_X = 1, 2, 3, 4, 5, 6, 7, 8
# ... and the page decoder's tensors (attention, embedding, head, prompt rows, norm gains).
KIND_WQ, KIND_WK, KIND_WV, KIND_WO, KIND_EMBED, KIND_LM_HEAD, KIND_PROMPT, KIND_NORM = 9, 10, 11, 12, 13, 14, 15, 16

# Every symbol include/uocr_decoder.h declares.
DECODER_EXPORTS = [
    "uocr_decoder_create", "uocr_decoder_destroy", "uocr_decoder_bytes", "uocr_decoder_set_layer",
    "uocr_decoder_set_head", "uocr_decoder_prefill", "uocr_decoder_decode", "uocr_decoder_profile_decode",
    "uocr_decoder_check",
]

# Every symbol include/uocr_moe.h declares.
EXPORTS = [
    "uocr_last_error", "uocr_abi_version", "uocr_moe_plan_create", "uocr_moe_plan_destroy", "uocr_moe_plan_bytes",
    "uocr_moe_set_layer", "uocr_moe_set_layer_parts", "uocr_checkpoint_open", "uocr_checkpoint_close",
    "uocr_checkpoint_count", "uocr_checkpoint_tensor", "uocr_moe_load_layer", "uocr_moe_forward", "uocr_moe_router_logits", "uocr_moe_forward_stack", "uocr_moe_check", "uocr_moe_profile_stack",
    "uocr_moe_ep_handle", "uocr_moe_ep_connect", "uocr_moe_ep_connect_local", "uocr_moe_ep_forward_local",
    "uocr_ops_check", "uocr_expert_topk",
    "uocr_expert_ffn_one", "uocr_expert_ffn_one_noalloc", "uocr_expert_ffn_one_q8", "uocr_linear", "uocr_quantize_q8", "uocr_synth_fill", "uocr_synth_stream",
]


class UocrError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class MoeDesc(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int64), ("routed_experts", ctypes.c_int64),
                ("experts_per_token", ctypes.c_int64), ("expert_ffn", ctypes.c_int64),
                ("shared_ffn", ctypes.c_int64), ("layers", ctypes.c_int64), ("max_rows", ctypes.c_int64),
                ("weight_format", ctypes.c_int32), ("renormalize", ctypes.c_int32),
                ("router_bias", ctypes.c_int32), ("device", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("ep_world", ctypes.c_int32), ("ep_rank", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
                ("reserved", ctypes.c_int32), ("ep_owner", ctypes.c_void_p)]


class EpHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * EP_HANDLE_BYTES)]


class LayerSrc(ctypes.Structure):
    _fields_ = [("memory", ctypes.c_int32), ("dtype", ctypes.c_int32), ("router", ctypes.c_void_p),
                ("router_bias", ctypes.c_void_p), ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p),
                ("down", ctypes.c_void_p), ("shared_gate", ctypes.c_void_p), ("shared_up", ctypes.c_void_p),
                ("shared_down", ctypes.c_void_p), ("norm", ctypes.c_void_p)]


class LayerParts(ctypes.Structure):
    _fields_ = [("memory", ctypes.c_int32), ("dtype", ctypes.c_int32), ("router", ctypes.c_void_p),
                ("router_bias", ctypes.c_void_p), ("gate", ctypes.POINTER(ctypes.c_void_p)),
                ("up", ctypes.POINTER(ctypes.c_void_p)), ("down", ctypes.POINTER(ctypes.c_void_p)),
                ("shared_gate", ctypes.c_void_p), ("shared_up", ctypes.c_void_p), ("shared_down", ctypes.c_void_p),
                ("norm", ctypes.c_void_p)]


MAX_TENSOR_RANK = 8


class TensorView(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("rank", ctypes.c_int32), ("shape", ctypes.c_int64 * MAX_TENSOR_RANK),
                ("data", ctypes.c_void_p), ("bytes", ctypes.c_int64)]


_lib = None


class DecoderDesc(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int64), ("layers", ctypes.c_int64), ("heads", ctypes.c_int64),
                ("kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64), ("vocab", ctypes.c_int64),
                ("max_positions", ctypes.c_int64), ("max_prefill", ctypes.c_int64),
                ("routed_experts", ctypes.c_int64), ("experts_per_token", ctypes.c_int64),
                ("expert_ffn", ctypes.c_int64), ("shared_ffn", ctypes.c_int64), ("rope_theta", ctypes.c_float),
                ("rms_norm_eps", ctypes.c_float), ("weight_format", ctypes.c_int32), ("renormalize", ctypes.c_int32),
                ("device", ctypes.c_int32), ("flags", ctypes.c_int32)]


class DecoderLayerSrc(ctypes.Structure):
    _fields_ = [("memory", ctypes.c_int32), ("dtype", ctypes.c_int32)] + [
        (n, ctypes.c_void_p) for n in ("input_norm", "wq", "wk", "wv", "wo", "post_norm", "router", "gate", "up",
                                       "down", "shared_gate", "shared_up", "shared_down")]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built: run grpc-unlimited-ocr_b200/build.py (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
        L.uocr_last_error.restype = ctypes.c_char_p
        L.uocr_moe_plan_create.argtypes = [ctypes.POINTER(MoeDesc), ctypes.POINTER(vp)]
        L.uocr_moe_plan_destroy.argtypes = [vp]
        L.uocr_moe_plan_bytes.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.uocr_moe_set_layer.argtypes = [vp, i64, ctypes.POINTER(LayerSrc), vp]
        L.uocr_moe_set_layer_parts.argtypes = [vp, i64, ctypes.POINTER(LayerParts), vp]
        L.uocr_checkpoint_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        L.uocr_checkpoint_close.argtypes = [vp]
        L.uocr_checkpoint_count.argtypes = [vp, ctypes.POINTER(i64)]
        L.uocr_checkpoint_tensor.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(TensorView)]
        L.uocr_moe_load_layer.argtypes = [vp, vp, i64, i64, vp]
        L.uocr_moe_forward.argtypes = [vp, i64, vp, i64, vp, vp, vp, vp]
        L.uocr_moe_router_logits.argtypes = [vp, i64, vp, i64, vp, vp]
        L.uocr_moe_forward_stack.argtypes = [vp, vp, i64, vp]
        L.uocr_moe_check.argtypes = [vp, vp]
        L.uocr_moe_profile_stack.argtypes = [vp, vp, i64, i32, ctypes.POINTER(f32), vp]
        L.uocr_moe_ep_handle.argtypes = [vp, ctypes.POINTER(EpHandle)]
        L.uocr_moe_ep_connect.argtypes = [vp, ctypes.POINTER(EpHandle)]
        L.uocr_moe_ep_connect_local.argtypes = [ctypes.POINTER(vp), i32]
        L.uocr_moe_ep_forward_local.argtypes = [ctypes.POINTER(vp), i32, i64, ctypes.POINTER(vp), ctypes.POINTER(i64),
                                                ctypes.POINTER(vp), vp]
        L.uocr_ops_check.argtypes = [vp]
        L.uocr_expert_topk.argtypes = [vp, i64, i64, i64, i32, vp, vp, vp]
        L.uocr_expert_ffn_one.argtypes = [vp, i64, i64, vp, vp, vp, vp, vp, i64, vp, vp]
        L.uocr_expert_ffn_one_noalloc.argtypes = [vp, i64, i64, vp, vp, vp, vp, vp, i64, vp, vp]
        L.uocr_expert_ffn_one_q8.argtypes =[vp, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, i64, vp, vp]
        L.uocr_quantize_q8.argtypes = [vp, i32, i64, i64, i64, vp, vp, vp]
        L.uocr_linear.argtypes = [vp, i64, i64, vp, i64, vp, vp, vp]
        L.uocr_synth_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint64, f32, i64, i64, i32, vp, vp]
        L.uocr_synth_stream.argtypes = [ctypes.c_uint64] * 3
        L.uocr_synth_stream.restype = ctypes.c_uint64
        L.uocr_decoder_create.argtypes = [ctypes.POINTER(DecoderDesc), ctypes.POINTER(vp)]
        L.uocr_decoder_destroy.argtypes = [vp]
        L.uocr_decoder_bytes.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.uocr_decoder_set_layer.argtypes = [vp, i64, ctypes.POINTER(DecoderLayerSrc), vp]
        L.uocr_decoder_set_head.argtypes = [vp, i32, i32, vp, vp, vp, vp]
        L.uocr_decoder_prefill.argtypes = [vp, vp, i64, vp, vp, vp]
        L.uocr_decoder_decode.argtypes = [vp, i64, vp, vp, vp]
        L.uocr_decoder_check.argtypes = [vp, vp]
        L.uocr_decoder_profile_decode.argtypes = [vp, i64, ctypes.POINTER(f32), vp]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != UOCR_OK:
        raise UocrError(rc, lib().uocr_last_error().decode())


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


@dataclass
class Dims:
    hidden: int
    experts: int
    top_k: int
    ffn: int
    shared_ffn: int
    layers: int = 1


class Plan:
    """One MoE stack on one device (uocr_moe_plan)."""

    def __init__(self, dims: Dims, max_rows: int, weight_format: int = WEIGHT_BF16, renormalize: bool = True,
                 router_bias: bool = False, device: int = 0, flags: int = 0, ep_world: int = 0, ep_rank: int = 0,
                 rms_norm_eps: float = 1e-6, ep_owner=None):
        """ep_world > 1 makes this plan rank ep_rank of an expert-parallel
        group (one process per GPU); connect it with ep_connect (see ep.py).
        ep_owner (a sequence of experts * ep_world ints, see
        ep.balanced_owner_table) places the experts; None = the built-in map.
        flags | PLAN_PRE_NORM puts the decoder's RMSNorm (epsilon
        rms_norm_eps) in front of every layer."""
        self.dims = dims
        self.max_rows = max_rows
        self.weight_format = weight_format
        self.ep_world, self.ep_rank = ep_world, ep_rank
        self._owner = None if ep_owner is None else (ctypes.c_int32 * len(ep_owner))(*[int(v) for v in ep_owner])
        desc = MoeDesc(dims.hidden, dims.experts, dims.top_k, dims.ffn, dims.shared_ffn, dims.layers, max_rows,
                       weight_format, int(renormalize), int(router_bias), device, flags, ep_world, ep_rank,
                       rms_norm_eps, 0,
                       None if self._owner is None else ctypes.cast(self._owner, ctypes.c_void_p).value)
        self.desc = desc
        h = ctypes.c_void_p()
        _check(lib().uocr_moe_plan_create(ctypes.byref(desc), ctypes.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().uocr_moe_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def bytes(self):
        w, a = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().uocr_moe_plan_bytes(self.h, ctypes.byref(w), ctypes.byref(a)))
        return w.value, a.value

    def set_layer(self, layer: int, router, gate, up, down, shared_gate=None, shared_up=None, shared_down=None,
                  router_bias=None, memory: int = MEMORY_DEVICE, dtype: int = DTYPE_F32, stream=None, norm=None):
        """Arguments are torch tensors (device memory) or raw addresses;
        norm is the layer's RMSNorm gain (PLAN_PRE_NORM; None = ones)."""
        src = LayerSrc(memory, dtype, _ptr(router), _ptr(router_bias), _ptr(gate), _ptr(up), _ptr(down),
                       _ptr(shared_gate), _ptr(shared_up), _ptr(shared_down), _ptr(norm))
        _check(lib().uocr_moe_set_layer(self.h, layer, ctypes.byref(src), _stream(stream)))

    def set_layer_parts(self, layer: int, router, gate, up, down, shared_gate=None, shared_up=None,
                        shared_down=None, router_bias=None, memory: int = MEMORY_DEVICE, dtype: int = DTYPE_BF16,
                        stream=None, norm=None):
        """One tensor (or raw address) per expert in gate/up/down, as a
        checkpoint holds them; None entries are allowed for experts another
        expert-parallel rank holds."""
        def arr(items):
            return (ctypes.c_void_p * len(items))(*[_ptr(t) for t in items]) if items is not None else None
        g, u, d = arr(gate), arr(up), arr(down)
        src = LayerParts(memory, dtype, _ptr(router), _ptr(router_bias),
                         ctypes.cast(g, ctypes.POINTER(ctypes.c_void_p)) if g is not None else None,
                         ctypes.cast(u, ctypes.POINTER(ctypes.c_void_p)) if u is not None else None,
                         ctypes.cast(d, ctypes.POINTER(ctypes.c_void_p)) if d is not None else None,
                         _ptr(shared_gate), _ptr(shared_up), _ptr(shared_down), _ptr(norm))
        _check(lib().uocr_moe_set_layer_parts(self.h, layer, ctypes.byref(src), _stream(stream)))

    def forward(self, layer: int, x, y, ids=None, weights=None, stream=None, rows: int | None = None):
        rows = x.shape[0] if rows is None else rows
        _check(lib().uocr_moe_forward(self.h, layer, _ptr(x), rows, _ptr(y), _ptr(ids), _ptr(weights),
                                      _stream(stream)))

    def router_logits(self, layer: int, x, logits, stream=None, rows: int | None = None):
        """logits [rows, E] = the layer's router gate on x (+ bias, after the plan's pre-norm)."""
        rows = x.shape[0] if rows is None else rows
        _check(lib().uocr_moe_router_logits(self.h, layer, _ptr(x), rows, _ptr(logits), _stream(stream)))

    def forward_stack(self, h, stream=None, rows: int | None = None):
        rows = h.shape[0] if rows is None else rows
        _check(lib().uocr_moe_forward_stack(self.h, _ptr(h), rows, _stream(stream)))

    DECODE_KERNELS = ("router", "gate_up", "down")
    PREFILL_KERNELS = ("router", "topk", "permute", "gate_up_gemm", "down_gemm", "combine")

    def profile_stack(self, h, iters: int, stream=None, rows: int | None = None):
        """Mean device ms per launch of each kernel of the path, and per stack pass."""
        rows = h.shape[0] if rows is None else rows
        out = (ctypes.c_float * 8)()
        _check(lib().uocr_moe_profile_stack(self.h, _ptr(h), rows, iters, out, _stream(stream)))
        names = self.DECODE_KERNELS if int(out[6]) == 3 else (self.EP_PHASES if self.ep_world > 1
                                                                   else self.PREFILL_KERNELS)
        res = {n: out[i] for i, n in enumerate(names)}
        res["stack"] = out[7]
        return res

    def check(self, stream=None):
        _check(lib().uocr_moe_check(self.h, _stream(stream)))

    # ---- expert parallelism
    EP_PHASES = ("route", "exchange_wait", "pull", "expert_gemms", "shared_and_wait", "combine")

    def ep_handle(self) -> bytes:
        h = EpHandle()
        _check(lib().uocr_moe_ep_handle(self.h, ctypes.byref(h)))
        return bytes(h.bytes)

    def ep_connect(self, handles: list[bytes]):
        arr = (EpHandle * len(handles))()
        for i, b in enumerate(handles):
            if len(b) != EP_HANDLE_BYTES:
                raise ValueError("an EP handle is 256 bytes")
            ctypes.memmove(arr[i].bytes, b, EP_HANDLE_BYTES)
        _check(lib().uocr_moe_ep_connect(self.h, arr))


DTYPE_NAMES = {0: "F32", 1: "BF16", 2: "F16", 3: "I64", 4: "I32", 5: "U8"}


class Checkpoint:
    """A checkpoint opened by the library's own reader (uocr_checkpoint_*):
    a shard index or one .safetensors file, memory-mapped read-only."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().uocr_checkpoint_open(os.fsencode(path), ctypes.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().uocr_checkpoint_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self):
        n = ctypes.c_int64()
        _check(lib().uocr_checkpoint_count(self.h, ctypes.byref(n)))
        return n.value

    def tensor(self, name: str):
        """(dtype name, shape, address, bytes) of a tensor in the mapping."""
        v = TensorView()
        _check(lib().uocr_checkpoint_tensor(self.h, name.encode(), ctypes.byref(v)))
        return DTYPE_NAMES[v.dtype], tuple(v.shape[:v.rank]), v.data, v.bytes

    def load_layer(self, plan: "Plan", layer: int, plan_layer: int, stream=None):
        _check(lib().uocr_moe_load_layer(plan.h, self.h, layer, plan_layer, _stream(stream)))


def ep_connect_local(plans: list[Plan]):
    """Joins plans on one GPU into a group of virtual expert-parallel ranks."""
    arr = (ctypes.c_void_p * len(plans))(*[p.h for p in plans])
    _check(lib().uocr_moe_ep_connect_local(arr, len(plans)))


def ep_forward_local(plans: list[Plan], layer: int, xs, ys, stream=None, rows=None):
    """One layer over a local group: rank i maps xs[i] [rows_i, H] to ys[i]."""
    n = len(plans)
    rows = [x.shape[0] for x in xs] if rows is None else rows
    parr = (ctypes.c_void_p * n)(*[p.h for p in plans])
    xarr = (ctypes.c_void_p * n)(*[_ptr(x) for x in xs])
    yarr = (ctypes.c_void_p * n)(*[_ptr(y) for y in ys])
    rarr = (ctypes.c_int64 * n)(*rows)
    _check(lib().uocr_moe_ep_forward_local(parr, n, layer, xarr, rarr, yarr, _stream(stream)))


def ops_check(stream=None):
    """Synchronises the stream and raises UocrError (UOCR_ERR_DEVICE) when an
    op-level mirror recorded a bad expert id since the last check."""
    _check(lib().uocr_ops_check(_stream(stream)))


def expert_topk(logits, k: int, renormalize: bool, ids, weights, stream=None):
    rows, experts = logits.shape
    _check(lib().uocr_expert_topk(_ptr(logits), rows, experts, k, int(renormalize), _ptr(ids), _ptr(weights),
                                  _stream(stream)))


def expert_ffn_one(x, hidden, ffn, gate, up, down, ids, weights, k, out, stream=None):
    _check(lib().uocr_expert_ffn_one(_ptr(x), hidden, ffn, _ptr(gate), _ptr(up), _ptr(down), _ptr(ids),
                                     _ptr(weights), k, _ptr(out), _stream(stream)))


def expert_ffn_one_noalloc(x, hidden, ffn, gate, up, down, ids, weights, k, out, stream=None):
    """expert_ffn_one for callers that cannot allocate device memory: its
    scratch is a static device array shared by every call (k <= 8,
    ffn <= 8192); calls that overlap on the GPU race."""
    _check(lib().uocr_expert_ffn_one_noalloc(_ptr(x), hidden, ffn, _ptr(gate), _ptr(up), _ptr(down), _ptr(ids),
                                             _ptr(weights), k, _ptr(out), _stream(stream)))


def expert_ffn_one_q8(x, hidden, ffn, gate_q, gate_s, up_q, up_s, down_q, down_s, ids, weights, k, out,
                      stream=None):
    _check(lib().uocr_expert_ffn_one_q8(_ptr(x), hidden, ffn, _ptr(gate_q), _ptr(gate_s), _ptr(up_q), _ptr(up_s),
                                        _ptr(down_q), _ptr(down_s), _ptr(ids), _ptr(weights), k, _ptr(out),
                                        _stream(stream)))


def quantize_q8(w, q, scales, group: int | None = None, stream=None):
    rows, cols = w.shape
    import torch
    dtype = DTYPE_BF16 if w.dtype == torch.bfloat16 else DTYPE_F32
    _check(lib().uocr_quantize_q8(_ptr(w), dtype, rows, cols, cols if group is None else group, _ptr(q),
                                  _ptr(scales), _stream(stream)))


def synth_stream(layer: int, kind: int, index: int) -> int:
    return lib().uocr_synth_stream(layer, kind, index)


def synth_fill(out, seed: int, layer: int, kind: int, index: int, sigma: float, offset: int = 0, stream=None):
    """Fills a contiguous fp32 or bf16 device tensor from the synthetic stream."""
    import torch
    dtype = DTYPE_BF16 if out.dtype == torch.bfloat16 else DTYPE_F32
    _check(lib().uocr_synth_fill(seed, synth_stream(layer, kind, index), sigma, offset, out.numel(), dtype,
                                 _ptr(out), _stream(stream)))


def linear(x, w_bf16, y, bias=None, stream=None):
    """y[m, n] = bf16(x)[m, k] . w[n, k]^T (+ bias) on the tensor cores (uocr_linear)."""
    m, k = x.shape
    n = w_bf16.shape[0]
    _check(lib().uocr_linear(_ptr(x), m, k, _ptr(w_bf16), n, _ptr(bias), _ptr(y), _stream(stream)))


class Decoder:
    """The page decoder around the MoE (uocr_decoder): attention layers with a
    bf16 KV cache, the MoE block of every layer, lm_head and greedy tokens."""

    def __init__(self, hidden, layers, heads, kv_heads, vocab, max_positions, max_prefill, experts, top_k, ffn,
                 shared_ffn, weight_format: int = WEIGHT_BF16, renormalize: bool = True, rope_theta: float = 1e4,
                 rms_norm_eps: float = 1e-6, device: int = 0, flags: int = 0):
        self.desc = DecoderDesc(hidden, layers, heads, kv_heads, 128, vocab, max_positions, max_prefill, experts,
                                top_k, ffn, shared_ffn, rope_theta, rms_norm_eps, weight_format, int(renormalize),
                                device, flags)
        h = ctypes.c_void_p()
        _check(lib().uocr_decoder_create(ctypes.byref(self.desc), ctypes.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().uocr_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def bytes(self):
        w, o = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().uocr_decoder_bytes(self.h, ctypes.byref(w), ctypes.byref(o)))
        return w.value, o.value

    def set_layer(self, layer: int, t: dict, memory: int = MEMORY_DEVICE, dtype: int = DTYPE_BF16, stream=None):
        """t: input_norm, wq, wk, wv, wo, post_norm (fp32 gains), router (fp32)
        and the MoE stacks gate, up, down, shared_gate, shared_up, shared_down."""
        src = DecoderLayerSrc(memory, dtype, *[_ptr(t[n]) for n in (
            "input_norm", "wq", "wk", "wv", "wo", "post_norm", "router", "gate", "up", "down", "shared_gate",
            "shared_up", "shared_down")])
        _check(lib().uocr_decoder_set_layer(self.h, layer, ctypes.byref(src), _stream(stream)))

    def set_head(self, embed, final_norm, lm_head, memory: int = MEMORY_DEVICE, dtype: int = DTYPE_BF16,
                 stream=None):
        _check(lib().uocr_decoder_set_head(self.h, memory, dtype, _ptr(embed), _ptr(final_norm), _ptr(lm_head),
                                           _stream(stream)))

    def prefill(self, embeds, logits=None, token=None, stream=None):
        _check(lib().uocr_decoder_prefill(self.h, _ptr(embeds), embeds.shape[0], _ptr(logits), _ptr(token),
                                          _stream(stream)))

    def decode(self, steps: int, tokens=None, logits=None, stream=None):
        _check(lib().uocr_decoder_decode(self.h, steps, _ptr(tokens), _ptr(logits), _stream(stream)))

    def check(self, stream=None):
        _check(lib().uocr_decoder_check(self.h, _stream(stream)))

    def profile_decode(self, steps: int, stream=None) -> dict:
        """Mean ms per step of each phase (plain launches, events between)."""
        ms = (ctypes.c_float * 5)()
        _check(lib().uocr_decoder_profile_decode(self.h, steps, ms, _stream(stream)))
        return dict(zip(("qkv", "attention", "out_proj", "moe", "lm_head"), [round(v, 5) for v in ms]))
