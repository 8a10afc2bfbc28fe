"""TEST INFRASTRUCTURE ONLY: a CPU restatement of the config-4 synthetic page
decoder around the MoE — RMSNorm, GQA attention with a rotate-half RoPE, the
MoE feed-forward block, the final norm, lm_head and greedy selection — on fp32
weights that hold bf16 (or dequantised per-channel int8) values. It checks the
device decoder; nothing in the product imports it.

What it restates, and from where:
  * the decoder layer (src/model/decoder.cpp:176-203, the CUDA body
    src/model/cuda/cuda_decode_step.cpp:47-70): h = rms_norm(x, input_norm);
    x += o(attention(q(h), k(h), v(h))); x += moe(rms_norm(x, post_norm));
    logits = lm_head(rms_norm(x, final_norm));
  * rms_norm (src/backend/reference/ops.cpp:129-141) through oracle.rms_norm;
  * attention_head (ops.cpp:219-251): s = dot(q, k) * scale, max shift, float
    exp, double total, p = s * float(1 / total), o = sum p * v — here with
    grouped heads (query head h reads key/value head h / (heads / kv_heads))
    and the causal mask of a decoder (key j visible to the query at position
    i when j <= i);
  * the rotate-half rotation of PageRope::apply (src/model/page_rope.cpp:
    37-53): per pair i the fp32 angle pos * inv[i], then (a, b) ->
    (a cos - b sin, b cos + a sin); plain RoPE (inv[i] = float(1 /
    theta^(i / 64)) over all 64 pairs, the page axis left out) is what
    config 4 names, which PageRope itself does not allow;
  * the MoE block through oracle.moe_forward (the reference's
    MixtureOfExperts restated, plus renormalisation);
  * greedy selection: the highest logit, lowest id on a tie (max_element,
    src/runtime/generator.cpp:41-84 with the plain policy).

Rounding points are the device's, so the comparison is about arithmetic
order only: every linear's input row is rounded to bf16 (the reference's CUDA
GEMVs stage x that way, src/backend/cuda/gemv_ops.cu:17-20), and q, k and v
are rounded to bf16 after the rotation (the device keeps its KV cache in bf16).
Products are formed in float64 and rounded to fp32.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import oracle as O

KIND_WQ, KIND_WK, KIND_WV, KIND_WO, KIND_EMBED, KIND_LM_HEAD, KIND_PROMPT, KIND_NORM = 9, 10, 11, 12, 13, 14, 15, 16


@dataclass
class DecoderDims:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    experts: int
    top_k: int
    ffn: int
    shared_ffn: int
    rope_theta: float = 1e4
    eps: float = 1e-6


@dataclass
class DecoderLayer:
    input_norm: np.ndarray   # [H]
    wq: np.ndarray           # [heads*hd, H]
    wk: np.ndarray           # [kv*hd, H]
    wv: np.ndarray           # [kv*hd, H]
    wo: np.ndarray           # [H, heads*hd]
    post_norm: np.ndarray    # [H]
    moe: O.MoeWeights


@dataclass
class DecoderWeights:
    layers: list
    embed: np.ndarray        # [vocab, H]
    final_norm: np.ndarray   # [H]
    lm_head: np.ndarray      # [vocab, H]


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    half = head_dim // 2
    return np.array([1.0 / theta ** (i / half) for i in range(half)], dtype=np.float64).astype(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, head_dim: int, inv: np.ndarray) -> np.ndarray:
    """Rotate-half rotation of every head of x [rows, heads*head_dim] at the
    rows' positions (page_rope.cpp:37-53 with one frequency table)."""
    x = np.array(x, np.float32, copy=True)
    rows = x.shape[0]
    half = head_dim // 2
    ang = (positions.astype(np.float32)[:, None] * inv[None, :]).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    v = x.reshape(rows, -1, head_dim)
    a = v[:, :, :half].copy()
    b = v[:, :, half:].copy()
    v[:, :, :half] = a * c[:, None, :] - b * s[:, None, :]
    v[:, :, half:] = b * c[:, None, :] + a * s[:, None, :]
    return v.reshape(rows, -1)


def attention_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, q_pos: np.ndarray) -> np.ndarray:
    """ops.cpp:219-251 for one head with a causal mask: q [Lq, d] at
    positions q_pos, k/v [Lk, d] at positions 0..Lk-1."""
    s = (q.astype(np.float64) @ k.astype(np.float64).T).astype(np.float32) * np.float32(scale)
    keys = np.arange(k.shape[0])
    s = np.where(keys[None, :] <= q_pos[:, None], s, np.float32(-np.inf)).astype(np.float32)
    peak = s.max(axis=1, keepdims=True)
    e = np.exp((s - peak).astype(np.float64)).astype(np.float32)
    total = e.astype(np.float64).sum(axis=1, keepdims=True)
    p = (e * (1.0 / total).astype(np.float32)).astype(np.float32)
    return (p.astype(np.float64) @ v.astype(np.float64)).astype(np.float32)


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    return (O.round_bf16(np.asarray(x, np.float32)).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def greedy(logits: np.ndarray) -> int:
    return int(np.argmax(logits))  # first (lowest) index of the maximum


@dataclass
class DecoderOracle:
    """The decoder on one sequence: prefill(embeds) then step(token)."""
    dims: DecoderDims
    w: DecoderWeights
    k_cache: list = field(default_factory=list)
    v_cache: list = field(default_factory=list)
    length: int = 0

    def _layer(self, li: int, x: np.ndarray, pos: np.ndarray) -> np.ndarray:
        d, L = self.dims, self.w.layers[li]
        hd = d.head_dim
        inv = rope_inv_freq(hd, d.rope_theta)
        h = O.rms_norm(x, L.input_norm, d.eps)
        q = O.round_bf16(rope(linear(h, L.wq), pos, hd, inv))
        k = O.round_bf16(rope(linear(h, L.wk), pos, hd, inv))
        v = O.round_bf16(linear(h, L.wv))
        self.k_cache[li] = np.concatenate([self.k_cache[li], k.reshape(-1, d.kv_heads, hd)])
        self.v_cache[li] = np.concatenate([self.v_cache[li], v.reshape(-1, d.kv_heads, hd)])
        group = d.heads // d.kv_heads
        out = np.empty((x.shape[0], d.heads * hd), np.float32)
        for hh in range(d.heads):
            g = hh // group
            out[:, hh * hd:(hh + 1) * hd] = attention_head(q[:, hh * hd:(hh + 1) * hd], self.k_cache[li][:, g],
                                                           self.v_cache[li][:, g], 1.0 / np.sqrt(hd), pos)
        x = (x + linear(out, L.wo)).astype(np.float32)
        m = O.moe_forward(L.moe, O.rms_norm(x, L.post_norm, d.eps), d.top_k, renormalize=True)
        return (x + m.y).astype(np.float32)

    def _logits(self, x_last: np.ndarray) -> np.ndarray:
        return linear(O.rms_norm(x_last[None, :], self.w.final_norm, self.dims.eps), self.w.lm_head)[0]

    def prefill(self, embeds: np.ndarray) -> np.ndarray:
        d = self.dims
        self.k_cache = [np.zeros((0, d.kv_heads, d.head_dim), np.float32) for _ in range(d.layers)]
        self.v_cache = [np.zeros((0, d.kv_heads, d.head_dim), np.float32) for _ in range(d.layers)]
        x = np.asarray(embeds, np.float32)
        pos = np.arange(x.shape[0])
        for li in range(d.layers):
            x = self._layer(li, x, pos)
        self.length = x.shape[0]
        return self._logits(x[-1])

    def step(self, token: int) -> np.ndarray:
        x = self.w.embed[token][None, :].astype(np.float32)
        pos = np.array([self.length])
        for li in range(self.dims.layers):
            x = self._layer(li, x, pos)
        self.length += 1
        return self._logits(x[0])


def synth_weights(d: DecoderDims, seed: int, int8: bool = False, norm_sigma: float = 0.0) -> DecoderWeights:
    """The synthetic decoder from the counter-based generator (the same
    streams the device fills): weights ~ 0.02-scaled, bf16 values, norm gains
    1 (+ norm_sigma noise), the router in fp32 storage. int8 dequantises
    every projection per output channel (the router and the embedding stay)."""
    H, hd = d.hidden, d.head_dim

    def g(layer, kind, idx, n, sigma=0.02):
        return O.round_bf16(O.synth(seed, layer, kind, idx, n, sigma))

    def q8(a):
        return O.dequantize_q8(*O.quantize_q8(a)) if int8 else a

    def gain(layer, idx):
        if norm_sigma == 0.0:
            return np.ones(H, np.float32)
        return (1.0 + O.synth(seed, layer, KIND_NORM, idx, H, norm_sigma)).astype(np.float32)

    layers = []
    E, F, S = d.experts, d.ffn, d.shared_ffn
    for li in range(d.layers):
        moe = O.MoeWeights(
            router=g(li, O.KIND_ROUTER, 0, E * H).reshape(E, H),
            gate=q8(np.concatenate([g(li, O.KIND_GATE, e, F * H) for e in range(E)]).reshape(E * F, H)),
            up=q8(np.concatenate([g(li, O.KIND_UP, e, F * H) for e in range(E)]).reshape(E * F, H)),
            down=q8(np.concatenate([g(li, O.KIND_DOWN, e, H * F) for e in range(E)]).reshape(E * H, F)),
            shared_gate=q8(g(li, O.KIND_SGATE, 0, S * H).reshape(S, H)),
            shared_up=q8(g(li, O.KIND_SUP, 0, S * H).reshape(S, H)),
            shared_down=q8(g(li, O.KIND_SDOWN, 0, H * S).reshape(H, S)))
        layers.append(DecoderLayer(
            input_norm=gain(li, 0),
            wq=q8(g(li, KIND_WQ, 0, d.heads * hd * H).reshape(d.heads * hd, H)),
            wk=q8(g(li, KIND_WK, 0, d.kv_heads * hd * H).reshape(d.kv_heads * hd, H)),
            wv=q8(g(li, KIND_WV, 0, d.kv_heads * hd * H).reshape(d.kv_heads * hd, H)),
            wo=q8(g(li, KIND_WO, 0, H * d.heads * hd).reshape(H, d.heads * hd)),
            post_norm=gain(li, 1), moe=moe))
    top = d.layers  # the embedding and head tensors use the layer index past the last layer
    embed = g(top, KIND_EMBED, 0, d.vocab * H).reshape(d.vocab, H)
    lm_head = q8(g(top, KIND_LM_HEAD, 0, d.vocab * H).reshape(d.vocab, H))
    return DecoderWeights(layers, embed, gain(top, 2), lm_head)


def synth_prompt(d: DecoderDims, seed: int, n: int) -> np.ndarray:
    """n rows of bf16-valued N(0, 1) embeddings standing in for image tokens."""
    return O.round_bf16(O.synth(seed, 0, KIND_PROMPT, 0, n * d.hidden, 1.0)).reshape(n, d.hidden)
