"""The synthetic workloads and their seeded inputs.

Every tensor of every layer is one stream of the counter-based generator
(uocr_synth_fill on the device; the tests' host copy of the same formula
gives the same bits). Weights ~ sigma 0.02, activations ~ sigma 1; configs
1-4 round weights (router included, kept in fp32) and the input rows to bf16.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import uocr_moe as M


@dataclass(frozen=True)
class MoeConfig:
    name: str
    seed: int
    hidden: int
    experts: int
    top_k: int
    ffn: int
    shared_ffn: int
    layers: int
    rows: tuple
    bf16_values: bool            # weights and inputs rounded to bf16 values
    weight_format: int = M.WEIGHT_BF16
    renormalize: bool = True
    zipf_s: float | None = None  # router bias skew (config 3)
    gpus: tuple = (1,)
    notes: str = ""

    def dims(self, layers: int | None = None) -> M.Dims:
        return M.Dims(self.hidden, self.experts, self.top_k, self.ffn, self.shared_ffn,
                      self.layers if layers is None else layers)


CONFIGS = {
    0: MoeConfig("c0_cpu_reference", 0, 1024, 16, 2, 512, 0, 1, (64,), False,
                 notes="64 tokens, fp32 values, no shared expert"),
    1: MoeConfig("c1_decode_bf16", 1, 2048, 64, 6, 1024, 2048, 24, (1, 4, 8), True),
    2: MoeConfig("c2_decode_int8", 2, 2048, 64, 6, 1024, 2048, 24, (1, 8), True, weight_format=M.WEIGHT_INT8),
    3: MoeConfig("c3_prefill_bf16_zipf", 3, 2048, 64, 6, 1024, 2048, 1, (32768,), True, zipf_s=1.2,
                 gpus=(1, 2, 4, 8)),
}

# Router bias scale for config 3: b_e = ZIPF_ALPHA * log(p_e), p_e ~ (e + 1)^-s.
# A token selects an expert at most once, so an expert's share of the k slots
# is capped at 1/k and Zipf(1.2) itself (top share 0.29 of 64) is out of reach;
# the target is Zipf with its head capped at 1/k and the excess spread over the
# rest in proportion. With the logit noise these weights give (sd ~0.02 *
# sqrt(2048) ~ 0.9), 0.6 minimises the L1 distance of the top-6 slot shares to
# that target (0.21, against 0.26 at 0.5 and 0.36 at 1.0; calibrated by
# simulation over 20000 rows); measured top-expert share ~0.14.
ZIPF_ALPHA = 0.6


def zipf_bias(experts: int, s: float, alpha: float = ZIPF_ALPHA):
    z = sum((e + 1) ** -s for e in range(experts))
    return [alpha * math.log(((e + 1) ** -s) / z) for e in range(experts)]


def weight_streams(cfg: MoeConfig, layer: int):
    """(name, kind, index, numel) of every weight tensor of one layer, in generation order."""
    H, E, F, S = cfg.hidden, cfg.experts, cfg.ffn, cfg.shared_ffn
    out = [("router", M.KIND_ROUTER, 0, E * H)]
    for e in range(E):
        out += [("gate", M.KIND_GATE, e, F * H), ("up", M.KIND_UP, e, F * H), ("down", M.KIND_DOWN, e, H * F)]
    if S > 0:
        out += [("shared_gate", M.KIND_SGATE, 0, S * H), ("shared_up", M.KIND_SUP, 0, S * H),
                ("shared_down", M.KIND_SDOWN, 0, H * S)]
    return out


def device_layer(cfg: MoeConfig, layer: int, device="cuda"):
    """One layer's weights generated on the device: fp32 router [E,H] and
    bf16 (or fp32 for config 0) stacks in the reference layout."""
    import torch
    H, E, F, S = cfg.hidden, cfg.experts, cfg.ffn, cfg.shared_ffn
    wdt = torch.bfloat16 if cfg.bf16_values else torch.float32
    router = torch.empty(E * H, dtype=wdt, device=device)
    M.synth_fill(router, cfg.seed, layer, M.KIND_ROUTER, 0, 0.02)
    t = {"router": router.float().view(E, H)}
    t["gate"] = torch.empty(E * F, H, dtype=wdt, device=device)
    t["up"] = torch.empty(E * F, H, dtype=wdt, device=device)
    t["down"] = torch.empty(E * H, F, dtype=wdt, device=device)
    for e in range(E):
        M.synth_fill(t["gate"][e * F:(e + 1) * F], cfg.seed, layer, M.KIND_GATE, e, 0.02)
        M.synth_fill(t["up"][e * F:(e + 1) * F], cfg.seed, layer, M.KIND_UP, e, 0.02)
        M.synth_fill(t["down"][e * H:(e + 1) * H], cfg.seed, layer, M.KIND_DOWN, e, 0.02)
    if S > 0:
        t["shared_gate"] = torch.empty(S, H, dtype=wdt, device=device)
        t["shared_up"] = torch.empty(S, H, dtype=wdt, device=device)
        t["shared_down"] = torch.empty(H, S, dtype=wdt, device=device)
        M.synth_fill(t["shared_gate"], cfg.seed, layer, M.KIND_SGATE, 0, 0.02)
        M.synth_fill(t["shared_up"], cfg.seed, layer, M.KIND_SUP, 0, 0.02)
        M.synth_fill(t["shared_down"], cfg.seed, layer, M.KIND_SDOWN, 0, 0.02)
    if cfg.zipf_s is not None:
        t["router_bias"] = torch.tensor(zipf_bias(E, cfg.zipf_s), dtype=torch.float32, device=device)
    return t


def device_input(cfg: MoeConfig, rows: int, device="cuda"):
    import torch
    dt = torch.bfloat16 if cfg.bf16_values else torch.float32
    x = torch.empty(rows, cfg.hidden, dtype=dt, device=device)
    M.synth_fill(x, cfg.seed, 0, M.KIND_X, 0, 1.0)
    return x.float()


def load_layer(plan: M.Plan, cfg: MoeConfig, layer: int, tensors: dict, plan_layer: int | None = None):
    plan.set_layer(layer if plan_layer is None else plan_layer, tensors["router"], tensors["gate"], tensors["up"],
                   tensors["down"], tensors.get("shared_gate"), tensors.get("shared_up"), tensors.get("shared_down"),
                   router_bias=tensors.get("router_bias"), memory=M.MEMORY_DEVICE,
                   dtype=M.DTYPE_BF16 if cfg.bf16_values else M.DTYPE_F32)


# ---- config 4: the synthetic page decoder around the config-1 MoE ---------

@dataclass(frozen=True)
class DecoderConfig:
    name: str
    seed: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    vocab: int
    experts: int
    top_k: int
    ffn: int
    shared_ffn: int
    prefill_rows: int
    decode_steps: int
    rope_theta: float = 1e4
    eps: float = 1e-6


PAGE_DECODER = DecoderConfig("c4_page_decode", 4, 2048, 24, 16, 4, 102400, 64, 6, 1024, 2048, 4096, 1024)


def decoder_device_layer(cfg: DecoderConfig, layer: int, device="cuda"):
    """One decoder layer generated on the device (the streams the CPU
    restatement's synth_weights reads): bf16 matrices, fp32 router, unit
    norm gains."""
    import torch
    H, A, KV = cfg.hidden, cfg.heads * 128, cfg.kv_heads * 128
    E, F, S = cfg.experts, cfg.ffn, cfg.shared_ffn
    bf = torch.bfloat16

    def mat(kind, idx, rows, cols):
        t = torch.empty(rows, cols, dtype=bf, device=device)
        M.synth_fill(t, cfg.seed, layer, kind, idx, 0.02)
        return t
    t = {"input_norm": torch.ones(H, device=device), "post_norm": torch.ones(H, device=device),
         "wq": mat(M.KIND_WQ, 0, A, H), "wk": mat(M.KIND_WK, 0, KV, H), "wv": mat(M.KIND_WV, 0, KV, H),
         "wo": mat(M.KIND_WO, 0, H, A)}
    r = torch.empty(E * H, dtype=bf, device=device)
    M.synth_fill(r, cfg.seed, layer, M.KIND_ROUTER, 0, 0.02)
    t["router"] = r.float().view(E, H)
    for name, kind, rows, cols in (("gate", M.KIND_GATE, F, H), ("up", M.KIND_UP, F, H), ("down", M.KIND_DOWN, H, F)):
        st = torch.empty(E * rows, cols, dtype=bf, device=device)
        for e in range(E):
            M.synth_fill(st[e * rows:(e + 1) * rows], cfg.seed, layer, kind, e, 0.02)
        t[name] = st
    t["shared_gate"] = mat(M.KIND_SGATE, 0, S, H)
    t["shared_up"] = mat(M.KIND_SUP, 0, S, H)
    t["shared_down"] = mat(M.KIND_SDOWN, 0, H, S)
    return t


def decoder_device_head(cfg: DecoderConfig, device="cuda"):
    """(embed, final_norm, lm_head) on the device; the head tensors use the
    layer index past the last layer."""
    import torch
    top = cfg.layers
    emb = torch.empty(cfg.vocab, cfg.hidden, dtype=torch.bfloat16, device=device)
    M.synth_fill(emb, cfg.seed, top, M.KIND_EMBED, 0, 0.02)
    head = torch.empty(cfg.vocab, cfg.hidden, dtype=torch.bfloat16, device=device)
    M.synth_fill(head, cfg.seed, top, M.KIND_LM_HEAD, 0, 0.02)
    return emb, torch.ones(cfg.hidden, device=device), head


def decoder_prompt(cfg: DecoderConfig, rows: int, device="cuda"):
    """rows bf16-valued N(0, 1) embedding rows standing in for image tokens (fp32)."""
    import torch
    x = torch.empty(rows, cfg.hidden, dtype=torch.bfloat16, device=device)
    M.synth_fill(x, cfg.seed, 0, M.KIND_PROMPT, 0, 1.0)
    return x.float()
