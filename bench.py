#!/usr/bin/env python
"""bench.py — the decoder MoE hot path on B200, one JSON line on stdout.

Default workload: the 24-layer decode-shape MoE stack in
bf16 — hidden 2048, 64 routed experts (top-6, renormalised) + shared width
2048, expert ffn 1024 — at a token batch of 1. One step = one pass of the
stack (h <- h + MoE_l(h), l = 0..23) over the batch; metric = tokens/s.
Synthetic seeded inputs (the counter-based generator, seed 1), random-init
weights of that architecture; weights (20 GB) exceed L2, so no flush is
needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch T] [--format bf16|int8]
  python bench.py --impl reference ...   # the reference's own fp32 CPU MoE, same metric

N > 1 (torchrun, one rank per GPU): decode does not shard — every rank runs
an independent replica ("replicas only"), value = all ranks' tokens / max
rank time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "grpc-unlimited-ocr_b200"))

HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []
        self.mark_at = 0

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 5.0):
        """Blocks until the sampler has printed once (its start-up takes longer
        than a short timed region), so that samples cover the region."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.01)

    def mark(self):
        """The timed region starts here: only later samples count."""
        self.mark_at = len(self.lines)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        during = self.lines[self.mark_at:]
        # a region shorter than one sampling period: the sample just before it
        lines = during if during else self.lines[max(0, self.mark_at - 1):self.mark_at]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "samples_in_region": len(during) > 0}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def decode_bytes(cfg, active_counts, fmt_int8: bool):
    """Algorithmic bytes of one stack pass and of the gate/up launches, from the
    distinct experts each layer's produced ids touched (U_l)."""
    H, F, S, E = cfg.hidden, cfg.ffn, cfg.shared_ffn, cfg.experts
    eb = 1 if fmt_int8 else 2
    sc = 4 if fmt_int8 else 0  # per-row fp32 scales
    expert_gu = 2 * (F * H * eb + F * sc)
    expert_dn = H * F * eb + H * sc
    shared_gu = 2 * (S * H * eb + S * sc)
    shared_dn = H * S * eb + H * sc
    router = E * H * 4
    total = sum(u * (expert_gu + expert_dn) + shared_gu + shared_dn + router for u in active_counts)
    gate_up = [u * expert_gu + shared_gu for u in active_counts]
    return total, gate_up


def traffic_from_profile(name):
    path = os.path.join(ROOT, "profiles", name)
    try:
        for ln in open(path):
            if ln.startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


def cpu_reference_layer_time(cfg, host_layer, T, budget_s, threads):
    """The reference's own MixtureOfExperts::forward (oracle/_ref) when built,
    else the C restatement; returns (seconds per layer call, kind, cores, reps)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    x = O.synth(cfg.seed, 0, O.KIND_X, 0, T * cfg.hidden, 1.0)
    x = (O.round_bf16(x) if cfg.bf16_values else x).reshape(T, cfg.hidden)
    if O.ref_available():
        O.set_ref_threads(threads)
        ref = O.RefMoe(host_layer, cfg.top_k)
        run, kind = (lambda: ref(x)), "reference"
    else:
        run, kind = (lambda: O.moe_forward(host_layer, x, cfg.top_k, True, threads=threads)), "port"
    run()  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), kind, threads, len(times)


def host_layer_weights(cfg, layer=0):
    """Layer weights generated on the host (no GPU), as the CPU arms need them."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    H, E, F, S = cfg.hidden, cfg.experts, cfg.ffn, cfg.shared_ffn

    def g(kind, idx, n):
        v = O.synth(cfg.seed, layer, kind, idx, n, 0.02)
        return O.round_bf16(v) if cfg.bf16_values else v
    w = O.MoeWeights(
        router=g(O.KIND_ROUTER, 0, E * H).reshape(E, H),
        gate=np.concatenate([g(O.KIND_GATE, e, F * H) for e in range(E)]).reshape(E * F, H),
        up=np.concatenate([g(O.KIND_UP, e, F * H) for e in range(E)]).reshape(E * F, H),
        down=np.concatenate([g(O.KIND_DOWN, e, H * F) for e in range(E)]).reshape(E * H, F),
        shared_gate=g(O.KIND_SGATE, 0, S * H).reshape(S, H), shared_up=g(O.KIND_SUP, 0, S * H).reshape(S, H),
        shared_down=g(O.KIND_SDOWN, 0, H * S).reshape(H, S))
    if cfg.weight_format == 1:  # int8: the CPU runs the dequantised per-channel weights
        deq = lambda a: O.dequantize_q8(*O.quantize_q8(a))  # noqa: E731
        w = O.MoeWeights(w.router, deq(w.gate), deq(w.up), deq(w.down), deq(w.shared_gate), deq(w.shared_up),
                         deq(w.shared_down))
    return w


def measured_tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def run_prefill(M, C, dev, stream, steps, warmup, cpu_budget, want_cpu, rows=None, world=1, rank=0, placement="",
                int8=False):
    """one MoE layer over 32768 rows (8 pages x 4096),
    Zipf-skewed router bias; tokens/s of the layer, per-kernel times, and the
    gate/up GEMM against the bf16 tensor roofline. With world > 1 the layer
    runs expert-parallel: each rank holds its share of the experts and
    32768 / world rows (strong scaling), and the time is the max over ranks.
    `placement` (world > 1): "balanced" = an owner table from the routing
    histogram of a calibration pass (ep.balanced_owner_table: hot experts
    replicated, longest-processing-time assignment), "contiguous" = ranges
    e // (E / G) as the north star names them, "strided" = e % G. The
    calibration pass is this rank's rows through a one-GPU plan, which also
    gives the reference output the expert-parallel rows must equal bit for
    bit. `rows` shrinks the batch (profiling captures only). `int8` (one
    GPU) quantises the layer per output channel; the prefill path then expands
    it to bf16 per layer before the GEMMs (the expansion is timed inside the
    router's interval of kernel_ms)."""
    import torch
    cfg = C.CONFIGS[3]
    total = rows or cfg.rows[0]
    import ep
    start, T = ep.rows_of(total, world, rank)
    E = cfg.experts
    t = C.device_layer(cfg, 0, device=dev)
    x = C.device_input(cfg, total, device=dev)[start:start + T].contiguous()
    y = torch.empty_like(x)
    ids = torch.empty(T, cfg.top_k, dtype=torch.int32, device=dev)
    owner, cbs, y1 = None, None, None
    # The inputs come from torch's default stream; the plans run on `stream`
    # (a non-blocking stream), so wait for them explicitly.
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        # Calibration and reference: this rank's rows through a one-GPU plan.
        single = M.Plan(cfg.dims(), max_rows=max(T, 1), router_bias=True, device=dev.index or 0)
        C.load_layer(single, cfg, 0, t)
        y1 = torch.empty_like(x)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            single.forward(0, x, y1, ids, stream=stream)
            single.check(stream=stream)
        torch.cuda.synchronize()
        single.close()
        mine = torch.bincount(ids.view(-1).long(), minlength=E).to(torch.int64)
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        cbs = [g.cpu().tolist() for g in gathered]
        owner = ep.balanced_owner_table(cbs, world) if placement == "balanced" else \
            ep.owner_table(E, world, placement == "strided")
    plan = M.Plan(cfg.dims(), max_rows=max(T, 1), router_bias=True, device=dev.index or 0,
                  weight_format=M.WEIGHT_INT8 if int8 else M.WEIGHT_BF16,
                  ep_world=world if world > 1 else 0, ep_rank=rank, ep_owner=owner)
    C.load_layer(plan, cfg, 0, t)
    if world > 1:
        ep.connect(plan)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            plan.forward(0, x, y, ids, stream=stream)
        plan.check(stream=stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start_ev = torch.cuda.Event(enable_timing=True)
        end_ev = torch.cuda.Event(enable_timing=True)
        start_ev.record(stream)
        for _ in range(steps):
            plan.forward(0, x, y, stream=stream)
        end_ev.record(stream)
        torch.cuda.synchronize()
        ms = start_ev.elapsed_time(end_ev) / steps
        if world > 1:
            dist.barrier()
        h = x.clone()
        prof = plan.profile_stack(h, iters=3, stream=stream)
        plan.check(stream=stream)
    ep_equal = None
    H, F, S = cfg.hidden, cfg.ffn, cfg.shared_ffn
    if world > 1:
        eq = torch.tensor([1 if torch.equal(y, y1) else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(eq, op=dist.ReduceOp.MIN)
        ep_equal = bool(eq.item())
        del y1
        # Bytes this rank moves over NVLink: the rows it pulls from other
        # ranks — each source row once however many of this rank's experts
        # take it — and the expert outputs of every selection it received,
        # which its down GEMM's epilogue stores back (bf16 rows of H).
        sent = torch.tensor(ep.rows_pulled_from(ids.cpu().numpy(), owner, world, rank), dtype=torch.int64,
                            device=dev)
        sent_all = [torch.empty_like(sent) for _ in range(world)]
        dist.all_gather(sent_all, sent)
        pulled = sum(int(v[rank]) for v in sent_all) * H * 2
        pushed = sum(cbs[s][e] for e in range(E) for s in range(world)
                     if owner[e * world + s] == rank and s != rank) * H * 2
        link = torch.tensor([pulled, prof["pull"], pushed, prof["expert_gemms"]], dtype=torch.float64, device=dev)
        links = [torch.empty_like(link) for _ in range(world)]
        dist.all_gather(links, link)
        links = [v.cpu().tolist() for v in links]
    counts_t = torch.bincount(ids.view(-1).long(), minlength=E)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(counts_t)
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms = float(ms_t[0])
    counts = counts_t.cpu().tolist()
    R = total * cfg.top_k
    gu_flops = R * 4 * F * H + total * 4 * S * H
    dn_flops = R * 2 * F * H + total * 2 * S * H
    total_flops = gu_flops + dn_flops + 2 * total * cfg.experts * H
    peak, peak_src = measured_tensor_peak()
    out = {
        "workload": f"{cfg.name}: 1 layer, {total} rows" + (" (8 pages x 4096)" if total == 32768 else "")
                    + ", Zipf(1.2)-biased router, "
                    + ("int8 per-channel weights expanded to bf16 per layer" if int8 else "bf16"),
        "value": total / (ms * 1e-3), "unit": "tokens/s", "ms_per_layer": ms, "n_gpus": world,
        "scaling": "strong" if world > 1 else None,
        "tflops_per_layer": total_flops / (ms * 1e-3) / 1e12,
        "kernel_ms": {k: round(v, 4) for k, v in prof.items()},
        "expert_rows": counts, "top_expert_share": max(counts) / R,
    }
    if world == 1:
        gu_tf = gu_flops / (prof["gate_up_gemm"] * 1e-3) / 1e12
        dn_tf = dn_flops / (prof["down_gemm"] * 1e-3) / 1e12
        out["roofline"] = {"bound": "tensor", "kernel": "gate_up_gemm (tcgen05 grouped, SwiGLU fused)",
                           "achieved": gu_tf, "peak": peak, "peak_source": peak_src, "unit": "TFLOP/s",
                           "frac": gu_tf / peak, "down_gemm_achieved": dn_tf, "down_gemm_frac": dn_tf / peak,
                           "algorithmic_flops_per_layer": total_flops}
    else:
        per_gpu = total_flops / (ms * 1e-3) / 1e12 / world
        owner_rows = ep.rows_received(owner, cbs, E, world)
        slots = [len(ep.slots_of(owner, E, world, d)) for d in range(world)]
        desc = {"balanced": "load-balanced owner table (hot experts replicated)",
                "strided": "e % G", "contiguous": "contiguous ranges e // (E / G)"}[placement]
        out["parallelism"] = f"expert-parallel x{world}: {desc}, {min(slots)}-{max(slots)} experts and " \
                             f"{total // world} rows per GPU; rows pulled over NVLink by peer loads, outputs stored back by the " \
                             f"down GEMM's epilogue (peer stores)"
        out["roofline"] = {"bound": "tensor", "kernel": "whole layer per GPU", "achieved": per_gpu, "peak": peak,
                           "peak_source": peak_src, "unit": "TFLOP/s", "frac": per_gpu / peak,
                           "algorithmic_flops_per_layer": total_flops}
        out["rows_received_per_rank"] = owner_rows
        out["rows_received_max_over_mean"] = max(owner_rows) / (sum(owner_rows) / world)
        out["experts_per_rank"] = slots
        out["ep_bitwise_equal"] = ep_equal
        # NVLink: bytes each rank pulls / its pull (or combine) kernel time.
        out["nvlink"] = {
            "pull_gbs_per_rank": [round(v[0] / (v[1] * 1e-3) / 1e9, 1) if v[1] > 0 else None for v in links],
            "pull_bytes_per_rank": [int(v[0]) for v in links],
            "push_bytes_per_rank": [int(v[2]) for v in links],
            "push_gbs_over_expert_gemms_per_rank": [round(v[2] / (v[3] * 1e-3) / 1e9, 1) if v[3] > 0 else None
                                                    for v in links],
            "note": "bytes crossing NVLink (rows from or to other ranks only). pull: the pull kernel's peer loads "
                    "(a source row once per owning rank) / its device time. push: expert outputs the down GEMM's epilogue stores into the ranks the rows "
                    "came from, tile by tile while the tensor cores work; their rate is given over the whole "
                    "expert-GEMM phase. Peer copy measured on this pool: 770 GB/s per direction"}
    if world == 1 and rank == 0:
        out["ids_check"] = route_check(cfg, [x.cpu().numpy()], [ids.cpu().numpy()], norm=False,
                                       bias=t["router_bias"].cpu().numpy())
    if want_cpu:
        cpu_rows = min(512, T)
        hw = host_layer_weights(cfg)
        hw.router_bias = t["router_bias"].cpu().numpy()
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        xs = x[:cpu_rows].cpu().numpy()
        O.moe_forward(hw, xs[:8], cfg.top_k, True)
        times = []
        t_end = time.perf_counter() + cpu_budget
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            O.moe_forward(hw, xs, cfg.top_k, True)
            times.append(time.perf_counter() - t0)
        cores = os.cpu_count() or 1
        out["cpu_baseline"] = {"value": cpu_rows / statistics.median(times), "unit": "tokens/s", "cores": cores,
                               "kind": "port",
                               "sample": f"{cpu_rows} of the {T} rows, median of {len(times)} runs (the reference "
                                         "MoE has no router bias, so the C restatement runs this config)"}
    plan.close()
    return out


def run_page_decode(M, C, dev, stream, int8, steps=None, prefill_rows=None, layers=None):
    """the 24-layer synthetic page decoder (RMSNorm, GQA
    attention 16 q / 4 kv heads of 128 with RoPE 1e4, the config-1 MoE block,
    vocab 102400) on one GPU: prefill of 4096 bf16-valued embedding rows, then
    1024 greedy decode steps, each a replayed CUDA graph. Reports prefill
    seconds, decode tokens/s, and the end-to-end figure through the public
    calls with the prompt copied from pinned host memory and the tokens read
    back inside the timed region."""
    import dataclasses

    import torch
    cfg = C.PAGE_DECODER if layers is None else dataclasses.replace(C.PAGE_DECODER, layers=layers)
    n = prefill_rows or cfg.prefill_rows
    steps = steps or cfg.decode_steps
    dec = M.Decoder(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.vocab, max_positions=n + steps,
                    max_prefill=n, experts=cfg.experts, top_k=cfg.top_k, ffn=cfg.ffn, shared_ffn=cfg.shared_ffn,
                    weight_format=M.WEIGHT_INT8 if int8 else M.WEIGHT_BF16, rope_theta=cfg.rope_theta,
                    rms_norm_eps=cfg.eps, device=dev.index or 0)
    for layer in range(cfg.layers):
        t = C.decoder_device_layer(cfg, layer, device=dev)
        dec.set_layer(layer, t, dtype=M.DTYPE_BF16)
        del t
    emb, fnorm, head = C.decoder_device_head(cfg, device=dev)
    dec.set_head(emb, fnorm, head, dtype=M.DTYPE_BF16)
    del emb, head
    torch.cuda.synchronize()
    wbytes, obytes = dec.bytes()
    x = C.decoder_prompt(cfg, n, device=dev)
    toks = torch.empty(steps, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()  # made on the default stream, used on `stream`
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.cuda.stream(stream):
        for _ in range(2):  # warm-up: captures the decode graph
            dec.prefill(x, stream=stream)
            dec.decode(8, toks, stream=stream)
        dec.check(stream=stream)
        torch.cuda.synchronize()
        ev[0].record(stream)
        dec.prefill(x, stream=stream)
        ev[1].record(stream)
        dec.decode(steps, toks, stream=stream)
        ev[2].record(stream)
        torch.cuda.synchronize()
        dec.check(stream=stream)
        prefill_ms = ev[0].elapsed_time(ev[1])
        decode_ms = ev[1].elapsed_time(ev[2])
        tokens = toks.cpu().numpy()
        # End to end through the public calls from host memory.
        x_host = x.cpu().pin_memory()
        t_host = torch.empty(steps, dtype=torch.int32).pin_memory()
        xd = torch.empty_like(x)
        torch.cuda.synchronize()
        ev[0].record(stream)
        xd.copy_(x_host, non_blocking=True)
        dec.prefill(xd, stream=stream)
        dec.decode(steps, toks, stream=stream)
        t_host.copy_(toks, non_blocking=True)
        ev[1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = ev[0].elapsed_time(ev[1])
        # Per-phase device times over the last positions of the sequence
        # (plain launches, events between the phases).
        prof_steps = min(16, steps)
        dec.prefill(xd, stream=stream)
        dec.decode(steps - prof_steps, toks, stream=stream)
        phases = dec.profile_decode(prof_steps, stream=stream)
    import numpy as np
    same = bool(np.array_equal(tokens, t_host.numpy()))
    dec.close()
    # Bytes a decode step must read: every layer's attention and MoE weights
    # (the distinct experts of one row: k), the KV cache up to the position,
    # and the head.
    H, A, KV = cfg.hidden, cfg.heads * 128, cfg.kv_heads * 128
    eb = 1 if int8 else 2
    attn_w = (A + 2 * KV) * H * eb + H * A * eb
    moe_w = (cfg.top_k * 3 * cfg.ffn * H + 3 * cfg.shared_ffn * H) * eb + cfg.experts * H * 4
    head_w = cfg.vocab * H * eb
    mean_pos = n + steps / 2
    kv_bytes = cfg.layers * mean_pos * 2 * KV * 2
    step_bytes = cfg.layers * (attn_w + moe_w) + head_w + kv_bytes
    hbm_peak, peak_kind = measured_peaks()
    step_s = decode_ms * 1e-3 / steps
    return {"workload": f"{cfg.name}: {cfg.layers}-layer decoder, GQA {cfg.heads}q/{cfg.kv_heads}kv x 128, "
                        f"RoPE 1e4, config-1 MoE, vocab {cfg.vocab}; prefill {n} rows then {steps} greedy steps, "
                        + ("int8 per-channel" if int8 else "bf16") + " weights",
            "prefill_s": prefill_ms * 1e-3, "prefill_tokens_per_s": n / (prefill_ms * 1e-3),
            "decode_tokens_per_s": steps / (decode_ms * 1e-3), "decode_ms_per_step": decode_ms / steps,
            "e2e": {"value": steps / (e2e_ms * 1e-3), "unit": "decode tokens/s (prefill included)",
                    "seconds": e2e_ms * 1e-3, "h2d_bytes": n * H * 4, "d2h_bytes": steps * 4,
                    "tokens_equal_device_run": same},
            "roofline": {"bound": "hbm", "achieved": step_bytes / step_s / 1e9, "peak": hbm_peak,
                         "peak_source": peak_kind, "unit": "GB/s", "frac": step_bytes / step_s / 1e9 / hbm_peak,
                         "algorithmic_bytes_per_step": step_bytes,
                         "note": "weights of every layer (k distinct experts), mean KV read, lm_head"},
            "phase_ms_per_step": phases,
            "device_bytes": {"weights": wbytes, "kv_cache_and_scratch": obytes},
            "first_tokens": tokens[:8].tolist(), "distinct_tokens": int(len(set(tokens.tolist())))}


def run_reference_arm(args, cfg, world, rank):
    """--impl reference: the reference's CPU MoE on the host cores, same metric."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    w = host_layer_weights(cfg)
    per_step = []
    kind = None
    for i in range(args.warmup + args.steps):
        t, kind, cores, reps = cpu_reference_layer_time(cfg, w, args.batch, budget_s=2.0, threads=threads)
        if i >= args.warmup:
            per_step.append(t)
    layer_s = statistics.median(per_step)
    step_s = layer_s * cfg.layers
    value = args.batch / step_s
    line = {
        "impl": "reference", "metric": "MoE layer tokens/s (decode)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: {cfg.layers}-layer MoE stack, batch {args.batch}",
                   "global_batch": args.batch * world, "layers": cfg.layers, "hidden": cfg.hidden,
                   "experts": cfg.experts, "top_k": cfg.top_k, "ffn": cfg.ffn, "shared_ffn": cfg.shared_ffn,
                   "parallelism": "replicas" if world > 1 else "single"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"layer 0 of {cfg.layers}, batch {args.batch}, median of ~2 s of calls per step, "
                                   f"scaled to the {cfg.layers}-layer stack"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if kind == "reference":
        line["note"] = ("reference MixtureOfExperts::forward has no renormalisation; its arithmetic is the same "
                        "as the renormalised config's")
    print(json.dumps(line), flush=True)


def route_check(cfg, inputs, got_ids, eps=1e-6, norm=True, bias=None):
    """Expert ids of every layer against the oracle (outside the timed region):
    the oracle's exact-order router on the layer's input rows (RMSNorm'd when
    `norm`, plus the router `bias` when given).
    Returns rows checked, rows whose ids differ inside the north-star margin
    exemption (k-th vs (k+1)-th gate-logit gap or an order gap below 1e-3),
    and rows that differ outside it (must be 0)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    H, E, K = cfg.hidden, cfg.experts, cfg.top_k
    Fd = 1  # the ids depend on the router alone: zero expert stacks of width 1
    z = np.zeros
    rows = exempt = bad = 0
    for layer, (h, ids) in enumerate(zip(inputs, got_ids)):
        r = O.synth(cfg.seed, layer, O.KIND_ROUTER, 0, E * H, 0.02)
        r = (O.round_bf16(r) if cfg.bf16_values else r).reshape(E, H)
        w = O.MoeWeights(r, z((E * Fd, H), np.float32), z((E * Fd, H), np.float32), z((E * H, Fd), np.float32),
                         z((0, H), np.float32), z((0, H), np.float32), z((H, 0), np.float32))
        if bias is not None:
            w.router_bias = np.asarray(bias, np.float32)
        want = O.moe_forward(w, O.rms_norm(h, None, eps) if norm else h, K, renormalize=True)
        for t in range(h.shape[0]):
            rows += 1
            if np.array_equal(ids[t], want.ids[t]):
                continue
            if want.margin[t] < 1e-3 or want.order_margin[t] < 1e-3:
                exempt += 1
            else:
                bad += 1
    return {"rows_checked": rows, "margin_exempt_rows": exempt, "mismatched_rows_outside_margin": bad,
            "rule": "ids and order equal to the oracle's except rows whose k-th vs (k+1)-th gate-logit margin "
                    "(or an order gap) is below 1e-3"}


def time_decode(plan, x, steps, warmup, stream, clocks=None, barrier=None):
    """Device time per step of the stack at batch x.shape[0] (CUDA events on
    the launching stream, inputs resident in HBM)."""
    import torch
    h = torch.empty_like(x)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            h.copy_(x)
            plan.forward_stack(h, stream=stream)
        plan.check(stream=stream)
        if clocks is not None:
            clocks.start()
            clocks.wait_first()
        if barrier is not None:
            barrier()
        torch.cuda.synchronize()
        if clocks is not None:
            clocks.mark()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            h.copy_(x)
            plan.forward_stack(h, stream=stream)
        end.record(stream)
        torch.cuda.synchronize()
        if barrier is not None:
            barrier()
        clk = clocks.stop() if clocks is not None else None
        plan.check(stream=stream)
    return start.elapsed_time(end) / steps, clk


def decode_ids_and_inputs(plan, cfg, x, stream):
    """Layer by layer (outside any timed region): each layer's input rows and
    produced ids, the distinct experts per layer, and whether the stack's
    output is finite. The layer is h <- h + MoE(RMSNorm(h))."""
    import torch
    T = x.shape[0]
    hh = x.clone()
    y = torch.empty_like(hh)
    ids = torch.empty(T, cfg.top_k, dtype=torch.int32, device=x.device)
    inputs, got, active = [], [], []
    with torch.cuda.stream(stream):
        for layer in range(cfg.layers):
            plan.forward(layer, hh, y, ids, None, stream=stream)
            torch.cuda.synchronize()
            inputs.append(hh.cpu().numpy())
            got.append(ids.cpu().numpy())
            active.append(len(set(got[-1].ravel().tolist())))
            hh = hh + y
        plan.check(stream=stream)
    return inputs, got, active, bool(torch.isfinite(hh).all().item())


def torch_sync():
    import torch
    torch.cuda.synchronize()


def decode_section(plan, cfg, T, fmt_int8, steps, stream, dev, check_routes):
    """One named decode configuration: tokens/s, the step's algorithmic bytes
    (from the distinct experts the produced ids touched) against the measured
    HBM peak, the gate/up kernel's fraction, and the ids check."""
    import moe_configs as C
    x = C.device_input(cfg, T, device=dev)
    torch_sync()
    ms, _ = time_decode(plan, x, steps, 3, stream)
    h = x.clone()
    prof = plan.profile_stack(h, iters=5, stream=stream)
    inputs, got, active, finite = decode_ids_and_inputs(plan, cfg, x, stream)
    step_bytes, gu_bytes = decode_bytes(cfg, active, fmt_int8)
    hbm_peak, peak_kind = measured_peaks()
    gu = (sum(gu_bytes) / len(gu_bytes)) / (prof["gate_up"] * 1e-3) / 1e9
    step_gbs = step_bytes / (ms * 1e-3) / 1e9
    out = {"workload": f"{cfg.name}: {cfg.layers}-layer MoE stack, batch {T}, "
                       + ("int8 per-channel" if fmt_int8 else "bf16") + " weights",
           "batch": T, "value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
           "roofline": {"bound": "hbm", "kernel": "gate_up_decode", "achieved": gu, "peak": hbm_peak,
                        "peak_source": peak_kind, "unit": "GB/s", "frac": gu / hbm_peak,
                        "step_achieved": step_gbs, "step_frac": step_gbs / hbm_peak,
                        "algorithmic_bytes_per_step": step_bytes,
                        "kernel_ms": {k: round(v, 5) for k, v in prof.items()}},
           "distinct_experts_per_layer": active, "stack_output_finite": finite}
    if check_routes:
        out["ids_check"] = route_check(cfg, inputs, got)
    return out, (inputs, got)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--format", default="bf16", choices=["bf16", "int8"])
    ap.add_argument("--layers", type=int, default=None, help="override the stack depth (default 24)")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill sections")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the other named decode configurations (config 1 at batch 4/8, config 2)")
    ap.add_argument("--prefill-rows", type=int, default=None, help="shrink the prefill batch (profiling captures)")
    ap.add_argument("--no-decoder", action="store_true", help="skip the config-4 page decoder section")
    ap.add_argument("--decoder-only", action="store_true",
                    help="run only the config-4 page decoder section (profiling captures)")
    ap.add_argument("--decoder-steps", type=int, default=None, help="decode steps of the page decoder section")
    ap.add_argument("--decoder-prefill", type=int, default=None, help="prefill rows of the page decoder section")
    ap.add_argument("--decoder-format", default="both", choices=["both", "bf16", "int8"])
    ap.add_argument("--decoder-layers", type=int, default=None,
                    help="shrink the page decoder's depth (profiling captures with a few GB on the device)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    import moe_configs as C
    cfg = C.CONFIGS[2 if args.format == "int8" else 1]
    if args.layers:
        import dataclasses
        cfg = dataclasses.replace(cfg, layers=args.layers)
    world, rank, local = dist_setup()

    if args.impl == "reference":
        if world > 1:
            import torch.distributed as dist
            dist.init_process_group("gloo")
        run_reference_arm(args, cfg, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch
    import uocr_moe as M
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    barrier = (lambda: dist.barrier()) if world > 1 else None

    def page_decode_sections():
        fmts = {"both": (False, True), "bf16": (False,), "int8": (True,)}[args.decoder_format]
        return [run_page_decode(M, C, dev, stream, int8, steps=args.decoder_steps, prefill_rows=args.decoder_prefill,
                                layers=args.decoder_layers) for int8 in fmts]

    if args.decoder_only:
        stream = torch.cuda.Stream(device=dev)
        print(json.dumps({"page_decode": page_decode_sections()}), flush=True)
        return

    T = args.batch
    fmt_int8 = args.format == "int8"
    sub_configs = not args.no_configs and world == 1 and args.layers is None
    # Each layer is the decoder's feed-forward block, h <- h + MoE(RMSNorm(h))
    # with unit gains: the layer inputs stay ~N(0, 1) as config 1 specifies
    # (a bare residual stack of N(0, 0.02) SwiGLU layers grows quadratically
    # and overflows by the last layers, which would collapse their routing).
    def make_plan(c, int8, max_rows):
        pl = M.Plan(c.dims(), max_rows=max_rows, weight_format=M.WEIGHT_INT8 if int8 else M.WEIGHT_BF16,
                    renormalize=True, device=local, flags=M.PLAN_PRE_NORM, rms_norm_eps=1e-6)
        for layer in range(c.layers):
            t = C.device_layer(c, layer, device=dev)
            C.load_layer(pl, c, layer, t)
            del t
        torch.cuda.synchronize()
        return pl

    other_batches = [b for b in cfg.rows if b != T] if sub_configs else []
    plan = make_plan(cfg, fmt_int8, max(T, *other_batches) if other_batches else T)
    stream = torch.cuda.Stream(device=dev)
    x = C.device_input(cfg, T, device=dev)
    h = torch.empty_like(x)
    torch.cuda.synchronize()  # made on the default stream, used on `stream`

    clocks = ClockSampler(local)
    ms, clk = time_decode(plan, x, args.steps, args.warmup, stream, clocks=clocks, barrier=barrier)

    with torch.cuda.stream(stream):
        # End to end through the public call with host buffers: pinned x in,
        # h out, both copies inside the timed region.
        x_host = x.cpu().pin_memory()
        h_host = torch.empty_like(x_host).pin_memory()
        for _ in range(3):
            h.copy_(x_host, non_blocking=True)
            plan.forward_stack(h, stream=stream)
            h_host.copy_(h, non_blocking=True)
        torch.cuda.synchronize()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(args.steps):
            h.copy_(x_host, non_blocking=True)
            plan.forward_stack(h, stream=stream)
            h_host.copy_(h, non_blocking=True)
        e_end.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e_start.elapsed_time(e_end) / args.steps

        # Per-kernel device times (same workload, events between the kernels).
        h.copy_(x)
        prof = plan.profile_stack(h, iters=5, stream=stream)
    inputs, got_ids, active, finite = decode_ids_and_inputs(plan, cfg, x, stream)

    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_max, e2e_max = float(times[0]), float(times[1])

    step_bytes, gu_bytes = decode_bytes(cfg, active, fmt_int8)
    hbm_peak, peak_kind = measured_peaks()
    gu_achieved = (sum(gu_bytes) / len(gu_bytes)) / (prof["gate_up"] * 1e-3) / 1e9
    step_gbs = step_bytes / (ms_max * 1e-3) / 1e9
    traffic = traffic_from_profile(f"decode_gate_up_{args.format}_t{T}.txt")

    # The other named decode configurations (one GPU): config 1 (or 2) at its
    # other batch sizes on the same plan, then the other weight format.
    configs = []
    if sub_configs:
        for b in other_batches:
            configs.append(decode_section(plan, cfg, b, fmt_int8, max(20, args.steps // 4), stream, dev,
                                          check_routes=rank == 0)[0])
    plan.close()  # free the stack's weights first
    if sub_configs:
        ocfg = C.CONFIGS[1 if fmt_int8 else 2]
        oplan = make_plan(ocfg, not fmt_int8, max(ocfg.rows))
        for b in ocfg.rows:
            configs.append(decode_section(oplan, ocfg, b, not fmt_int8, max(20, args.steps // 4), stream, dev,
                                          check_routes=rank == 0)[0])
        oplan.close()

    page_decode = []
    if not args.no_decoder and world == 1 and args.layers is None:
        page_decode = page_decode_sections()

    prefill = prefill_int8 = None
    if not args.no_prefill:
        # Expert parallelism (world > 1) places the experts from a calibration
        # histogram (hot experts replicated, load-balanced); the contiguous
        # ranges the north star names and the strided map are measured beside it.
        prefill = run_prefill(M, C, dev, stream, steps=10, warmup=3, cpu_budget=min(10.0, args.cpu_budget),
                              want_cpu=not args.no_cpu_baseline and world == 1 and rank == 0,
                              rows=args.prefill_rows, world=world, rank=rank,
                              placement="balanced" if world > 1 else "")
        if world > 1:
            for alt_map in ("contiguous", "strided"):
                alt = run_prefill(M, C, dev, stream, steps=10, warmup=3, cpu_budget=0, want_cpu=False,
                                  rows=args.prefill_rows, world=world, rank=rank, placement=alt_map)
                prefill[f"{alt_map}_experts"] = {k: alt[k] for k in (
                    "value", "ms_per_layer", "kernel_ms", "rows_received_per_rank", "rows_received_max_over_mean",
                    "parallelism", "ep_bitwise_equal")}
        elif sub_configs:
            prefill_int8 = run_prefill(M, C, dev, stream, steps=10, warmup=3, cpu_budget=0, want_cpu=False,
                                       rows=args.prefill_rows, int8=True)

    cpu = None
    ids_check = None
    if rank == 0:
        ids_check = route_check(cfg, inputs, got_ids)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_layer0 = host_layer_weights(cfg)
        t_layer, kind, cores, reps = cpu_reference_layer_time(cfg, host_layer0, T, args.cpu_budget,
                                                              os.cpu_count() or 1)
        cpu = {"value": T / (t_layer * cfg.layers), "unit": "tokens/s", "cores": cores, "kind": kind,
               "sample": f"layer 0 of {cfg.layers} at batch {T}: median of {reps} calls over ~{args.cpu_budget:.0f} s, "
                         f"scaled to the {cfg.layers}-layer stack"}

    if rank == 0:
        launches_per_step = 3 * cfg.layers
        line = {
            "metric": "MoE layer tokens/s (decode)",
            "value": world * T / (ms_max * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8" if fmt_int8 else "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: {cfg.layers}-layer MoE stack, batch {T}",
                       "global_batch": T * world, "layers": cfg.layers, "hidden": cfg.hidden,
                       "experts": cfg.experts, "top_k": cfg.top_k, "ffn": cfg.ffn, "shared_ffn": cfg.shared_ffn,
                       "weights": args.format, "renormalize": True,
                       "layer": "h <- h + MoE(RMSNorm(h)), unit RMSNorm gain, eps 1e-6",
                       "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": "no flush: 20 GB of weights per step pass exceed the 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": "gate_up_decode", "achieved": gu_achieved, "peak": hbm_peak,
                         "peak_source": peak_kind, "unit": "GB/s", "frac": gu_achieved / hbm_peak,
                         "traffic": traffic,
                         "step_achieved": step_gbs, "step_frac": step_gbs / hbm_peak,
                         "algorithmic_bytes_per_step": step_bytes,
                         "kernel_ms": {k: round(v, 5) for k, v in prof.items()},
                         "distinct_experts_per_layer": active, "stack_output_finite": finite},
            "ids_check": ids_check,
            "cpu_baseline": cpu,
            "e2e": {"value": world * T / (e2e_max * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * cfg.hidden * 4, "d2h_bytes_per_step": T * cfg.hidden * 4,
                    "ms_per_step": e2e_max},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if configs:
            line["decode_configs"] = configs
        if page_decode:
            line["page_decode"] = page_decode
        if prefill is not None:
            line["prefill"] = prefill
        if prefill_int8 is not None:
            line["prefill_int8"] = prefill_int8
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
