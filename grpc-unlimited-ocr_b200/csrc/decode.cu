// Decode-path expert kernels (rows <= 16) on the CUDA cores: weight streaming
// over only the experts the batch selected, plus the shared expert.
//
// One block per SM with 15 streaming warps and one routing warp. A streaming
// warp works through a stream of weight rows (or gate+up row pairs) in steps
// of four 16-byte loads per lane and matrix, the next steps' loads issued
// before the current step's products, so an SM keeps ~90-120 KB in flight;
// work is dealt grid-stride so all SMs stream. bf16 rows are 8 weights per
// load, int8 rows 16 weights per load with the per-output-channel scale
// applied once to a row's sum. The routing warp copies the routing table the
// router built (or builds it from the logits) into shared memory while the
// streaming warps work through the shared expert, which needs none.
// Reference equivalents: expert_gate_up_kernel / expert_down_kernel
// (src/backend/cuda/gemv_ops.cu:145-169) and the shared expert's gemv_kernel
// calls (:133-141, src/model/cuda/cuda_decoder.cpp:119-125, 155-156).
//
//   gate/up: act[slot, f] = bf16(silu(gate[e,f] . x^) * (up[e,f] . x^)), x^ = bf16(x)
//   down:    y[t, c] = shared[t, c] + sum over the row's experts, in id order, of w * (down[e,c] . act)
//
// The combine and the shared add happen in the down kernel in the order the
// reference adds them (src/model/feed_forward.cpp:65-76): no atomics, the
// same bits on every run. Both kernels are launched with programmatic
// dependent launch: gate/up streams the shared expert before it needs the
// router; down issues its first weight loads before it needs the activations.
#include <mutex>

#include "moe_kernels.h"
#include "ptx.cuh"
#include "decode_fmt.cuh"
#include "rms_norm.cuh"
#include "route.cuh"

namespace uocr_b200 {
namespace {

// 16 warps = 4 per SM sub-partition, which leaves 128 registers a thread.
constexpr int kWorkers = 15;                   // streaming warps per block
constexpr int kThreads = (kWorkers + 1) * 32;  // + the routing warp

// 16-byte chunks per lane (and per matrix) in one pipelined step: as many as
// the registers hold without spilling at every row bound (8 spills at 1 row).
// The bytes in flight set the streaming rate here: halving the step cost 30 %
// at one row, and four chunks instead of two gave 21 % at eight.
template <int MaxT>
constexpr int step_chunks() { return 4; }

// Routing source: the router's logits (plan path) or a prepared table (the
// op-level mirrors of expert_ffn_one).
struct RouteSrc {
  const float* logits;
  const DecodeRoute* table;
  int E, K, renorm;
  int* ids_out;  // block 0 writes the rank-order ids/weights here when not null
  float* w_out;
};

// The routing warp builds the table (lane = its lane index) and signals `ready`.
__device__ __forceinline__ void build_route_warp(const RouteSrc& src, int T, SmemRoute* r, int lane, bool with_ids,
                                                 uint64_t* ready) {
  if (src.logits != nullptr) {
    const bool out = with_ids && blockIdx.x == 0;
    route_from_logits(src.logits, T, src.E, src.K, src.renorm, r, lane, 32, 0, out ? src.ids_out : nullptr,
                      out ? src.w_out : nullptr);
  } else {
    route_from_table(src.table, T, r, lane, 32, 0);
  }
  if (lane == 0) mbar_arrive(ready);
}

__device__ __forceinline__ bool wait_ready(uint64_t* ready, ErrorWord* err, int site) {
  if (mbar_wait(ready, 0)) return true;
  raise_error(err, kDevWaitTimeout, site, 0, 0);
  return false;
}

// ---------------------------------------------------------------------------
// gate/up: units are shared rows f (all batch rows), then the U*F
// (selected expert, ffn row) pairs in ascending expert order; streaming warps
// take units grid-stride.
template <typename Rows, int MaxT>
__global__ void __launch_bounds__(kThreads, 1)
    gate_up_decode_kernel(const float* __restrict__ x, int T, int H, int F, int S, Rows gate, Rows up, Rows sgate,
                          Rows sup, RouteSrc rsrc, __nv_bfloat16* __restrict__ act,
                          __nv_bfloat16* __restrict__ act_s, ErrorWord* err, RowNorm norm) {
  using Fm = Fmt<Rows>;
  // bf16-rounded inputs, [T][kQuads][chunks] float4s: the lanes reading
  // consecutive chunks read consecutive 16-byte words (no bank conflicts).
  extern __shared__ __align__(16) float xs[];
  __shared__ SmemRoute sroute;
  __shared__ uint64_t route_ready;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&route_ready, 1);
    fence_mbar_init();
  }
  // The first shared-expert rows of each streaming warp start towards L2
  // while x is staged (the copy engine fetches them; nothing is held). Worth
  // it at one row (0.80 against 0.81 ms per step); at eight it cost 0.4 %.
  if (MaxT == 1 && warp < kWorkers && lane == 0) {
    const int f = blockIdx.x * kWorkers + warp;
    if (f < S) {
      prefetch_l2(Fm::row(sgate, f), static_cast<uint32_t>(H) * Fm::kElemBytes);
      prefetch_l2(Fm::row(sup, f), static_cast<uint32_t>(H) * Fm::kElemBytes);
    }
  }
  // x was written by the grid two launches back, complete before this one
  // started. Staged once as [T][kQuads][chunks] 16-byte words; with the
  // pre-norm the raw rows land first, their inverse RMS is taken from shared
  // memory in the router's summation order (rms_inv_rows, so both see the
  // same bits), and then they are normalised and rounded in place.
  {
    constexpr int kPer = Fm::kPerChunk, kQ = Fm::kQuads;
    const int nch = H / kPer;
    for (int i = threadIdx.x; i < T * H; i += blockDim.x) {
      const int t = i / H, k = i % H, c = k / kPer, q = (k % kPer) >> 2;
      const float v = __ldcg(x + i);
      xs[((static_cast<size_t>(t) * kQ + q) * nch + c) * 4 + (k & 3)] = norm.on ? v : bf16_round(v);
    }
    if (norm.on) {
      __shared__ double s_part[kDecodeMaxRows * kNormWarps];
      __shared__ float s_inv[kDecodeMaxRows];
      __syncthreads();
      float4* xs4 = reinterpret_cast<float4*>(xs);
      // word w of row t (elements 4w .. 4w+3) is chunk w / kQ, quad w % kQ
      rms_inv_rows(
          T, H, norm.eps,
          [&](int t, int w) { return xs4[(static_cast<size_t>(t) * kQ + w % kQ) * nch + w / kQ]; }, s_part,
          s_inv);
      const float4* g4 = reinterpret_cast<const float4*>(norm.gain);
      for (int t = 0; t < T; ++t)
        for (int q = 0; q < kQ; ++q)
          for (int c = threadIdx.x; c < nch; c += blockDim.x) {
            float4& v = xs4[(static_cast<size_t>(t) * kQ + q) * nch + c];
            const float4 g = __ldg(g4 + c * kQ + q);
            const float inv = s_inv[t];
            v = make_float4(bf16_round(rms_apply(v.x, inv, g.x)), bf16_round(rms_apply(v.y, inv, g.y)),
                            bf16_round(rms_apply(v.z, inv, g.z)), bf16_round(rms_apply(v.w, inv, g.w)));
          }
    }
  }
  __syncthreads();
  if (warp == kWorkers) {
    pdl_wait();  // the router's logits
    build_route_warp(rsrc, T, &sroute, lane, true, &route_ready);
    pdl_launch_dependents();
    return;
  }
  const int gw = blockIdx.x * kWorkers + warp, GW = gridDim.x * kWorkers;
  const int nchunks = H * Fm::kElemBytes / 16;

  // The warp's work is a stream of jobs — one (gate row, up row) pair against
  // `ntok` batch rows — cut into steps of kStep 16-byte chunks per lane and
  // matrix. Software-pipelined two deep: the next step's loads are issued
  // before this step's products, so the warp always has rows in flight.
  constexpr int kStep = step_chunks<MaxT>();
  const int spj = (nchunks + 32 * kStep - 1) / (32 * kStep);  // steps per job
  struct Job {
    const uint4* g;
    const uint4* u;
    float gs, us;
    int ntok;
    const int* toks;
    __nv_bfloat16* out;
    int64_t stride;
  };
  float gacc[MaxT], uacc[MaxT];
#pragma unroll
  for (int j = 0; j < MaxT; ++j) gacc[j] = uacc[j] = 0.0f;
  auto run = [&](int njobs, auto&& job) {
    const int nsteps = njobs * spj;
    uint4 ga[kStep], ua[kStep], gb[kStep], ub[kStep];
    auto issue = [&](int s, uint4 (&g)[kStep], uint4 (&u)[kStep]) {
      const Job J = job(s / spj);
      const int base = (s % spj) * 32 * kStep + lane;
#pragma unroll
      for (int c = 0; c < kStep; ++c) {
        const int idx = base + 32 * c;
        if (idx < nchunks) {
          g[c] = ld_stream(J.g + idx);
          u[c] = ld_stream(J.u + idx);
        }
      }
    };
    auto consume = [&](int s, const uint4 (&g)[kStep], const uint4 (&u)[kStep]) {
      const Job J = job(s / spj);
      const int base = (s % spj) * 32 * kStep + lane;
#pragma unroll
      for (int j = 0; j < MaxT; ++j) {
        if (j >= J.ntok) break;
        const float4* xr = reinterpret_cast<const float4*>(xs) +
                           static_cast<size_t>(J.toks == nullptr ? j : J.toks[j]) * Fm::kQuads * nchunks;
#pragma unroll
        for (int c = 0; c < kStep; ++c) {
          const int idx = base + 32 * c;
          if (idx < nchunks) {
            gacc[j] += Fm::dot_xq(g[c], xr + idx, nchunks);
            uacc[j] += Fm::dot_xq(u[c], xr + idx, nchunks);
          }
        }
      }
      if (s % spj == spj - 1) {
#pragma unroll
        for (int j = 0; j < MaxT; ++j) {
          if (j < J.ntok) {
            const float gv = warp_sum(gacc[j]) * J.gs;
            const float uv = warp_sum(uacc[j]) * J.us;
            if (lane == 0) J.out[j * J.stride] = __float2bfloat16_rn(swiglu(gv, uv));
          }
          gacc[j] = uacc[j] = 0.0f;
        }
      }
    };
    if (nsteps > 0) issue(0, ga, ua);
    for (int s = 0; s < nsteps; s += 2) {
      if (s + 1 < nsteps) issue(s + 1, gb, ub);
      consume(s, ga, ua);
      if (s + 2 < nsteps) issue(s + 2, ga, ua);
      if (s + 1 < nsteps) consume(s + 1, gb, ub);
    }
  };

  // Shared expert rows f = gw, gw + GW, ... (no routing needed).
  run(S > gw ? (S - gw + GW - 1) / GW : 0, [&](int k) {
    const int f = gw + k * GW;
    return Job{Fm::row(sgate, f), Fm::row(sup, f), Fm::scale(sgate, f), Fm::scale(sup, f), T, nullptr, act_s + f, S};
  });
  if (!wait_ready(&route_ready, err, 12)) return;
  pdl_launch_dependents();
  const int U = sroute.count;
  run(U * F > gw ? (U * F - gw + GW - 1) / GW : 0, [&](int k) {
    const int q = gw + k * GW;
    const int u = q / F, f = q % F;
    const int64_t row = static_cast<int64_t>(sroute.expert[u]) * F + f;
    const int base = sroute.base[u];
    return Job{Fm::row(gate, row), Fm::row(up, row), Fm::scale(gate, row), Fm::scale(up, row), sroute.ntok[u],
               sroute.slot_tok + base, act + static_cast<int64_t>(base) * F + f, F};
  });
}

// ---------------------------------------------------------------------------
// down + combine: one streaming warp per output channel c (grid-stride): the
// shared down row against every batch row's shared activation, then the
// selected experts' down rows, each finished in registers and added to its
// rows' sums in ascending expert order.
template <typename Rows, int MaxT>
__global__ void __launch_bounds__(kThreads, 1)
    down_decode_kernel(int T, int H, int F, int S, Rows down, Rows sdown, RouteSrc rsrc,
                       const __nv_bfloat16* __restrict__ act, const __nv_bfloat16* __restrict__ act_s,
                       const float* resid, float* y, ErrorWord* err, int stage_act) {
  using Fm = Fmt<Rows>;
  // stage_act: the block copies activations into shared memory once, so the
  // products read them at shared-memory latency instead of one L2 round trip
  // per step: 1 = the shared rows [T, S] then the routed slots [slots, F];
  // 2 = the routed slots only (when both do not fit: the many routed steps
  // read shared memory, the shared row's few steps read L2); 0 = none.
  extern __shared__ __align__(16) __nv_bfloat16 act_sm[];
  __shared__ SmemRoute sroute;
  __shared__ uint64_t route_ready;
  __shared__ float row_sum[kWorkers][kDecodeMaxRows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&route_ready, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kWorkers) {
    // The router grid completed before the gate/up grid released this one
    // (gate/up releases only after its own wait on the router).
    build_route_warp(rsrc, T, &sroute, lane, false, &route_ready);
    pdl_wait();
    pdl_launch_dependents();
    return;
  }
  const int gw = blockIdx.x * kWorkers + warp, GW = gridDim.x * kWorkers;
  // A channel's rows — the shared row, then each selected expert's in
  // ascending id — cut into steps of kStep chunks per lane and pipelined four
  // deep (three steps' loads in flight while one is multiplied). The first
  // steps are issued before waiting for the gate/up grid's activations.
  constexpr int kStep = step_chunks<MaxT>();
  const int nch_s = S * Fm::kElemBytes / 16, nch_f = F * Fm::kElemBytes / 16;
  const int spr_s = S > 0 ? (nch_s + 32 * kStep - 1) / (32 * kStep) : 0;
  const int spr_f = (nch_f + 32 * kStep - 1) / (32 * kStep);
  // int8 at one row with F = 1024: an expert's down row fills half a step,
  // so a step carries two experts' rows (the first's chunks in w[0 .. qpr),
  // the second's in w[qpr .. 2 qpr)): half the dependent steps, the same sums.
  constexpr int qpr = kStep / 2;  // 16-byte chunks of one row per lane in a paired step
  const bool pair = Fm::kElemBytes == 1 && MaxT == 1 && nch_f == 32 * qpr;
  float* sum = row_sum[warp];
  bool waited = false, have_route = false, staged = !stage_act;
  const __nv_bfloat16* acts = stage_act == 1 ? act_sm : act_s;  // [T, S]
  const __nv_bfloat16* actr =
      stage_act == 1 ? act_sm + static_cast<int64_t>(T) * S : (stage_act == 2 ? act_sm : act);  // [slots, F]
  // Every streaming warp calls this exactly once (also on its error paths,
  // so that none waits at the barrier for a warp that left): wait for the
  // activations and the routing table, copy, and meet the other streaming warps.
  auto stage = [&]() -> bool {
    if (staged) return true;
    staged = true;
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    bool good = have_route;
    if (!good) good = have_route = wait_ready(&route_ready, err, 25);
    if (good) {
      const int U = sroute.count;
      const int slots = U > 0 ? sroute.base[U - 1] + sroute.ntok[U - 1] : 0;
      const int n_s = stage_act == 1 ? T * S / 8 : 0, n_r = slots * F / 8;  // 16-byte chunks
      const uint4* src_s = reinterpret_cast<const uint4*>(act_s);
      const uint4* src_r = reinterpret_cast<const uint4*>(act);
      uint4* dst = reinterpret_cast<uint4*>(act_sm);
      for (int i = threadIdx.x; i < n_s + n_r; i += kWorkers * 32)
        dst[i] = i < n_s ? __ldcg(src_s + i) : __ldcg(src_r + (i - n_s));
    }
    named_bar_sync(1, kWorkers * 32);
    return good;
  };
  bool ok = true;
  for (int c = gw; c < H; c += GW) {
    if (lane < kDecodeMaxRows) sum[lane] = 0.0f;
    __syncwarp();
    float acc[MaxT];
#pragma unroll
    for (int j = 0; j < MaxT; ++j) acc[j] = 0.0f;
    int nsteps = spr_s;  // + U * spr_f once the routing table is known
    bool known = false;
    auto learn = [&]() {
      if (known) return true;
      if (!have_route) {
        if (!wait_ready(&route_ready, err, 24)) return false;
        have_route = true;
      }
      nsteps = spr_s + (pair ? (sroute.count + 1) / 2 : sroute.count * spr_f);
      known = true;
      return true;
    };
    auto issue = [&](int st, uint4 (&w)[kStep]) {
      const uint4* p;
      int n, base;
      if (st < spr_s) {
        p = Fm::row(sdown, c);
        n = nch_s;
        base = st * 32 * kStep + lane;
      } else if (pair) {
        const int r0 = 2 * (st - spr_s);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (r0 + h >= sroute.count) break;
          const uint4* pr = Fm::row(down, static_cast<int64_t>(sroute.expert[r0 + h]) * H + c);
#pragma unroll
          for (int q = 0; q < qpr; ++q) w[h * qpr + q] = ld_stream(pr + lane + 32 * q);
        }
        return;
      } else {
        const int r = (st - spr_s) / spr_f;
        p = Fm::row(down, static_cast<int64_t>(sroute.expert[r]) * H + c);
        n = nch_f;
        base = ((st - spr_s) % spr_f) * 32 * kStep + lane;
      }
#pragma unroll
      for (int q = 0; q < kStep; ++q)
        if (base + 32 * q < n) w[q] = ld_stream(p + base + 32 * q);
    };
    auto consume = [&](int st, const uint4 (&w)[kStep]) {
      if (!waited) {
        pdl_wait();  // the activations come from the gate/up grid
        waited = true;
      }
      if (!staged && !stage()) ok = false;
      if (!ok) return;
      if (st < spr_s) {
        const int base = st * 32 * kStep + lane;
#pragma unroll
        for (int t = 0; t < MaxT; ++t) {
          if (t >= T) break;
          const __nv_bfloat16* ar = acts + static_cast<int64_t>(t) * S;
#pragma unroll
          for (int q = 0; q < kStep; ++q)
            if (base + 32 * q < nch_s) acc[t] += Fm::template dot_act<2, (MaxT > 1)>(w[q], ar + (base + 32 * q) * Fm::kPerChunk);
        }
        if (st == spr_s - 1) {
          const float sc = Fm::scale(sdown, c);
#pragma unroll
          for (int t = 0; t < MaxT; ++t) {
            if (t < T) {
              const float v = warp_sum(acc[t]) * sc;
              if (lane == 0) sum[t] = v;
            }
            acc[t] = 0.0f;
          }
        }
        return;
      }
      if (pair) {
        // (int8, one row) two experts' rows, each finished as below.
        const int r0 = 2 * (st - spr_s);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = r0 + h;
          if (r >= sroute.count) break;
          const int b0 = sroute.base[r], n0 = sroute.ntok[r];
          const float sc = Fm::scale(down, static_cast<int64_t>(sroute.expert[r]) * H + c);
          for (int j = 0; j < n0; ++j) {
            const __nv_bfloat16* ar = actr + static_cast<int64_t>(b0 + j) * F;
            float a = 0.0f;
#pragma unroll
            for (int q = 0; q < qpr; ++q)
              a += Fm::template dot_act<2, (MaxT > 1)>(w[h * qpr + q], ar + (lane + 32 * q) * Fm::kPerChunk);
            const float v = warp_sum(a) * sc;
            if (lane == 0) {
              const int t = sroute.slot_tok[b0 + j];
              sum[t] = __fadd_rn(sum[t], __fmul_rn(sroute.slot_w[b0 + j], v));
            }
          }
        }
        return;
      }
      if (Fm::kElemBytes == 2 && spr_f == 1) {
        // (bf16) The expert's whole row is in this step: each of its batch
        // rows is finished here (same sums in the same order as below), with
        // a loop that is not unrolled over the row bound. (The int8 form of
        // this loop spills registers.)
        const int r = st - spr_s;
        const int b0 = sroute.base[r], n0 = sroute.ntok[r];
        const float sc = Fm::scale(down, static_cast<int64_t>(sroute.expert[r]) * H + c);
#pragma unroll 1
        for (int j = 0; j < n0; ++j) {
          const __nv_bfloat16* ar = actr + static_cast<int64_t>(b0 + j) * F;
          float a = 0.0f;
#pragma unroll
          for (int q = 0; q < kStep; ++q)
            if (lane + 32 * q < nch_f) a += Fm::template dot_act<2, (MaxT > 1)>(w[q], ar + (lane + 32 * q) * Fm::kPerChunk);
          const float v = warp_sum(a) * sc;
          if (lane == 0) {
            const int t = sroute.slot_tok[b0 + j];
            sum[t] = __fadd_rn(sum[t], __fmul_rn(sroute.slot_w[b0 + j], v));
          }
        }
        return;
      }
      const int r = (st - spr_s) / spr_f, sr = (st - spr_s) % spr_f;
      const int b0 = sroute.base[r], n0 = sroute.ntok[r];
      const int base = sr * 32 * kStep + lane;
#pragma unroll
      for (int j = 0; j < MaxT; ++j) {
        if (j >= n0) break;
        const __nv_bfloat16* ar = actr + static_cast<int64_t>(b0 + j) * F;
#pragma unroll
        for (int q = 0; q < kStep; ++q)
          if (base + 32 * q < nch_f) acc[j] += Fm::template dot_act<2, (MaxT > 1)>(w[q], ar + (base + 32 * q) * Fm::kPerChunk);
      }
      if (sr == spr_f - 1) {
        const float sc = Fm::scale(down, static_cast<int64_t>(sroute.expert[r]) * H + c);
#pragma unroll
        for (int j = 0; j < MaxT; ++j) {
          if (j < n0) {
            const float v = warp_sum(acc[j]) * sc;
            if (lane == 0) {
              const int t = sroute.slot_tok[b0 + j];
              sum[t] = __fadd_rn(sum[t], __fmul_rn(sroute.slot_w[b0 + j], v));
            }
          }
          acc[j] = 0.0f;
        }
      }
    };
    // Four steps in flight: a ring of four register buffers, unrolled.
    uint4 w0[kStep], w1[kStep], w2[kStep], w3[kStep];
    auto issue_at = [&](int st, uint4 (&w)[kStep]) {
      if (st >= spr_s && !learn()) ok = false;
      if (ok && st < nsteps) issue(st, w);
    };
    issue_at(0, w0);
    issue_at(1, w1);
    issue_at(2, w2);
    for (int st = 0; ok && st < nsteps; st += 4) {
      issue_at(st + 3, w3);
      if (!ok) break;
      consume(st, w0);
      issue_at(st + 4, w0);
      if (!ok) break;
      if (st + 1 < nsteps) consume(st + 1, w1);
      issue_at(st + 5, w1);
      if (!ok) break;
      if (st + 2 < nsteps) consume(st + 2, w2);
      issue_at(st + 6, w2);
      if (!ok) break;
      if (st + 3 < nsteps) consume(st + 3, w3);
    }
    if (!ok || !learn()) {  // (a channel with no rows to stream still needs its routing)
      ok = false;
      break;
    }
    __syncwarp();
    for (int t = lane; t < T; t += 32) {
      const int64_t o = static_cast<int64_t>(t) * H + c;
      y[o] = resid != nullptr ? __fadd_rn(resid[o], sum[t]) : sum[t];
    }
    __syncwarp();
  }
  stage();  // warps without a channel (or that stopped early) still meet the others
}

std::mutex g_prep_mu;
size_t g_down_dyn_limit[kMaxDevices] = {};  // dynamic shared memory the down kernel may take

template <typename Rows>
cudaError_t prepare_kernels() {
  static bool done[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  std::lock_guard<std::mutex> lock(g_prep_mu);
  if (dev < kMaxDevices && done[dev]) return cudaSuccess;
  st = allow_max_dynamic_smem(gate_up_decode_kernel<Rows, 1>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(gate_up_decode_kernel<Rows, 4>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(gate_up_decode_kernel<Rows, 8>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(gate_up_decode_kernel<Rows, kDecodeMaxRows>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(down_decode_kernel<Rows, 1>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(down_decode_kernel<Rows, 4>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(down_decode_kernel<Rows, 8>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(down_decode_kernel<Rows, kDecodeMaxRows>);
  if (st == cudaSuccess && dev < kMaxDevices) {
    cudaFuncAttributes a{};
    int optin = 0;
    st = cudaFuncGetAttributes(&a, down_decode_kernel<Rows, kDecodeMaxRows>);
    if (st == cudaSuccess) st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (st == cudaSuccess) {
      g_down_dyn_limit[dev] = static_cast<size_t>(optin) - a.sharedSizeBytes;
      done[dev] = true;
    }
  }
  return st;
}

// The kernel pair compiled for the smallest row bound >= T.
template <typename Rows>
void pick_kernels(int T, const void** gu, const void** dn) {
  if (T <= 1) {
    *gu = reinterpret_cast<const void*>(gate_up_decode_kernel<Rows, 1>);
    *dn = reinterpret_cast<const void*>(down_decode_kernel<Rows, 1>);
  } else if (T <= 4) {
    *gu = reinterpret_cast<const void*>(gate_up_decode_kernel<Rows, 4>);
    *dn = reinterpret_cast<const void*>(down_decode_kernel<Rows, 4>);
  } else if (T <= 8) {
    *gu = reinterpret_cast<const void*>(gate_up_decode_kernel<Rows, 8>);
    *dn = reinterpret_cast<const void*>(down_decode_kernel<Rows, 8>);
  } else {
    *gu = reinterpret_cast<const void*>(gate_up_decode_kernel<Rows, kDecodeMaxRows>);
    *dn = reinterpret_cast<const void*>(down_decode_kernel<Rows, kDecodeMaxRows>);
  }
}

template <typename Rows>
cudaError_t launch_decode_experts_t(const float* x, int T, int H, int F, int S, Rows gate, Rows up, Rows down,
                                    Rows sgate, Rows sup, Rows sdown, const DecodeRouting& routing,
                                    __nv_bfloat16* act, __nv_bfloat16* act_s, const float* resid, float* y,
                                    ErrorWord* err, int sm_count, cudaStream_t stream, cudaEvent_t between,
                                    bool pdl, RowNorm norm) {
  cudaError_t st = prepare_kernels<Rows>();
  if (st != cudaSuccess) return st;
  RouteSrc rs{routing.logits, routing.table, routing.experts, routing.top_k, routing.renormalize, routing.ids_out,
              routing.weights_out};
  const size_t smem = static_cast<size_t>(T) * H * sizeof(float);
  const void* gu = nullptr;
  const void* dn = nullptr;
  pick_kernels<Rows>(T, &gu, &dn);
  {
    void* args[] = {&x, &T, &H, &F, &S, &gate, &up, &sgate, &sup, &rs, &act, &act_s, &err, &norm};
    st = launch_maybe_pdl(gu, dim3(sm_count),
                          dim3(kThreads), smem, stream, args, pdl);
    if (st != cudaSuccess) return st;
  }
  if (between != nullptr) {
    st = cudaEventRecord(between, stream);
    if (st != cudaSuccess) return st;
  }
  rs.ids_out = nullptr;
  rs.w_out = nullptr;
  // Activations staged in shared memory when they fit (T*S + T*k*F bf16), else
  // the routed slots alone (T*k*F) when those fit.
  int dev = 0;
  if ((st = cudaGetDevice(&dev)) != cudaSuccess) return st;
  const size_t need_s = static_cast<size_t>(T) * S * 2, need_r = static_cast<size_t>(T) * routing.top_k * F * 2;
  const size_t limit = dev < kMaxDevices ? g_down_dyn_limit[dev] : 0;
  int stage = need_s + need_r <= limit ? 1 : (need_r <= limit ? 2 : 0);
  const size_t dn_smem = stage == 1 ? need_s + need_r : (stage == 2 ? need_r : 0);
  void* args[] = {&T, &H, &F, &S, &down, &sdown, &rs, &act, &act_s, &resid, &y, &err, &stage};
  return launch_maybe_pdl(dn, dim3(sm_count), dim3(kThreads), dn_smem, stream, args, pdl && between == nullptr);
}

}  // namespace

cudaError_t launch_maybe_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args,
                             bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, func, args);
}

cudaError_t launch_decode_experts_bf16(const float* x, int T, int H, int F, int S, const __nv_bfloat16* gate,
                                       const __nv_bfloat16* up, const __nv_bfloat16* down,
                                       const __nv_bfloat16* sgate, const __nv_bfloat16* sup,
                                       const __nv_bfloat16* sdown, const DecodeRouting& routing, __nv_bfloat16* act,
                                       __nv_bfloat16* act_s, const float* resid, float* y, ErrorWord* err,
                                       int sm_count, cudaStream_t stream, cudaEvent_t between, bool pdl,
                                       RowNorm norm) {
  return launch_decode_experts_t<Bf16Rows>(x, T, H, F, S, Bf16Rows{gate, H}, Bf16Rows{up, H}, Bf16Rows{down, F},
                                           Bf16Rows{sgate, H}, Bf16Rows{sup, H}, Bf16Rows{sdown, S}, routing, act,
                                           act_s, resid, y, err, sm_count, stream, between, pdl, norm);
}

cudaError_t launch_decode_experts_q8(const float* x, int T, int H, int F, int S, Q8Rows gate, Q8Rows up,
                                     Q8Rows down, Q8Rows sgate, Q8Rows sup, Q8Rows sdown,
                                     const DecodeRouting& routing, __nv_bfloat16* act, __nv_bfloat16* act_s,
                                     const float* resid, float* y, ErrorWord* err, int sm_count, cudaStream_t stream,
                                     cudaEvent_t between, bool pdl, RowNorm norm) {
  return launch_decode_experts_t<Q8Rows>(x, T, H, F, S, gate, up, down, sgate, sup, sdown, routing, act, act_s,
                                         resid, y, err, sm_count, stream, between, pdl, norm);
}

cudaError_t prepare_decode_experts(int max_rows, int H) {
  (void)max_rows;
  (void)H;
  cudaError_t st = prepare_kernels<Bf16Rows>();
  if (st == cudaSuccess) st = prepare_kernels<Q8Rows>();
  return st;
}

}  // namespace uocr_b200
