// Decode-path expert kernels (rows <= 16) on the CUDA cores: weight streaming
// over only the experts the batch selected, plus the shared expert.
//
// One block per SM with 16 streaming warps and one routing warp. A streaming
// warp owns one weight row (or the gate+up pair of one row) at a time and
// issues every 128-bit load of it before using any, so an SM keeps ~16 rows
// (about 128 KB) in flight; work is dealt grid-stride so all SMs stream. bf16
// rows are 8 weights per load, int8 rows 16 weights per load with the
// per-output-channel scale applied once to a row's sum. The routing warp
// builds the routing table in shared memory from the router's logits while
// the streaming warps work through the shared expert, which needs none.
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
#include "route.cuh"

namespace uocr_b200 {
namespace {

// 16 warps = 4 per SM sub-partition, which leaves 128 registers a thread.
constexpr int kWorkers = 15;                   // streaming warps per block
constexpr int kThreads = (kWorkers + 1) * 32;  // + the routing warp

// 16-byte loads a lane issues per pass over a row: more when few batch rows
// leave registers free.
template <int MaxT>
constexpr int chunk_count() { return MaxT <= 4 ? 8 : 4; }

// L2 prefetch: how many of its own units ahead a warp keeps on their way, and
// how many bytes of down rows the gate/up kernel brings in for the down
// kernel (more would push the gate/up rows still in use out of L2).
constexpr int kPrefetchUnits = 4;
constexpr int64_t kDownPrefetchBytes = 48ll << 20;

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
                          Rows sup, Rows down, Rows sdown, RouteSrc rsrc, __nv_bfloat16* __restrict__ act,
                          __nv_bfloat16* __restrict__ act_s, ErrorWord* err) {
  using Fm = Fmt<Rows>;
  constexpr int kChunkMax = chunk_count<MaxT>();
  extern __shared__ __align__(16) float xs[];  // [T][H] bf16-rounded inputs
  __shared__ SmemRoute sroute;
  __shared__ uint64_t route_ready;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&route_ready, 1);
    fence_mbar_init();
  }
  // x was written by the grid two launches back, complete before this one started.
  for (int i = threadIdx.x; i < T * H; i += blockDim.x) xs[i] = bf16_round(__ldcg(x + i));
  __syncthreads();
  if (warp == kWorkers) {
    pdl_wait();  // the router's logits
    build_route_warp(rsrc, T, &sroute, lane, true, &route_ready);
    pdl_launch_dependents();
    return;
  }
  const int gw = blockIdx.x * kWorkers + warp, GW = gridDim.x * kWorkers;
  const int nchunks = H * Fm::kElemBytes / 16;

  // One (gate row, up row) pair against `ntok` batch rows.
  auto unit = [&](const uint4* gr, const uint4* ur, float gsc, float usc, int ntok, const int* toks,
                  __nv_bfloat16* out, int64_t out_stride) {
    float gacc[MaxT], uacc[MaxT];
#pragma unroll
    for (int j = 0; j < MaxT; ++j) gacc[j] = uacc[j] = 0.0f;
    for (int pass = 0; pass < nchunks; pass += 32 * kChunkMax) {
      uint4 wg[kChunkMax], wu[kChunkMax];
#pragma unroll
      for (int c = 0; c < kChunkMax; ++c) {
        const int idx = pass + lane + 32 * c;
        if (idx < nchunks) {
          wg[c] = ld_stream(gr + idx);
          wu[c] = ld_stream(ur + idx);
        }
      }
#pragma unroll
      for (int j = 0; j < MaxT; ++j) {
        if (j >= ntok) break;
        const float* xr = xs + static_cast<size_t>(toks == nullptr ? j : toks[j]) * H;
#pragma unroll
        for (int c = 0; c < kChunkMax; ++c) {
          const int idx = pass + lane + 32 * c;
          if (idx < nchunks) {
            gacc[j] += Fm::dot_x(wg[c], xr + idx * Fm::kPerChunk);
            uacc[j] += Fm::dot_x(wu[c], xr + idx * Fm::kPerChunk);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < MaxT; ++j) {
      if (j >= ntok) break;
      const float gv = warp_sum(gacc[j]) * gsc;
      const float uv = warp_sum(uacc[j]) * usc;
      if (lane == 0) out[j * out_stride] = __float2bfloat16_rn(swiglu(gv, uv));
    }
  };

  const uint32_t xrow_bytes = static_cast<uint32_t>(H) * Fm::kElemBytes;
  for (int f = gw; f < S; f += GW)
    unit(Fm::row(sgate, f), Fm::row(sup, f), Fm::scale(sgate, f), Fm::scale(sup, f), T, nullptr, act_s + f, S);
  if (!wait_ready(&route_ready, err, 12)) return;
  pdl_launch_dependents();
  const int U = sroute.count;
  auto routed_row = [&](int q) { return static_cast<int64_t>(sroute.expert[q / F]) * F + q % F; };
  if (lane == 0)
    for (int k = 0; k < kPrefetchUnits; ++k) {
      const int q = gw + k * GW;
      if (q >= U * F) break;
      prefetch_l2(Fm::row(gate, routed_row(q)), xrow_bytes);
      prefetch_l2(Fm::row(up, routed_row(q)), xrow_bytes);
    }
  for (int q = gw; q < U * F; q += GW) {
    const int qn = q + kPrefetchUnits * GW;
    if (lane == 0 && qn < U * F) {
      prefetch_l2(Fm::row(gate, routed_row(qn)), xrow_bytes);
      prefetch_l2(Fm::row(up, routed_row(qn)), xrow_bytes);
    }
    const int u = q / F, f = q % F;
    const int64_t row = static_cast<int64_t>(sroute.expert[u]) * F + f;
    const int base = sroute.base[u];
    unit(Fm::row(gate, row), Fm::row(up, row), Fm::scale(gate, row), Fm::scale(up, row), sroute.ntok[u],
         sroute.slot_tok + base, act + static_cast<int64_t>(base) * F + f, F);
  }
  // The down kernel's warp gw takes output channels gw, gw + GW, ...: bring
  // their shared and expert rows into L2 now, while the other warps finish.
  if (lane == 0) {
    const int64_t per_expert = static_cast<int64_t>(H) * F * Fm::kElemBytes;
    const int64_t shared_bytes = static_cast<int64_t>(H) * S * Fm::kElemBytes;
    int ucap = static_cast<int>((kDownPrefetchBytes - shared_bytes) / (per_expert > 0 ? per_expert : 1));
    ucap = ucap < 0 ? 0 : (ucap > U ? U : ucap);
    for (int ch = gw; ch < H; ch += GW) {
      if (S > 0) prefetch_l2(Fm::row(sdown, ch), static_cast<uint32_t>(S) * Fm::kElemBytes);
      for (int u = 0; u < ucap; ++u)
        prefetch_l2(Fm::row(down, static_cast<int64_t>(sroute.expert[u]) * H + ch),
                    static_cast<uint32_t>(F) * Fm::kElemBytes);
    }
  }
}

// ---------------------------------------------------------------------------
// down + combine: one streaming warp per output channel c (grid-stride): the
// shared down row against every batch row's shared activation, then the
// selected experts' down rows two at a time (the second's loads in flight
// while the first's dot products run), each finished in registers and added
// to its rows' sums in ascending expert order.
template <typename Rows, int MaxT>
__global__ void __launch_bounds__(kThreads, 1)
    down_decode_kernel(int T, int H, int F, int S, Rows down, Rows sdown, RouteSrc rsrc,
                       const __nv_bfloat16* __restrict__ act, const __nv_bfloat16* __restrict__ act_s,
                       const float* resid, float* y, ErrorWord* err, DecodeNext next) {
  using Fm = Fmt<Rows>;
  constexpr int kChunkMax = chunk_count<MaxT>();
  constexpr int kHalf = kChunkMax / 2;
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
  const int nch_s = S * Fm::kElemBytes / 16, nch_f = F * Fm::kElemBytes / 16;
  float* sum = row_sum[warp];
  bool waited = false, have_route = false;
  for (int c = gw; c < H; c += GW) {
    if (lane < kDecodeMaxRows) sum[lane] = 0.0f;
    __syncwarp();
    if (S > 0) {
      const uint4* wr = Fm::row(sdown, c);
      float acc[MaxT];
#pragma unroll
      for (int t = 0; t < MaxT; ++t) acc[t] = 0.0f;
      for (int pass = 0; pass < nch_s; pass += 32 * kChunkMax) {
        uint4 w[kChunkMax];
#pragma unroll
        for (int q = 0; q < kChunkMax; ++q) {
          const int idx = pass + lane + 32 * q;
          if (idx < nch_s) w[q] = ld_stream(wr + idx);
        }
        if (!waited) {
          pdl_wait();  // the activations come from the gate/up grid
          waited = true;
        }
#pragma unroll
        for (int t = 0; t < MaxT; ++t) {
          if (t >= T) break;
          const __nv_bfloat16* ar = act_s + static_cast<int64_t>(t) * S;
#pragma unroll
          for (int q = 0; q < kChunkMax; ++q) {
            const int idx = pass + lane + 32 * q;
            if (idx < nch_s) acc[t] += Fm::dot_act(w[q], ar + idx * Fm::kPerChunk);
          }
        }
      }
      const float sc = Fm::scale(sdown, c);
#pragma unroll
      for (int t = 0; t < MaxT; ++t) {
        if (t >= T) break;
        const float v = warp_sum(acc[t]) * sc;
        if (lane == 0) sum[t] = v;
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    if (!have_route) {
      if (!wait_ready(&route_ready, err, 24)) return;
      have_route = true;
    }
    const int U = sroute.count;
    for (int u0 = 0; u0 < U; u0 += 2) {
      const bool two = u0 + 1 < U;
      const int64_t r0 = static_cast<int64_t>(sroute.expert[u0]) * H + c;
      const int64_t r1 = two ? static_cast<int64_t>(sroute.expert[u0 + 1]) * H + c : r0;
      const int b0 = sroute.base[u0], n0 = sroute.ntok[u0];
      const int b1 = two ? sroute.base[u0 + 1] : 0, n1 = two ? sroute.ntok[u0 + 1] : 0;
      const uint4* p0 = Fm::row(down, r0);
      const uint4* p1 = Fm::row(down, r1);
      float a0[MaxT], a1[MaxT];
#pragma unroll
      for (int j = 0; j < MaxT; ++j) a0[j] = a1[j] = 0.0f;
      for (int pass = 0; pass < nch_f; pass += 32 * kHalf) {
        uint4 w0[kHalf], w1[kHalf];
#pragma unroll
        for (int q = 0; q < kHalf; ++q) {
          const int idx = pass + lane + 32 * q;
          if (idx < nch_f) {
            w0[q] = ld_stream(p0 + idx);
            if (two) w1[q] = ld_stream(p1 + idx);
          }
        }
#pragma unroll
        for (int j = 0; j < MaxT; ++j) {
          if (j >= n0) break;
          const __nv_bfloat16* ar = act + static_cast<int64_t>(b0 + j) * F;
#pragma unroll
          for (int q = 0; q < kHalf; ++q) {
            const int idx = pass + lane + 32 * q;
            if (idx < nch_f) a0[j] += Fm::dot_act(w0[q], ar + idx * Fm::kPerChunk);
          }
        }
#pragma unroll
        for (int j = 0; j < MaxT; ++j) {
          if (j >= n1) break;
          const __nv_bfloat16* ar = act + static_cast<int64_t>(b1 + j) * F;
#pragma unroll
          for (int q = 0; q < kHalf; ++q) {
            const int idx = pass + lane + 32 * q;
            if (idx < nch_f) a1[j] += Fm::dot_act(w1[q], ar + idx * Fm::kPerChunk);
          }
        }
      }
      const float s0 = Fm::scale(down, r0), s1 = Fm::scale(down, r1);
#pragma unroll
      for (int j = 0; j < MaxT; ++j) {
        if (j >= n0) break;
        const float v = warp_sum(a0[j]) * s0;
        if (lane == 0) {
          const int t = sroute.slot_tok[b0 + j];
          sum[t] = __fadd_rn(sum[t], __fmul_rn(sroute.slot_w[b0 + j], v));
        }
      }
#pragma unroll
      for (int j = 0; j < MaxT; ++j) {
        if (j >= n1) break;
        const float v = warp_sum(a1[j]) * s1;
        if (lane == 0) {
          const int t = sroute.slot_tok[b1 + j];
          sum[t] = __fadd_rn(sum[t], __fmul_rn(sroute.slot_w[b1 + j], v));
        }
      }
    }
    __syncwarp();
    for (int t = lane; t < T; t += 32) {
      const int64_t o = static_cast<int64_t>(t) * H + c;
      y[o] = resid != nullptr ? __fadd_rn(resid[o], sum[t]) : sum[t];
    }
    __syncwarp();
  }
  // The next layer of a stack: its router rows and shared gate/up rows start
  // towards L2 now, ahead of its router and gate/up kernels.
  if (lane == 0 && next.router != nullptr) {
    for (int e = gw; e < rsrc.E; e += GW)
      prefetch_l2(next.router + static_cast<int64_t>(e) * H, static_cast<uint32_t>(H) * 4);
    for (int f = gw; f < S; f += GW) {
      prefetch_l2(static_cast<const char*>(next.sgate) + f * next.srow_bytes, static_cast<uint32_t>(next.srow_bytes));
      prefetch_l2(static_cast<const char*>(next.sup) + f * next.srow_bytes, static_cast<uint32_t>(next.srow_bytes));
    }
  }
}

std::mutex g_prep_mu;

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
  if (st == cudaSuccess && dev < kMaxDevices) done[dev] = true;
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
                                    bool pdl, const DecodeNext* next) {
  cudaError_t st = prepare_kernels<Rows>();
  if (st != cudaSuccess) return st;
  RouteSrc rs{routing.logits, routing.table, routing.experts, routing.top_k, routing.renormalize, routing.ids_out,
              routing.weights_out};
  const size_t smem = static_cast<size_t>(T) * H * sizeof(float);
  const void* gu = nullptr;
  const void* dn = nullptr;
  pick_kernels<Rows>(T, &gu, &dn);
  {
    void* args[] = {&x, &T, &H, &F, &S, &gate, &up, &sgate, &sup, &down, &sdown, &rs, &act, &act_s, &err};
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
  DecodeNext nx = next != nullptr ? *next : DecodeNext{nullptr, nullptr, nullptr, 0};
  void* args[] = {&T, &H, &F, &S, &down, &sdown, &rs, &act, &act_s, &resid, &y, &err, &nx};
  return launch_maybe_pdl(dn, dim3(sm_count), dim3(kThreads), 0,
                          stream, args, pdl && between == nullptr);
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
                                       const DecodeNext* next) {
  return launch_decode_experts_t<Bf16Rows>(x, T, H, F, S, Bf16Rows{gate, H}, Bf16Rows{up, H}, Bf16Rows{down, F},
                                           Bf16Rows{sgate, H}, Bf16Rows{sup, H}, Bf16Rows{sdown, S}, routing, act,
                                           act_s, resid, y, err, sm_count, stream, between, pdl, next);
}

cudaError_t launch_decode_experts_q8(const float* x, int T, int H, int F, int S, Q8Rows gate, Q8Rows up,
                                     Q8Rows down, Q8Rows sgate, Q8Rows sup, Q8Rows sdown,
                                     const DecodeRouting& routing, __nv_bfloat16* act, __nv_bfloat16* act_s,
                                     const float* resid, float* y, ErrorWord* err, int sm_count, cudaStream_t stream,
                                     cudaEvent_t between, bool pdl, const DecodeNext* next) {
  return launch_decode_experts_t<Q8Rows>(x, T, H, F, S, gate, up, down, sgate, sup, sdown, routing, act, act_s,
                                         resid, y, err, sm_count, stream, between, pdl, next);
}

cudaError_t prepare_decode_experts(int max_rows, int H) {
  (void)max_rows;
  (void)H;
  cudaError_t st = prepare_kernels<Bf16Rows>();
  if (st == cudaSuccess) st = prepare_kernels<Q8Rows>();
  return st;
}

}  // namespace uocr_b200
