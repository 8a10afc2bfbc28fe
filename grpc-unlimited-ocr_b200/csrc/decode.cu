// Decode-path expert kernels: weight-streaming GEMVs over only the experts
// the batch selected, plus the shared expert.
//
// Work is cut into weight rows, and one warp streams one row (or the gate+up
// pair of one row) with 128-bit coalesced loads, every chunk of the row in
// flight at once; bf16 rows are 8 weights per load, int8 rows 16 weights per
// load with the per-output-channel scale applied once to the row's sum. The
// reference equivalents are expert_gate_up_kernel / expert_down_kernel
// (src/backend/cuda/gemv_ops.cu:145-169) and the shared expert's gemv_kernel
// calls (:133-141, src/model/cuda/cuda_decoder.cpp:119-125,155-156).
//
//   gate/up:  act[slot, f] = bf16(silu(gate[e,f] . x^) * (up[e,f] . x^)), x^ = bf16(x)
//   down:     y[t, c] = shared[t, c] + sum over the row's experts in id order of w * (down[e,c] . act)
//
// The combine and the shared add happen in the down kernel, in the order the
// reference adds them (src/model/feed_forward.cpp:65-76), so nothing is
// accumulated with atomics and the result is the same on every run.
#include <map>
#include <mutex>
#include <utility>

#include "moe_kernels.h"

namespace uocr_b200 {
namespace {

constexpr int kChunkMax = 8;  // 128-bit loads per lane per pass

// Row view helpers: load up to kChunkMax 16-byte chunks of a row (lane-strided).
template <typename Rows>
struct RowTraits;

template <>
struct RowTraits<Bf16Rows> {
  static constexpr int kPerChunk = 8;  // weights per 16-byte load
  __device__ static const uint4* row(const Bf16Rows& r, int64_t i) {
    return reinterpret_cast<const uint4*>(r.w + i * r.cols);
  }
  __device__ static float scale(const Bf16Rows&, int64_t) { return 1.0f; }
  // chunk of weights dotted with 16 fp32 inputs (only 8 used for bf16)
  __device__ static float dot(const uint4& w, const float* xs) {
    const float4 x0 = reinterpret_cast<const float4*>(xs)[0];
    const float4 x1 = reinterpret_cast<const float4*>(xs)[1];
    return dot8_bf16(w, x0, x1);
  }
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    return dot8_bf16_bf16(w, *reinterpret_cast<const uint4*>(act));
  }
};

template <>
struct RowTraits<Q8Rows> {
  static constexpr int kPerChunk = 16;
  __device__ static const uint4* row(const Q8Rows& r, int64_t i) {
    return reinterpret_cast<const uint4*>(r.q + i * r.cols);
  }
  __device__ static float scale(const Q8Rows& r, int64_t i) { return r.scale[i]; }
  __device__ static float dot(const uint4& w, const float* xs) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a, b, c, d;
      i8x4_to_f32(words[q], a, b, c, d);
      const float4 xv = reinterpret_cast<const float4*>(xs)[q];
      s = fmaf(a, xv.x, s);
      s = fmaf(b, xv.y, s);
      s = fmaf(c, xv.z, s);
      s = fmaf(d, xv.w, s);
    }
    return s;
  }
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    const uint4 a0 = reinterpret_cast<const uint4*>(act)[0];
    const uint4 a1 = reinterpret_cast<const uint4*>(act)[1];
    const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&a0);
    const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&a1);
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a, b, c, d;
      i8x4_to_f32(words[q], a, b, c, d);
      const __nv_bfloat162* p = q < 2 ? p0 : p1;
      const float2 f0 = __bfloat1622float2(p[(q & 1) * 2]);
      const float2 f1 = __bfloat1622float2(p[(q & 1) * 2 + 1]);
      s = fmaf(a, f0.x, s);
      s = fmaf(b, f0.y, s);
      s = fmaf(c, f1.x, s);
      s = fmaf(d, f1.y, s);
    }
    return s;
  }
};

// Gate/up for the shared expert and every (selected expert, ffn row) pair.
// Units: [0, S) are shared rows (all T batch rows), then U*F routed rows in
// ascending expert order. Warps take units grid-stride.
template <typename Rows>
__global__ void __launch_bounds__(256) gate_up_decode_kernel(const float* __restrict__ x, int T, int H, int F, int S,
                                                             Rows gate, Rows up, Rows sgate, Rows sup,
                                                             const DecodeRoute* __restrict__ route,
                                                             __nv_bfloat16* __restrict__ act,
                                                             __nv_bfloat16* __restrict__ act_s, ErrorWord* err) {
  using Tr = RowTraits<Rows>;
  extern __shared__ __align__(16) float xs[];  // [T][H] bf16-rounded inputs
  for (int i = threadIdx.x; i < T * H; i += blockDim.x) xs[i] = bf16_round(x[i]);
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * nwarps + (threadIdx.x >> 5);
  const int64_t total_warps = static_cast<int64_t>(gridDim.x) * nwarps;
  const int U = route->active_count;
  const int64_t units = static_cast<int64_t>(S) + static_cast<int64_t>(U) * F;
  const int nchunks = H / Tr::kPerChunk;

  for (int64_t unit = warp_global; unit < units; unit += total_warps) {
    const bool is_shared = unit < S;
    const Rows g = is_shared ? sgate : gate;
    const Rows u = is_shared ? sup : up;
    int64_t row;
    int ntok;
    int u_idx = -1;
    int f;
    if (is_shared) {
      row = unit;
      ntok = T;
      f = static_cast<int>(unit);
    } else {
      const int64_t r = unit - S;
      u_idx = static_cast<int>(r / F);
      f = static_cast<int>(r % F);
      const int e = route->active_expert[u_idx];
      row = static_cast<int64_t>(e) * F + f;
      ntok = route->tok_count[u_idx];
    }
    const uint4* gr = Tr::row(g, row);
    const uint4* ur = Tr::row(u, row);
    const float gscale = Tr::scale(g, row), uscale = Tr::scale(u, row);
    float gacc[kDecodeMaxRows], uacc[kDecodeMaxRows];
#pragma unroll
    for (int s = 0; s < kDecodeMaxRows; ++s) gacc[s] = uacc[s] = 0.0f;
    for (int base = 0; base < nchunks; base += 32 * kChunkMax) {
      uint4 wg[kChunkMax], wu[kChunkMax];
#pragma unroll
      for (int c = 0; c < kChunkMax; ++c) {
        const int idx = base + lane + 32 * c;
        if (idx < nchunks) {
          wg[c] = __ldg(gr + idx);
          wu[c] = __ldg(ur + idx);
        }
      }
#pragma unroll
      for (int s = 0; s < kDecodeMaxRows; ++s) {
        if (s >= ntok) break;
        const int t = u_idx < 0 ? s : route->tok_index[u_idx][s];
        const float* xr = xs + t * H;
        float pg = 0.0f, pu = 0.0f;
#pragma unroll
        for (int c = 0; c < kChunkMax; ++c) {
          const int idx = base + lane + 32 * c;
          if (idx < nchunks) {
            pg += Tr::dot(wg[c], xr + idx * Tr::kPerChunk);
            pu += Tr::dot(wu[c], xr + idx * Tr::kPerChunk);
          }
        }
        gacc[s] += pg;
        uacc[s] += pu;
      }
    }
#pragma unroll
    for (int s = 0; s < kDecodeMaxRows; ++s) {
      if (s >= ntok) break;
      const float gv = warp_sum(gacc[s]) * gscale;
      const float uv = warp_sum(uacc[s]) * uscale;
      if (lane == 0) {
        const __nv_bfloat16 a = __float2bfloat16_rn(swiglu(gv, uv));
        if (u_idx < 0) {
          act_s[static_cast<int64_t>(s) * S + f] = a;
        } else {
          act[static_cast<int64_t>(route->slot_base[u_idx] + s) * F + f] = a;
        }
      }
    }
  }
}

// Down projection, combine and shared add. One warp per output channel c:
// the shared down row against every batch row's shared activation, then each
// selected expert's down row against the activations of the rows routed to
// it, added per row in ascending expert order.
template <typename Rows>
__global__ void __launch_bounds__(128) down_decode_kernel(int T, int H, int F, int S, Rows down, Rows sdown,
                                                          const DecodeRoute* __restrict__ route,
                                                          const __nv_bfloat16* __restrict__ act,
                                                          const __nv_bfloat16* __restrict__ act_s,
                                                          const float* resid, float* y) {
  using Tr = RowTraits<Rows>;
  __shared__ float routed[4][kDecodeMaxRows];
  __shared__ float shared_out[4][kDecodeMaxRows];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 4 + warp;
  if (c >= H) return;
  if (lane < kDecodeMaxRows) {
    routed[warp][lane] = 0.0f;
    shared_out[warp][lane] = 0.0f;
  }
  __syncwarp();

  if (S > 0) {
    const uint4* wr = Tr::row(sdown, c);
    const float sc = Tr::scale(sdown, c);
    const int nchunks = S / Tr::kPerChunk;
    float acc[kDecodeMaxRows];
#pragma unroll
    for (int t = 0; t < kDecodeMaxRows; ++t) acc[t] = 0.0f;
    for (int base = 0; base < nchunks; base += 32 * kChunkMax) {
      uint4 w[kChunkMax];
#pragma unroll
      for (int q = 0; q < kChunkMax; ++q) {
        const int idx = base + lane + 32 * q;
        if (idx < nchunks) w[q] = __ldg(wr + idx);
      }
#pragma unroll
      for (int t = 0; t < kDecodeMaxRows; ++t) {
        if (t >= T) break;
        const __nv_bfloat16* ar = act_s + static_cast<int64_t>(t) * S;
        float p = 0.0f;
#pragma unroll
        for (int q = 0; q < kChunkMax; ++q) {
          const int idx = base + lane + 32 * q;
          if (idx < nchunks) p += Tr::dot_act(w[q], ar + idx * Tr::kPerChunk);
        }
        acc[t] += p;
      }
    }
#pragma unroll
    for (int t = 0; t < kDecodeMaxRows; ++t) {
      if (t >= T) break;
      const float v = warp_sum(acc[t]) * sc;
      if (lane == 0) shared_out[warp][t] = v;
    }
  }

  const int U = route->active_count;
  const int nchunks = F / Tr::kPerChunk;
  for (int ui = 0; ui < U; ++ui) {
    const int e = route->active_expert[ui];
    const int n = route->tok_count[ui];
    const int64_t row = static_cast<int64_t>(e) * H + c;
    const uint4* wr = Tr::row(down, row);
    const float sc = Tr::scale(down, row);
    float acc[kDecodeMaxRows];
#pragma unroll
    for (int s = 0; s < kDecodeMaxRows; ++s) acc[s] = 0.0f;
    for (int base = 0; base < nchunks; base += 32 * kChunkMax) {
      uint4 w[kChunkMax];
#pragma unroll
      for (int q = 0; q < kChunkMax; ++q) {
        const int idx = base + lane + 32 * q;
        if (idx < nchunks) w[q] = __ldg(wr + idx);
      }
#pragma unroll
      for (int s = 0; s < kDecodeMaxRows; ++s) {
        if (s >= n) break;
        const __nv_bfloat16* ar = act + static_cast<int64_t>(route->slot_base[ui] + s) * F;
        float p = 0.0f;
#pragma unroll
        for (int q = 0; q < kChunkMax; ++q) {
          const int idx = base + lane + 32 * q;
          if (idx < nchunks) p += Tr::dot_act(w[q], ar + idx * Tr::kPerChunk);
        }
        acc[s] += p;
      }
    }
#pragma unroll
    for (int s = 0; s < kDecodeMaxRows; ++s) {
      if (s >= n) break;
      const float v = warp_sum(acc[s]) * sc;
      if (lane == 0) {
        const int t = route->tok_index[ui][s];
        routed[warp][t] = __fadd_rn(routed[warp][t], __fmul_rn(route->tok_weight[ui][s], v));
      }
    }
  }
  __syncwarp();
  if (lane < T) {
    const int64_t o = static_cast<int64_t>(lane) * H + c;
    float out = __fadd_rn(shared_out[warp][lane], routed[warp][lane]);
    if (resid != nullptr) out = __fadd_rn(resid[o], out);
    y[o] = out;
  }
}

// Resident gate/up blocks per SM for a shared-memory size, computed once per
// (device, size) — never inside a stream capture once the plan prepared it.
template <typename Rows>
int gate_up_blocks_per_sm(size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<int, size_t>, int> cache;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(mu);
  const auto it = cache.find({dev, smem});
  if (it != cache.end()) return it->second;
  if (!attr_set[dev]) {
    if (allow_max_dynamic_smem(gate_up_decode_kernel<Rows>) != cudaSuccess) return -1;
    attr_set[dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gate_up_decode_kernel<Rows>, 256, smem) != cudaSuccess)
    return -1;
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  cache[{dev, smem}] = per_sm;
  return per_sm;
}

template <typename Rows>
cudaError_t launch_decode_experts_t(const float* x, int T, int H, int F, int S, Rows gate, Rows up, Rows down,
                                    Rows sgate, Rows sup, Rows sdown, const DecodeRoute* route,
                                    __nv_bfloat16* act, __nv_bfloat16* act_s, const float* resid, float* y,
                                    ErrorWord* err, int sm_count, cudaStream_t stream, cudaEvent_t between) {
  const size_t smem = static_cast<size_t>(T) * H * sizeof(float);
  const int per_sm = gate_up_blocks_per_sm<Rows>(smem);
  if (per_sm < 0) return cudaErrorInvalidConfiguration;
  cudaError_t st;
  gate_up_decode_kernel<Rows><<<sm_count * per_sm, 256, smem, stream>>>(x, T, H, F, S, gate, up, sgate, sup, route,
                                                                       act, act_s, err);
  st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  if (between != nullptr) {
    st = cudaEventRecord(between, stream);
    if (st != cudaSuccess) return st;
  }
  down_decode_kernel<Rows><<<(H + 3) / 4, 128, 0, stream>>>(T, H, F, S, down, sdown, route, act, act_s, resid, y);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_experts_bf16(const float* x, int T, int H, int F, int S, const __nv_bfloat16* gate,
                                       const __nv_bfloat16* up, const __nv_bfloat16* down,
                                       const __nv_bfloat16* sgate, const __nv_bfloat16* sup,
                                       const __nv_bfloat16* sdown, const DecodeRoute* route, __nv_bfloat16* act,
                                       __nv_bfloat16* act_s, const float* resid, float* y, ErrorWord* err,
                                       int sm_count, cudaStream_t stream, cudaEvent_t between) {
  return launch_decode_experts_t<Bf16Rows>(x, T, H, F, S, Bf16Rows{gate, H}, Bf16Rows{up, H}, Bf16Rows{down, F},
                                           Bf16Rows{sgate, H}, Bf16Rows{sup, H}, Bf16Rows{sdown, S}, route, act,
                                           act_s, resid, y, err, sm_count, stream, between);
}

cudaError_t launch_decode_experts_q8(const float* x, int T, int H, int F, int S, Q8Rows gate, Q8Rows up,
                                     Q8Rows down, Q8Rows sgate, Q8Rows sup, Q8Rows sdown, const DecodeRoute* route,
                                     __nv_bfloat16* act, __nv_bfloat16* act_s, const float* resid, float* y,
                                     ErrorWord* err, int sm_count, cudaStream_t stream, cudaEvent_t between) {
  return launch_decode_experts_t<Q8Rows>(x, T, H, F, S, gate, up, down, sgate, sup, sdown, route, act, act_s, resid,
                                         y, err, sm_count, stream, between);
}

cudaError_t prepare_decode_experts(int max_rows, int H) {
  for (int T = 1; T <= max_rows; ++T) {
    const size_t smem = static_cast<size_t>(T) * H * sizeof(float);
    if (gate_up_blocks_per_sm<Bf16Rows>(smem) < 0 || gate_up_blocks_per_sm<Q8Rows>(smem) < 0)
      return cudaErrorInvalidConfiguration;
  }
  return cudaSuccess;
}

}  // namespace uocr_b200
