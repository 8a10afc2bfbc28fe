// Decode-path expert kernels (rows <= 16): weight streaming over only the
// experts the batch selected, plus the shared expert.
//
// Both kernels run one persistent block per SM: a producer warp streams
// weight rows from HBM into a shared-memory ring with bulk async copies (TMA,
// cp.async.bulk) completing on mbarriers, and eight consumer warps do the
// dot products from shared memory. Rows are split over blocks by count, so
// every SM streams the same number of bytes. bf16 rows are read as 8
// weights per 16 bytes, int8 rows as 16 with the per-output-channel scale
// applied once to a row's sum. Reference equivalents: expert_gate_up_kernel /
// expert_down_kernel (src/backend/cuda/gemv_ops.cu:145-169) and the shared
// expert's gemv_kernel calls (:133-141, src/model/cuda/cuda_decoder.cpp:
// 119-125, 155-156).
//
//   gate/up: act[slot, f] = bf16(silu(gate[e,f] . x^) * (up[e,f] . x^)), x^ = bf16(x)
//   down:    y[t, c] = shared[t, c] + sum over the row's experts, in id order, of w * (down[e,c] . act)
//
// Each block builds the routing table itself from the router's logits
// (route.cuh), so the router kernel is a plain GEMV. The combine and the
// shared add happen in the down kernel in the order the reference adds them
// (src/model/feed_forward.cpp:65-76): no atomics, the same bits on every run.
//
// Launch order per layer is router -> gate/up -> down, each launched with
// programmatic dependent launch: gate/up streams the shared expert (which
// needs only x) before it waits for the router; down streams its weights
// before it waits for the activations.
#include <mutex>

#include "moe_kernels.h"
#include "ptx.cuh"
#include "route.cuh"

namespace uocr_b200 {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kMaxStages = 4;
constexpr int kChunkMax = 8;               // 16-byte chunks per lane per pass
constexpr int kMaxChan = 64;               // output channels one down block owns
constexpr int kBarAll = 2;                 // named barrier over all kThreads
constexpr int kBarConsumers = 1;           // named barrier over the consumer warps

template <typename Rows>
struct Fmt;

template <>
struct Fmt<Bf16Rows> {
  static constexpr int kElemBytes = 2;
  static constexpr int kPerChunk = 8;  // weights per 16 bytes
  __device__ static const char* row(const Bf16Rows& r, int64_t i) {
    return reinterpret_cast<const char*>(r.w + i * r.cols);
  }
  __device__ static float scale(const Bf16Rows&, int64_t) { return 1.0f; }
  // 16 bytes of weights against fp32 inputs (8 of them for bf16)
  __device__ static float dot_x(const uint4& w, const float* x) {
    const float4 x0 = reinterpret_cast<const float4*>(x)[0];
    const float4 x1 = reinterpret_cast<const float4*>(x)[1];
    return dot8_bf16(w, x0, x1);
  }
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    return dot8_bf16_bf16(w, __ldg(reinterpret_cast<const uint4*>(act)));
  }
};

template <>
struct Fmt<Q8Rows> {
  static constexpr int kElemBytes = 1;
  static constexpr int kPerChunk = 16;
  __device__ static const char* row(const Q8Rows& r, int64_t i) {
    return reinterpret_cast<const char*>(r.q + i * r.cols);
  }
  __device__ static float scale(const Q8Rows& r, int64_t i) { return __ldg(r.scale + i); }
  __device__ static float dot_x(const uint4& w, const float* x) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a, b, c, d;
      i8x4_to_f32(words[q], a, b, c, d);
      const float4 xv = reinterpret_cast<const float4*>(x)[q];
      s = fmaf(a, xv.x, s);
      s = fmaf(b, xv.y, s);
      s = fmaf(c, xv.z, s);
      s = fmaf(d, xv.w, s);
    }
    return s;
  }
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(act));
    const uint4 a1 = __ldg(reinterpret_cast<const uint4*>(act) + 1);
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

// Shared state of one block's copy pipeline. route_ready completes once the
// block's routing table is in shared memory.
struct Pipe {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t route_ready;
  int abort;
};

__device__ __forceinline__ int split_begin(int64_t n, int parts, int part) {
  return static_cast<int>(n * part / parts);
}

__device__ __forceinline__ void init_pipe(Pipe& pipe, int stages) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&pipe.full[s], 1);
    mbar_init(&pipe.empty[s], kConsumerWarps);
  }
  mbar_init(&pipe.route_ready, 1);
  pipe.abort = 0;
  fence_mbar_init();
}

// Routing source: the router's logits (plan path) or a prepared table (the
// op-level mirrors of expert_ffn_one).
struct RouteSrc {
  const float* logits;
  const DecodeRoute* table;
  int E, K, renorm;
  int* ids_out;  // block 0 writes the rank-order ids/weights here when not null
  float* w_out;
};

__device__ __forceinline__ void build_route(const RouteSrc& src, int T, SmemRoute* r, int tid, int nthreads,
                                            int bar) {
  if (src.logits != nullptr) {
    const bool first = blockIdx.x == 0;
    route_from_logits(src.logits, T, src.E, src.K, src.renorm, r, tid, nthreads, bar, first ? src.ids_out : nullptr,
                      first ? src.w_out : nullptr);
  } else {
    route_from_table(src.table, T, r, tid, nthreads, bar);
  }
}

// Small batches: the producer warp builds the routing table alone while the
// consumers work through the shared expert; larger batches build it with
// every warp of the block.
__device__ __forceinline__ bool producer_routes(int T) { return T <= 2; }

// Consumers wait for the producer warp's table (bounded).
__device__ __forceinline__ bool wait_route(Pipe& pipe, ErrorWord* err, int site) {
  if (mbar_wait(&pipe.route_ready, 0)) return true;
  raise_error(err, kDevWaitTimeout, site, 0, 0);
  pipe.abort = 1;
  return false;
}

// ---------------------------------------------------------------------------
// gate/up. Block b owns shared rows [S*b/G, S*(b+1)/G) and routed rows
// [UF*b/G, UF*(b+1)/G) of the U*F (expert, ffn row) pairs, in ascending
// expert order. A stage holds up to `rps` consecutive (gate row, up row)
// pairs, copied as one bulk copy per matrix and per expert run; consumer warp
// w computes pair w of each stage.
template <typename Rows>
__global__ void __launch_bounds__(kThreads, 1)
    gate_up_decode_kernel(const float* __restrict__ x, int T, int H, int F, int S, Rows gate, Rows up, Rows sgate,
                          Rows sup, RouteSrc rsrc, __nv_bfloat16* __restrict__ act,
                          __nv_bfloat16* __restrict__ act_s, ErrorWord* err, int stages, int rps) {
  using Fm = Fmt<Rows>;
  extern __shared__ __align__(128) unsigned char dyn[];
  __shared__ Pipe pipe;
  __shared__ SmemRoute sroute;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int row_bytes = H * Fm::kElemBytes;
  const int stage_bytes = 2 * rps * row_bytes;
  const int nchunks = row_bytes / 16;
  float* xs = reinterpret_cast<float*>(dyn);
  unsigned char* ring = dyn + ((static_cast<size_t>(T) * H * 4 + 127) & ~static_cast<size_t>(127));
  const int G = gridDim.x, b = blockIdx.x;
  const int s0 = split_begin(S, G, b), s1 = split_begin(S, G, b + 1);
  const int sh_stages = (s1 - s0 + rps - 1) / rps;
  const bool solo_route = producer_routes(T);

  if (tid == 0) init_pipe(pipe, stages);
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---- producer warp: lane 0 issues the copies ----
    int k = 0;
    bool ok = true;
    // Stage of n consecutive row pairs; run(i0) gives the expert run starting
    // at item i0 (its first gate row, up row and length).
    auto issue = [&](int n, auto&& run) {
      if (lane == 0 && ok) {
        const int s = k % stages;
        if (!mbar_wait(&pipe.empty[s], ((k / stages) & 1) ^ 1)) {
          raise_error(err, kDevWaitTimeout, 10, k, 0);
          pipe.abort = 1;
          ok = false;
        } else {
          mbar_arrive_expect_tx(&pipe.full[s], static_cast<uint32_t>(2 * n * row_bytes));
          unsigned char* dst = ring + static_cast<size_t>(s) * stage_bytes;
          for (int i0 = 0; i0 < n;) {
            const char* g;
            const char* u;
            int len;
            run(i0, n - i0, g, u, len);
            const uint32_t bytes = static_cast<uint32_t>(len * row_bytes);
            bulk_g2s(dst + static_cast<size_t>(i0) * row_bytes, g, bytes, &pipe.full[s]);
            bulk_g2s(dst + static_cast<size_t>(rps + i0) * row_bytes, u, bytes, &pipe.full[s]);
            i0 += len;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++k;
    };
    for (int st = 0; st < sh_stages; ++st) {
      const int first = s0 + st * rps;
      issue(min(rps, s1 - first), [&](int i0, int left, const char*& g, const char*& u, int& len) {
        g = Fm::row(sgate, first + i0);
        u = Fm::row(sup, first + i0);
        len = left;
      });
    }
    pdl_wait();  // the router's logits are complete from here on
    if (solo_route) {
      build_route(rsrc, T, &sroute, lane, 32, 0);
      if (lane == 0) mbar_arrive(&pipe.route_ready);
    } else {
      build_route(rsrc, T, &sroute, tid, kThreads, kBarAll);
    }
    pdl_launch_dependents();
    const int64_t UF = static_cast<int64_t>(sroute.count) * F;
    const int q0 = split_begin(UF, G, b), q1 = split_begin(UF, G, b + 1);
    for (int first = q0; first < q1; first += rps) {
      issue(min(rps, q1 - first), [&](int i0, int left, const char*& g, const char*& u, int& len) {
        const int q = first + i0;
        const int f = q % F;
        const int64_t row = static_cast<int64_t>(sroute.expert[q / F]) * F + f;
        g = Fm::row(gate, row);
        u = Fm::row(up, row);
        len = min(left, F - f);  // rows of one expert are contiguous
      });
    }
    // Before leaving, every copy this block issued must have landed.
    if (lane == 0)
      for (int j = max(0, k - stages); j < k; ++j)
        if (!mbar_wait(&pipe.full[j % stages], (j / stages) & 1)) raise_error(err, kDevWaitTimeout, 11, j, 0);
    return;
  }

  // ---- consumers ----
  for (int i = tid; i < T * H; i += kConsumers) xs[i] = bf16_round(__ldcg(x + i));
  named_bar_sync(kBarConsumers, kConsumers);
  // One row and one pass: each lane keeps its inputs in registers.
  const bool x_in_regs = T == 1 && nchunks <= 32 * kChunkMax;
  float xr[kChunkMax][Fm::kPerChunk];
  if (x_in_regs) {
#pragma unroll
    for (int c = 0; c < kChunkMax; ++c) {
      const int idx = lane + 32 * c;
#pragma unroll
      for (int q = 0; q < Fm::kPerChunk; ++q) xr[c][q] = idx < nchunks ? xs[idx * Fm::kPerChunk + q] : 0.0f;
    }
  }

  int k = 0;
  bool ok = true;
  auto consume = [&](int n_items, bool shared_rows, int first) {
    const int s = k % stages;
    if (ok && !mbar_wait(&pipe.full[s], (k / stages) & 1)) {
      raise_error(err, kDevWaitTimeout, 12, k, warp);
      pipe.abort = 1;
      ok = false;
    }
    if (ok && warp < n_items) {
      const uint4* gs = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(s) * stage_bytes +
                                                       static_cast<size_t>(warp) * row_bytes);
      const uint4* us = reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(gs) +
                                                       static_cast<size_t>(rps) * row_bytes);
      const int q = first + warp;
      const int u_idx = shared_rows ? -1 : q / F;
      const int f = shared_rows ? q : q % F;
      const int64_t row = shared_rows ? q : static_cast<int64_t>(sroute.expert[u_idx]) * F + f;
      const int ntok = shared_rows ? T : sroute.ntok[u_idx];
      const int base = shared_rows ? 0 : sroute.base[u_idx];
      float gacc[kDecodeMaxRows], uacc[kDecodeMaxRows];
#pragma unroll
      for (int j = 0; j < kDecodeMaxRows; ++j) gacc[j] = uacc[j] = 0.0f;
      for (int pass = 0; pass < nchunks; pass += 32 * kChunkMax) {
        uint4 wg[kChunkMax], wu[kChunkMax];
#pragma unroll
        for (int c = 0; c < kChunkMax; ++c) {
          const int idx = pass + lane + 32 * c;
          if (idx < nchunks) {
            wg[c] = gs[idx];
            wu[c] = us[idx];
          }
        }
        if (x_in_regs) {
#pragma unroll
          for (int c = 0; c < kChunkMax; ++c) {
            if (lane + 32 * c < nchunks) {
              gacc[0] += Fm::dot_x(wg[c], xr[c]);
              uacc[0] += Fm::dot_x(wu[c], xr[c]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kDecodeMaxRows; ++j) {
            if (j >= ntok) break;
            const int t = shared_rows ? j : sroute.slot_tok[base + j];
            const float* xrow = xs + static_cast<size_t>(t) * H;
            float pg = 0.0f, pu = 0.0f;
#pragma unroll
            for (int c = 0; c < kChunkMax; ++c) {
              const int idx = pass + lane + 32 * c;
              if (idx < nchunks) {
                pg += Fm::dot_x(wg[c], xrow + idx * Fm::kPerChunk);
                pu += Fm::dot_x(wu[c], xrow + idx * Fm::kPerChunk);
              }
            }
            gacc[j] += pg;
            uacc[j] += pu;
          }
        }
      }
      const float gsc = Fm::scale(shared_rows ? sgate : gate, row);
      const float usc = Fm::scale(shared_rows ? sup : up, row);
#pragma unroll
      for (int j = 0; j < kDecodeMaxRows; ++j) {
        if (j >= ntok) break;
        const float gv = warp_sum(gacc[j]) * gsc;
        const float uv = warp_sum(uacc[j]) * usc;
        if (lane == 0) {
          const __nv_bfloat16 a = __float2bfloat16_rn(swiglu(gv, uv));
          if (shared_rows)
            act_s[static_cast<int64_t>(j) * S + f] = a;
          else
            act[static_cast<int64_t>(base + j) * F + f] = a;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&pipe.empty[s]);
    ++k;
  };

  for (int st = 0; st < sh_stages; ++st) {
    const int first = s0 + st * rps;
    consume(min(rps, s1 - first), true, first);
  }
  if (solo_route) {
    if (ok) ok = wait_route(pipe, err, 13);
  } else {
    pdl_wait();
    build_route(rsrc, T, &sroute, tid, kThreads, kBarAll);
  }
  pdl_launch_dependents();
  const int64_t UF = static_cast<int64_t>(sroute.count) * F;
  const int q0 = split_begin(UF, G, b), q1 = split_begin(UF, G, b + 1);
  for (int first = q0; first < q1; first += rps) consume(min(rps, q1 - first), false, first);
}

// ---------------------------------------------------------------------------
// down + combine. Block b owns output channels [H*b/G, H*(b+1)/G). Parts:
// the shared down rows of those channels, then each selected expert's down
// rows of those channels (ascending expert id). A stage holds up to
// stage_bytes / row_bytes rows of one part (one bulk copy); channel r of the
// block is always computed by consumer warp r % 8, which owns its sums.
template <typename Rows>
__global__ void __launch_bounds__(kThreads, 1)
    down_decode_kernel(int T, int H, int F, int S, Rows down, Rows sdown, RouteSrc rsrc,
                       const __nv_bfloat16* __restrict__ act, const __nv_bfloat16* __restrict__ act_s,
                       const float* resid, float* y, ErrorWord* err, int stages, int stage_bytes) {
  using Fm = Fmt<Rows>;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ Pipe pipe;
  __shared__ SmemRoute sroute;
  __shared__ float shared_sum[kMaxChan][kDecodeMaxRows];
  __shared__ float routed_sum[kMaxChan][kDecodeMaxRows];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int c0 = split_begin(H, G, b), c1 = split_begin(H, G, b + 1);
  const int nc = c1 - c0;
  const bool solo_route = producer_routes(T);
  if (tid == 0) {
    init_pipe(pipe, stages);
    if (nc > kMaxChan) raise_error(err, kDevCapacity, 20, nc, kMaxChan);
  }
  for (int i = tid; i < kMaxChan * kDecodeMaxRows; i += kThreads) {
    (&shared_sum[0][0])[i] = 0.0f;
    (&routed_sum[0][0])[i] = 0.0f;
  }
  __syncthreads();
  if (nc > kMaxChan || nc <= 0) {
    pdl_launch_dependents();
    return;
  }
  // The router's logits are complete when this grid starts: the gate/up grid
  // released it only after the router grid had finished.
  if (!solo_route) build_route(rsrc, T, &sroute, tid, kThreads, kBarAll);
  const int shared_parts = S > 0 ? 1 : 0;

  if (warp == kConsumerWarps) {
    int k = 0;
    bool ok = true;
    auto issue_part = [&](int p) {
      const bool shared_part = p < shared_parts;
      const int rb = (shared_part ? S : F) * Fm::kElemBytes;
      const int rcap = stage_bytes / rb;
      const int u = p - shared_parts;
      for (int r0 = 0; r0 < nc && ok; r0 += rcap) {
        const int n = min(rcap, nc - r0);
        const int s = k % stages;
        if (!mbar_wait(&pipe.empty[s], ((k / stages) & 1) ^ 1)) {
          raise_error(err, kDevWaitTimeout, 21, k, 0);
          pipe.abort = 1;
          ok = false;
          break;
        }
        // One part's rows for consecutive channels are contiguous: one copy.
        const int64_t row = shared_part ? (c0 + r0) : static_cast<int64_t>(sroute.expert[u]) * H + c0 + r0;
        const char* src = Fm::row(shared_part ? sdown : down, row);
        mbar_arrive_expect_tx(&pipe.full[s], static_cast<uint32_t>(n * rb));
        bulk_g2s(ring + static_cast<size_t>(s) * stage_bytes, src, static_cast<uint32_t>(n * rb), &pipe.full[s]);
        ++k;
      }
    };
    if (lane == 0)
      for (int p = 0; p < shared_parts; ++p) issue_part(p);  // needs no routing
    if (solo_route) {
      __syncwarp();
      build_route(rsrc, T, &sroute, lane, 32, 0);
      if (lane == 0) mbar_arrive(&pipe.route_ready);
    }
    if (lane == 0) {
      for (int p = shared_parts; p < shared_parts + sroute.count && ok; ++p) issue_part(p);
      for (int j = max(0, k - stages); j < k; ++j)
        if (!mbar_wait(&pipe.full[j % stages], (j / stages) & 1)) raise_error(err, kDevWaitTimeout, 22, j, 0);
    }
    __syncwarp();
    pdl_launch_dependents();
    return;
  }

  // Consumers read the activations: wait for the gate/up grid.
  pdl_wait();
  pdl_launch_dependents();
  int k = 0;
  bool ok = true;
  bool have_route = !solo_route;
  for (int p = 0; ok && !pipe.abort; ++p) {
    if (p >= shared_parts && !have_route) {
      ok = wait_route(pipe, err, 24);
      have_route = true;
      if (!ok) break;
    }
    if (p >= shared_parts + (have_route ? sroute.count : 0)) break;
    const bool shared_part = p < shared_parts;
    const int rb = (shared_part ? S : F) * Fm::kElemBytes;
    const int rcap = stage_bytes / rb;
    const int u = p - shared_parts;
    const int ntok = shared_part ? T : sroute.ntok[u];
    const int base = shared_part ? 0 : sroute.base[u];
    const int nchunks = rb / 16;
    for (int r0 = 0; r0 < nc; r0 += rcap) {
      const int n = min(rcap, nc - r0);
      const int s = k % stages;
      if (!mbar_wait(&pipe.full[s], (k / stages) & 1)) {
        raise_error(err, kDevWaitTimeout, 23, k, warp);
        pipe.abort = 1;
        ok = false;
        break;
      }
      const unsigned char* stage = ring + static_cast<size_t>(s) * stage_bytes;
      // The first row of this stage that this warp owns (rows r with r % 8 == warp).
      const int first = r0 + ((warp - r0 % kConsumerWarps) + kConsumerWarps) % kConsumerWarps;
      for (int r = first; r < r0 + n; r += kConsumerWarps) {
        const uint4* wrow = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r - r0) * rb);
        const int c = c0 + r;
        const int64_t grow = shared_part ? c : static_cast<int64_t>(sroute.expert[u]) * H + c;
        const float sc = Fm::scale(shared_part ? sdown : down, grow);
        float acc[kDecodeMaxRows];
#pragma unroll
        for (int j = 0; j < kDecodeMaxRows; ++j) acc[j] = 0.0f;
        for (int pass = 0; pass < nchunks; pass += 32 * kChunkMax) {
          uint4 w[kChunkMax];
#pragma unroll
          for (int q = 0; q < kChunkMax; ++q) {
            const int idx = pass + lane + 32 * q;
            if (idx < nchunks) w[q] = wrow[idx];
          }
#pragma unroll
          for (int j = 0; j < kDecodeMaxRows; ++j) {
            if (j >= ntok) break;
            const __nv_bfloat16* ar = shared_part ? act_s + static_cast<int64_t>(j) * S
                                                  : act + static_cast<int64_t>(base + j) * F;
            float pr = 0.0f;
#pragma unroll
            for (int q = 0; q < kChunkMax; ++q) {
              const int idx = pass + lane + 32 * q;
              if (idx < nchunks) pr += Fm::dot_act(w[q], ar + idx * Fm::kPerChunk);
            }
            acc[j] += pr;
          }
        }
#pragma unroll
        for (int j = 0; j < kDecodeMaxRows; ++j) {
          if (j >= ntok) break;
          const float v = warp_sum(acc[j]) * sc;
          if (lane == 0) {
            if (shared_part) {
              shared_sum[r][j] = v;
            } else {
              const int t = sroute.slot_tok[base + j];
              routed_sum[r][t] = __fadd_rn(routed_sum[r][t], __fmul_rn(sroute.slot_w[base + j], v));
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pipe.empty[s]);
      ++k;
    }
  }
  __syncwarp();
  // Each warp writes the channels it owns.
  for (int r = warp; r < nc; r += kConsumerWarps) {
    const int c = c0 + r;
    for (int t = lane; t < T; t += 32) {
      const int64_t o = static_cast<int64_t>(t) * H + c;
      float out = __fadd_rn(shared_sum[r][t], routed_sum[r][t]);
      if (resid != nullptr) out = __fadd_rn(resid[o], out);
      y[o] = out;
    }
  }
}

// Launch geometry.
struct Geometry {
  int stages = 0;
  int param = 0;  // rps for gate/up, stage bytes for down
  size_t smem = 0;
};

int device_optin_smem() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return v;
}

template <typename Rows>
int static_smem(bool gate_up) {
  cudaFuncAttributes a{};
  if (gate_up)
    cudaFuncGetAttributes(&a, gate_up_decode_kernel<Rows>);
  else
    cudaFuncGetAttributes(&a, down_decode_kernel<Rows>);
  return static_cast<int>(a.sharedSizeBytes);
}

template <typename Rows>
bool gate_up_geometry(int T, int H, Geometry& g) {
  const long avail = static_cast<long>(device_optin_smem()) - static_smem<Rows>(true) - 512;
  const long xs = (static_cast<long>(T) * H * 4 + 127) & ~127L;
  const long row = static_cast<long>(H) * Fmt<Rows>::kElemBytes;
  if (avail - xs < 2 * 2 * row) return false;
  const long budget = avail - xs < 192 * 1024 ? avail - xs : 192 * 1024;
  int rps = kConsumerWarps;
  while (rps > 1 && 2 * 2 * rps * row > budget) --rps;
  int stages = kMaxStages;
  while (stages > 2 && stages * 2 * rps * row > budget) --stages;
  if (stages * 2 * rps * row > avail - xs) return false;
  g.stages = stages;
  g.param = rps;
  g.smem = static_cast<size_t>(xs + stages * 2 * rps * row);
  return true;
}

template <typename Rows>
bool down_geometry(int H, int F, int S, int blocks, Geometry& g) {
  const long avail = static_cast<long>(device_optin_smem()) - static_smem<Rows>(false) - 512;
  const long nc = (H + blocks - 1) / blocks;
  const long row = static_cast<long>(S > F ? S : F) * Fmt<Rows>::kElemBytes;
  const int stages = 3;
  long stage = nc * row;
  if (stage * stages > avail) stage = (avail / stages) / row * row;
  if (stage < row) return false;
  g.stages = stages;
  g.param = static_cast<int>(stage);
  g.smem = static_cast<size_t>(stage * stages);
  return true;
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
  st = allow_max_dynamic_smem(gate_up_decode_kernel<Rows>);
  if (st == cudaSuccess) st = allow_max_dynamic_smem(down_decode_kernel<Rows>);
  if (st == cudaSuccess && dev < kMaxDevices) done[dev] = true;
  return st;
}

template <typename Rows>
cudaError_t launch_decode_experts_t(const float* x, int T, int H, int F, int S, Rows gate, Rows up, Rows down,
                                    Rows sgate, Rows sup, Rows sdown, const DecodeRouting& routing,
                                    __nv_bfloat16* act, __nv_bfloat16* act_s, const float* resid, float* y,
                                    ErrorWord* err, int sm_count, cudaStream_t stream, cudaEvent_t between,
                                    bool pdl) {
  cudaError_t st = prepare_kernels<Rows>();
  if (st != cudaSuccess) return st;
  Geometry gu, dn;
  const int dn_blocks = H < sm_count ? H : sm_count;
  if (!gate_up_geometry<Rows>(T, H, gu) || !down_geometry<Rows>(H, F, S, dn_blocks, dn))
    return cudaErrorInvalidConfiguration;
  if ((H + dn_blocks - 1) / dn_blocks > kMaxChan) return cudaErrorInvalidConfiguration;
  RouteSrc rs{routing.logits, routing.table, routing.experts, routing.top_k, routing.renormalize, routing.ids_out,
              routing.weights_out};
  {
    void* args[] = {&x, &T, &H, &F, &S, &gate, &up, &sgate, &sup, &rs, &act, &act_s, &err, &gu.stages, &gu.param};
    st = launch_maybe_pdl(reinterpret_cast<const void*>(gate_up_decode_kernel<Rows>), dim3(sm_count),
                          dim3(kThreads), gu.smem, stream, args, pdl);
    if (st != cudaSuccess) return st;
  }
  if (between != nullptr) {
    st = cudaEventRecord(between, stream);
    if (st != cudaSuccess) return st;
  }
  rs.ids_out = nullptr;
  rs.w_out = nullptr;
  void* args[] = {&T, &H, &F, &S, &down, &sdown, &rs, &act, &act_s, &resid, &y, &err, &dn.stages, &dn.param};
  return launch_maybe_pdl(reinterpret_cast<const void*>(down_decode_kernel<Rows>), dim3(dn_blocks), dim3(kThreads),
                          dn.smem, stream, args, pdl && between == nullptr);
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
                                       int sm_count, cudaStream_t stream, cudaEvent_t between, bool pdl) {
  return launch_decode_experts_t<Bf16Rows>(x, T, H, F, S, Bf16Rows{gate, H}, Bf16Rows{up, H}, Bf16Rows{down, F},
                                           Bf16Rows{sgate, H}, Bf16Rows{sup, H}, Bf16Rows{sdown, S}, routing, act,
                                           act_s, resid, y, err, sm_count, stream, between, pdl);
}

cudaError_t launch_decode_experts_q8(const float* x, int T, int H, int F, int S, Q8Rows gate, Q8Rows up,
                                     Q8Rows down, Q8Rows sgate, Q8Rows sup, Q8Rows sdown,
                                     const DecodeRouting& routing, __nv_bfloat16* act, __nv_bfloat16* act_s,
                                     const float* resid, float* y, ErrorWord* err, int sm_count, cudaStream_t stream,
                                     cudaEvent_t between, bool pdl) {
  return launch_decode_experts_t<Q8Rows>(x, T, H, F, S, gate, up, down, sgate, sup, sdown, routing, act, act_s,
                                         resid, y, err, sm_count, stream, between, pdl);
}

cudaError_t prepare_decode_experts(int max_rows, int H) {
  cudaError_t st = prepare_kernels<Bf16Rows>();
  if (st == cudaSuccess) st = prepare_kernels<Q8Rows>();
  if (st != cudaSuccess) return st;
  Geometry g;
  if (!gate_up_geometry<Bf16Rows>(max_rows, H, g) || !gate_up_geometry<Q8Rows>(max_rows, H, g))
    return cudaErrorInvalidConfiguration;
  return cudaSuccess;
}

}  // namespace uocr_b200
