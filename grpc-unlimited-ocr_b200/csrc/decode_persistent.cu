// Persistent decode: the whole stack of MoE layers for a batch of <= 16 rows
// in one cooperative launch — one block per SM, 15 streaming warps and one
// control warp — with three grid-wide barriers per layer and the weight
// streaming of the next phase started before each barrier:
//
//   R  router logits: block e stages router row e (before the previous
//      layer's last barrier — it does not depend on x) and runs the exact
//      8-lane dot order of the reference (src/backend/reference/ops.cpp:25-38).
//      [barrier 1]  the streaming warps already stream the shared expert's
//      gate/up rows, which need no routing; the control warp waits, then
//      builds the routing table from the logits (softmax, top-k, renorm).
//   G  gate/up of the selected experts: act = bf16(silu(g) * u), grid-wide
//      over (expert, ffn row) pairs.
//      [barrier 2]  each warp has issued its first down rows' loads first.
//   D  down + combine: block b owns a slice of output channels; its warps
//      take (channel, shared or expert row) units two at a time; the
//      partials meet in shared memory and are added per row in ascending
//      expert id, then the residual (src/model/feed_forward.cpp:65-76).
//      [barrier 3]  the next layer's router row is staged first.
//
// Same arithmetic as the per-layer kernels of decode.cu, which remain the
// fallback for shapes whose rows do not fit in shared memory. Every grid
// wait is bounded (2 s, then an error word and an orderly exit of all blocks).
#include <mutex>

#include "decode_fmt.cuh"
#include "decode_persistent.h"
#include "moe_kernels.h"
#include "ptx.cuh"
#include "route.cuh"

namespace uocr_b200 {
namespace {

constexpr int kWorkers = 15;
constexpr int kThreads = (kWorkers + 1) * 32;
constexpr int kCtl = kWorkers;  // the control warp
constexpr uint64_t kGridWaitNs = 2000000000ull;

// 16-byte loads per lane per pass: gate/up (each of the two rows) and each
// of the two down units of a pair.
template <int MaxT>
constexpr int chunk_count() { return MaxT <= 4 ? 8 : 4; }

// Output channels one block owns in phase D: ceil(H / blocks) <= this.
constexpr int kMaxChannelsPerBlock = 64;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// CTA barrier that warps may reach from different places in the code.
__device__ __forceinline__ void cta_sync_any(unsigned id) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(kThreads) : "memory");
}

// One thread per block. Returns the generation to wait on.
__device__ unsigned grid_arrive(GridBarrier* b, unsigned nblocks) {
  const unsigned g = ld_acquire_gpu(&b->gen);  // cannot move before this block arrives
  __threadfence();
  if (atomicAdd(&b->count, 1u) == nblocks - 1) {
    atomicExch(&b->count, 0u);
    __threadfence();
    st_release_gpu(&b->gen, g + 1);
  }
  return g;
}

// One thread per block; false when it gave up (time limit, or another block
// already recorded an error).
__device__ bool grid_wait(GridBarrier* b, unsigned g, ErrorWord* err, int site) {
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_gpu(&b->gen) != g) return true;
    if ((i & 15u) == 15u) {
      if (ld_volatile(&err->code) != 0) return false;
      if (global_timer_ns() - start > kGridWaitNs || i > (1u << 26)) {
        raise_error(err, kDevWaitTimeout, site, static_cast<int>(blockIdx.x), static_cast<int>(g));
        return false;
      }
    }
    __nanosleep(32);
  }
}

template <typename Rows>
__device__ Rows rows_of(const void* w, const float* s, int64_t cols);
template <>
__device__ Bf16Rows rows_of<Bf16Rows>(const void* w, const float*, int64_t cols) {
  return Bf16Rows{static_cast<const __nv_bfloat16*>(w), cols};
}
template <>
__device__ Q8Rows rows_of<Q8Rows>(const void* w, const float* s, int64_t cols) {
  return Q8Rows{static_cast<const int8_t*>(w), s, cols};
}

// n floats from global (fp32, 16-byte aligned) into shared memory, every
// thread's loads issued before its stores. `cg`: written in this kernel.
__device__ __forceinline__ void stage_f32(float* dst, const float* src, int n, bool cg) {
  const int n4 = n / 4;
  for (int i0 = threadIdx.x; i0 < n4; i0 += kThreads * 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * kThreads;
      if (i < n4)
        v[u] = cg ? __ldcg(reinterpret_cast<const float4*>(src) + i) : __ldg(reinterpret_cast<const float4*>(src) + i);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * kThreads;
      if (i < n4) reinterpret_cast<float4*>(dst)[i] = v[u];
    }
  }
}

// A down-projection unit: one weight row against `nt` activation rows.
struct DownUnit {
  const uint4* w;
  float scale;
  int nchunks;
  int nt;
  const __nv_bfloat16* act;
  int64_t act_stride;
  float* out;  // nt partial sums (shared memory)
};

// One gate/up unit: rows f of gate and up against `ntok` input rows (toks:
// their indices into `xs`, or null for 0..ntok-1); lane 0 writes
// act = bf16(silu(g) * u) to out[j * out_stride].
template <typename Rows, int MaxT>
__device__ __forceinline__ void gate_up_unit(const float* xs, int H, int nx, const uint4* gr, const uint4* ur, float gsc,
                                          float usc, int ntok, const int* toks, __nv_bfloat16* out,
                                          int64_t out_stride) {
  using Fm = Fmt<Rows>;
  constexpr int kC = chunk_count<MaxT>();
  const int lane = threadIdx.x & 31;
  float gacc[MaxT], uacc[MaxT];
#pragma unroll
  for (int j = 0; j < MaxT; ++j) gacc[j] = uacc[j] = 0.0f;
  for (int pass = 0; pass < nx; pass += 32 * kC) {
    uint4 wg[kC], wu[kC];
#pragma unroll
    for (int q = 0; q < kC; ++q) {
      const int idx = pass + lane + 32 * q;
      if (idx < nx) {
        wg[q] = ld_stream(gr + idx);
        wu[q] = ld_stream(ur + idx);
      }
    }
#pragma unroll
    for (int j = 0; j < MaxT; ++j) {
      if (j >= ntok) break;
      const float* xr = xs + static_cast<size_t>(toks == nullptr ? j : toks[j]) * H;
#pragma unroll
      for (int q = 0; q < kC; ++q) {
        const int idx = pass + lane + 32 * q;
        if (idx < nx) {
          gacc[j] += Fm::dot_x(wg[q], xr + idx * Fm::kPerChunk);
          uacc[j] += Fm::dot_x(wu[q], xr + idx * Fm::kPerChunk);
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
}

// Two down units at once (the second's loads in flight with the first's);
// before the first dot product the warp meets the rest of the block at
// barrier 1 (`sync`), where the control warp has passed the grid barrier.
// Returns false if the block is aborting.
template <typename Rows, int MaxT>
__device__ __forceinline__ bool down_pair(const DownUnit& A, const DownUnit& B, bool* synced, const int* abort_flag) {
  using Fm = Fmt<Rows>;
  constexpr int kC = chunk_count<MaxT>() / 2;  // per unit: the pair issues as many loads as one gate/up unit
  const int lane = threadIdx.x & 31;
  float a0[MaxT], a1[MaxT];
#pragma unroll
  for (int j = 0; j < MaxT; ++j) a0[j] = a1[j] = 0.0f;
  const int n = A.nchunks > B.nchunks ? A.nchunks : B.nchunks;
  for (int pass = 0; pass < n || !*synced; pass += 32 * kC) {
    uint4 w0[kC], w1[kC];
#pragma unroll
    for (int q = 0; q < kC; ++q) {
      const int idx = pass + lane + 32 * q;
      if (idx < A.nchunks) w0[q] = ld_stream(A.w + idx);
      if (idx < B.nchunks) w1[q] = ld_stream(B.w + idx);
    }
    if (!*synced) {
      cta_sync_any(1);
      *synced = true;
    }
    if (ld_volatile(abort_flag)) return false;
#pragma unroll
    for (int j = 0; j < MaxT; ++j) {
      if (j >= A.nt) break;
      const __nv_bfloat16* ar = A.act + j * A.act_stride;
#pragma unroll
      for (int q = 0; q < kC; ++q) {
        const int idx = pass + lane + 32 * q;
        if (idx < A.nchunks) a0[j] += Fm::template dot_act<1>(w0[q], ar + idx * Fm::kPerChunk);
      }
    }
#pragma unroll
    for (int j = 0; j < MaxT; ++j) {
      if (j >= B.nt) break;
      const __nv_bfloat16* ar = B.act + j * B.act_stride;
#pragma unroll
      for (int q = 0; q < kC; ++q) {
        const int idx = pass + lane + 32 * q;
        if (idx < B.nchunks) a1[j] += Fm::template dot_act<1>(w1[q], ar + idx * Fm::kPerChunk);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < MaxT; ++j) {
    if (j >= A.nt) break;
    const float v = warp_sum(a0[j]) * A.scale;
    if (lane == 0) A.out[j] = v;
  }
#pragma unroll
  for (int j = 0; j < MaxT; ++j) {
    if (j >= B.nt) break;
    const float v = warp_sum(a1[j]) * B.scale;
    if (lane == 0) B.out[j] = v;
  }
  return true;
}

// The streaming warps' gate/up work of one layer: the shared expert's rows
// (r == null: every input row) or the selected experts' (expert, row) pairs,
// dealt grid-wide by global warp index.
template <typename Rows, int MaxT>
__device__ __forceinline__ void gate_up_phase(const float* xs, int T, int H, int F, int S, Rows g, Rows u,
                                           const SmemRoute* r, __nv_bfloat16* act, __nv_bfloat16* act_s, int gw,
                                           int GW) {
  using Fm = Fmt<Rows>;
  const int nx = H * Fm::kElemBytes / 16;
  if (r == nullptr) {
    for (int f = gw; f < S; f += GW)
      gate_up_unit<Rows, MaxT>(xs, H, nx, Fm::row(g, f), Fm::row(u, f), Fm::scale(g, f), Fm::scale(u, f), T,
                               nullptr, act_s + f, S);
    return;
  }
  const int U = r->count;
  for (int q = gw; q < U * F; q += GW) {
    const int e = q / F, f = q % F;
    const int64_t row = static_cast<int64_t>(r->expert[e]) * F + f;
    const int base = r->base[e];
    gate_up_unit<Rows, MaxT>(xs, H, nx, Fm::row(g, row), Fm::row(u, row), Fm::scale(g, row), Fm::scale(u, row),
                             r->ntok[e], r->slot_tok + base, act + static_cast<int64_t>(base) * F + f, F);
  }
}

// What a streaming warp needs for its down units in one layer.
template <typename Rows>
struct DownCtx {
  Rows down, sdown;
  const SmemRoute* r;
  const __nv_bfloat16* act;
  const __nv_bfloat16* act_s;
  float* part;  // [units][MaxT] in shared memory
  int T, H, F, S, c_begin, P, nunits;
};

// The streaming warps' down work: units (channel, shared row or expert row),
// block-local, two at a time; the first loads precede barrier 1.
template <typename Rows, int MaxT>
__device__ __forceinline__ void down_phase(const DownCtx<Rows>& d, int warp, const int* abort_flag) {
  using Fm = Fmt<Rows>;
  auto describe = [&](int q) {
    DownUnit u{};
    if (q >= d.nunits) return u;
    const int cl = q / d.P, p = q % d.P, ch = d.c_begin + cl;
    u.out = d.part + static_cast<int64_t>(q) * MaxT;
    if (d.S > 0 && p == 0) {
      u.w = Fm::row(d.sdown, ch);
      u.scale = Fm::scale(d.sdown, ch);
      u.nchunks = d.S * Fm::kElemBytes / 16;
      u.nt = d.T;
      u.act = d.act_s;
      u.act_stride = d.S;
    } else {
      const int e = p - (d.S > 0 ? 1 : 0);
      const int64_t row = static_cast<int64_t>(d.r->expert[e]) * d.H + ch;
      u.w = Fm::row(d.down, row);
      u.scale = Fm::scale(d.down, row);
      u.nchunks = d.F * Fm::kElemBytes / 16;
      u.nt = d.r->ntok[e];
      u.act = d.act + static_cast<int64_t>(d.r->base[e]) * d.F;
      u.act_stride = d.F;
    }
    return u;
  };
  bool synced = false;
  for (int q0 = warp; q0 < d.nunits || !synced; q0 += 2 * kWorkers)
    if (!down_pair<Rows, MaxT>(describe(q0), describe(q0 + kWorkers), &synced, abort_flag)) break;
}

template <typename Rows, int MaxT>
__global__ void __launch_bounds__(kThreads, 1)
    persistent_decode_kernel(PersistentDecodeCall c, int region_floats) {
  using Fm = Fmt<Rows>;
  extern __shared__ __align__(16) float smem[];
  float* region = smem;                 // phase R/G: the T input rows; phase D: the down partials
  float* rrow = smem + region_floats;   // one router row
  __shared__ SmemRoute sroute;
  __shared__ uint64_t route_ready;
  __shared__ unsigned s_gen;
  __shared__ int s_abort;
  __shared__ float resid_s[kDecodeMaxRows * kMaxChannelsPerBlock];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int T = c.T, H = c.H, E = c.E, K = c.K, F = c.F, S = c.S;
  const unsigned G = gridDim.x;
  if (tid == 0) {
    mbar_init(&route_ready, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  const int gw = static_cast<int>(blockIdx.x) * kWorkers + warp, GW = static_cast<int>(G) * kWorkers;
  const int c_begin = static_cast<int>(static_cast<int64_t>(H) * blockIdx.x / G);
  const int c_end = static_cast<int>(static_cast<int64_t>(H) * (blockIdx.x + 1) / G);
  const int nch = c_end - c_begin;
  unsigned gen = 0;

  for (int l = 0; l < c.n_layers; ++l) {
    // Weight pointers are read where each phase needs them (not held in
    // registers across the phases).
    const DecodeLayerW* Wp = c.layers + l;
    const float* xin = l == 0 ? c.x : c.y;
    const bool last = l + 1 == c.n_layers;

    // ---- R: router row (independent of x), then the previous layer's end.
    if (static_cast<int>(blockIdx.x) < E) stage_f32(rrow, Wp->router + static_cast<int64_t>(blockIdx.x) * H, H, false);
    if (l > 0) {
      if (tid == 0 && !grid_wait(c.barrier, gen, c.err, 70)) s_abort = 1;
      __syncthreads();
      if (s_abort) return;
    }
    stage_f32(region, xin, T * H, true);
    __syncthreads();
    for (int e = blockIdx.x; e < E; e += G) {
      if (e != static_cast<int>(blockIdx.x)) {
        __syncthreads();
        stage_f32(rrow, Wp->router + static_cast<int64_t>(e) * H, H, false);
        __syncthreads();
      }
      if (tid < ((T * 8 + 31) & ~31)) {  // whole warps: the shuffles below need every lane
        const bool valid = tid < T * 8;
        const int t = tid >> 3, l8 = tid & 7;
        const float* xr = region + static_cast<int64_t>(valid ? t : 0) * H;
        const int full = H & ~7;
        float acc = 0.0f, tail = 0.0f;
        if (valid) {
          // Eight elements of the chain loaded before they are added: the
          // shared-memory latency is paid once per eight dependent adds.
          int i = l8;
          for (; i + 56 < full; i += 64) {
            float xv[8], wv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              xv[u] = xr[i + 8 * u];
              wv[u] = rrow[i + 8 * u];
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(xv[u], wv[u]));
          }
          for (; i < full; i += 8) acc = __fadd_rn(acc, __fmul_rn(xr[i], rrow[i]));
          if (l8 == 0)
            for (int k = full; k < H; ++k) tail = __fadd_rn(tail, __fmul_rn(xr[k], rrow[k]));
        }
        float a[8];
        const int base = lane & ~7;
#pragma unroll
        for (int q = 0; q < 8; ++q) a[q] = __shfl_sync(0xffffffffu, acc, base + q, 32);
        if (valid && l8 == 0) {
          const float lo = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
          const float hi = __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7]));
          float s = __fadd_rn(__fadd_rn(lo, hi), tail);
          const float* bias = Wp->bias;
          if (bias != nullptr) s = __fadd_rn(s, bias[e]);
          c.logits[static_cast<int64_t>(t) * E + e] = s;
        }
      }
    }
    __syncthreads();
    // This block's output channels of the (unrounded) input rows: the
    // residual, kept here because phase D reuses the region.
    if (c.residual)
      for (int i = tid; i < nch * T; i += kThreads) resid_s[i] = region[(i / nch) * H + c_begin + i % nch];
    for (int i = tid; i < T * H; i += kThreads) region[i] = bf16_round(region[i]);
    __syncthreads();
    if (tid == 0) s_gen = grid_arrive(c.barrier, G);
    __syncthreads();
    gen = s_gen;

    // ---- G: shared expert (no routing needed) during the barrier, then routed.
    if (warp == kCtl) {
      int ok = 1;
      if (lane == 0) ok = grid_wait(c.barrier, gen, c.err, 71) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) {
        const bool ids = last && blockIdx.x == 0;
        route_from_logits(c.logits, T, E, K, c.renorm, &sroute, lane, 32, 0, ids ? c.ids_out : nullptr,
                          ids ? c.w_out : nullptr);
      } else if (lane == 0) {
        s_abort = 1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&route_ready);
    } else {
      gate_up_phase<Rows, MaxT>(region, T, H, F, S, rows_of<Rows>(Wp->sgate, Wp->sgate_s, H),
                                rows_of<Rows>(Wp->sup, Wp->sup_s, H), nullptr, c.act, c.act_s, gw, GW);
      if (!mbar_wait(&route_ready, static_cast<uint32_t>(l & 1))) {
        if (lane == 0) {
          raise_error(c.err, kDevWaitTimeout, 72, static_cast<int>(blockIdx.x), l);
          s_abort = 1;
        }
      }
      __syncwarp();
      if (!ld_volatile(&s_abort))
        gate_up_phase<Rows, MaxT>(region, T, H, F, S, rows_of<Rows>(Wp->gate, Wp->gate_s, H),
                                  rows_of<Rows>(Wp->up, Wp->up_s, H), &sroute, c.act, c.act_s, gw, GW);
    }
    __syncthreads();
    if (s_abort) return;
    if (tid == 0) s_gen = grid_arrive(c.barrier, G);
    __syncthreads();
    gen = s_gen;

    // ---- D: this block's channels; first loads issued before the barrier wait.
    const int U = sroute.count;
    const int P = (S > 0 ? 1 : 0) + U;  // units per channel: shared row, then one per expert
    const int nunits = nch * P;
    float* part = region;  // [nunits][MaxT]
    if (warp == kCtl) {
      int ok = 1;
      if (lane == 0) ok = grid_wait(c.barrier, gen, c.err, 73) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok && lane == 0) s_abort = 1;
      __syncwarp();
      cta_sync_any(1);
    } else {
      const DownCtx<Rows> dc{rows_of<Rows>(Wp->down, Wp->down_s, F), rows_of<Rows>(Wp->sdown, Wp->sdown_s, S),
                             &sroute, c.act, c.act_s, part, T, H, F, S, c_begin, P, nunits};
      down_phase<Rows, MaxT>(dc, warp, &s_abort);
    }
    __syncthreads();
    if (s_abort) return;
    // Combine: shared part, then the experts in ascending id, then the residual.
    for (int i = tid; i < nch * T; i += kThreads) {
      const int cl = i / T, t = i % T;
      const float* pc = part + static_cast<int64_t>(cl) * P * MaxT;
      float sum = S > 0 ? pc[t] : 0.0f;
      const int p0 = S > 0 ? 1 : 0;
      for (int u = 0; u < U; ++u) {
        const int base = sroute.base[u], n = sroute.ntok[u];
        for (int j = 0; j < n; ++j)
          if (sroute.slot_tok[base + j] == t)
            sum = __fadd_rn(sum, __fmul_rn(sroute.slot_w[base + j], pc[(p0 + u) * MaxT + j]));
      }
      const int64_t o = static_cast<int64_t>(t) * H + c_begin + cl;
      c.y[o] = c.residual ? __fadd_rn(resid_s[t * nch + cl], sum) : sum;
    }
    __syncthreads();
    if (!last) {
      if (tid == 0) s_gen = grid_arrive(c.barrier, G);
      __syncthreads();
      gen = s_gen;
    }
  }
}

struct KernelInfo {
  bool ready = false;
  size_t static_smem[2][4] = {};
  size_t max_dynamic = 0;
};
KernelInfo g_info[kMaxDevices];
std::mutex g_mu;

template <typename Rows>
const void* pick(int T) {
  if (T <= 1) return reinterpret_cast<const void*>(persistent_decode_kernel<Rows, 1>);
  if (T <= 4) return reinterpret_cast<const void*>(persistent_decode_kernel<Rows, 4>);
  if (T <= 8) return reinterpret_cast<const void*>(persistent_decode_kernel<Rows, 8>);
  return reinterpret_cast<const void*>(persistent_decode_kernel<Rows, kDecodeMaxRows>);
}

int max_t_of(int T) { return T <= 1 ? 1 : T <= 4 ? 4 : T <= 8 ? 8 : kDecodeMaxRows; }

// Dynamic shared memory: the region (T input rows, or the down partials) and one router row.
size_t region_floats(int T, int H, int E, int K, int S, int blocks) {
  const int mt = max_t_of(T);
  const int64_t nch = (H + blocks - 1) / blocks;
  const int64_t P = (S > 0 ? 1 : 0) + (E < T * K ? E : T * K);
  const int64_t a = static_cast<int64_t>(T) * H, b = nch * P * mt;
  const int64_t r = a > b ? a : b;
  return static_cast<size_t>((r + 3) / 4 * 4);
}

size_t static_smem_bound() {
  // SmemRoute plus a few words; checked against the compiled value in prepare.
  return sizeof(SmemRoute) + sizeof(float) * kDecodeMaxRows * kMaxChannelsPerBlock + 64;
}

}  // namespace

bool persistent_decode_fits(int T, int H, int E, int K, int S, int sm_count, size_t smem_optin) {
  if (T < 1 || T > kDecodeMaxRows || H % 16 != 0) return false;
  if ((H + sm_count - 1) / sm_count > kMaxChannelsPerBlock) return false;
  const size_t dyn = (region_floats(T, H, E, K, S, sm_count) + static_cast<size_t>(H)) * sizeof(float);
  return dyn + static_smem_bound() + 1024 <= smem_optin;
}

cudaError_t prepare_persistent_decode() {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  std::lock_guard<std::mutex> lock(g_mu);
  if (dev < kMaxDevices && g_info[dev].ready) return cudaSuccess;
  const void* fns[8] = {pick<Bf16Rows>(1), pick<Bf16Rows>(4), pick<Bf16Rows>(8), pick<Bf16Rows>(16),
                        pick<Q8Rows>(1),   pick<Q8Rows>(4),   pick<Q8Rows>(8),   pick<Q8Rows>(16)};
  int optin = 0;
  if ((st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return st;
  for (const void* f : fns) {
    cudaFuncAttributes a{};
    if ((st = cudaFuncGetAttributes(&a, f)) != cudaSuccess) return st;
    if (a.sharedSizeBytes > static_smem_bound()) return cudaErrorInvalidValue;
    if ((st = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   optin - static_cast<int>(a.sharedSizeBytes))) != cudaSuccess)
      return st;
  }
  if (dev < kMaxDevices) g_info[dev].ready = true;
  return cudaSuccess;
}

cudaError_t launch_persistent_decode(const PersistentDecodeCall& c, cudaStream_t stream) {
  cudaError_t st = prepare_persistent_decode();
  if (st != cudaSuccess) return st;
  if ((st = cudaMemsetAsync(c.barrier, 0, sizeof(GridBarrier), stream)) != cudaSuccess) return st;
  int rf = static_cast<int>(region_floats(c.T, c.H, c.E, c.K, c.S, c.sm_count));
  const size_t smem = (static_cast<size_t>(rf) + static_cast<size_t>(c.H)) * sizeof(float);
  const void* fn = c.int8 ? pick<Q8Rows>(c.T) : pick<Bf16Rows>(c.T);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(c.sm_count);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PersistentDecodeCall arg = c;
  void* args[] = {&arg, &rf};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace uocr_b200
