// Prefill path (rows > 16): router logits for many rows, top-k, the
// token -> expert permutation, and the weighted combine. The expert GEMMs are
// the tcgen05 grouped GEMM (tc_gemm.cu).
//
// The permutation is a histogram / exclusive scan / scatter that keeps every
// expert's rows in token order, so the permuted layout — and everything
// computed from it — is the same on every run. It replaces the reference's
// host-side routing and per-expert gather/scatter loop
// (src/model/cuda/cuda_decoder.cpp:159-191; gather_kernel / scatter_add_kernel,
// src/backend/cuda/ops.cu:171-191), which downloads the logits and runs
// ~2 host synchronisations per expert.
#include "moe_kernels.h"
#include "prefill.h"
#include "route.cuh"

namespace uocr_b200 {
namespace {

constexpr int kRouterTokens = 32;   // rows per router block
constexpr int kRouterExperts = 32;  // experts per router block
constexpr int kRouterChunk = 128;   // K elements staged per step
constexpr int kPermBlock = 256;     // rows per permutation block (8 warps x 32)

// logits[t, e] in the reference's dot order (eight lane partial sums over
// i = 8j + lane, fixed tree, tail, bias: src/backend/reference/ops.cpp:25-38,
// :91-109), every product and sum separately rounded. Block = 32 rows x 8
// lanes; blockIdx.y selects 32 experts; K is staged in chunks.
__global__ void __launch_bounds__(256) router_logits_rows_kernel(const float* __restrict__ x, int T, int H,
                                                                 const float* __restrict__ router,
                                                                 const float* __restrict__ bias, int E,
                                                                 float* __restrict__ logits) {
  __shared__ float xs[kRouterTokens][kRouterChunk + 8];
  __shared__ float ws[kRouterExperts][kRouterChunk];
  const int tid = threadIdx.x;
  const int lane8 = tid & 7, tl = tid >> 3;
  const int t = blockIdx.x * kRouterTokens + tl;
  const int e0 = blockIdx.y * kRouterExperts;
  const int ne = min(kRouterExperts, E - e0);
  float acc[kRouterExperts];
#pragma unroll
  for (int i = 0; i < kRouterExperts; ++i) acc[i] = 0.0f;
  const int full = H & ~7;
  for (int k0 = 0; k0 < full; k0 += kRouterChunk) {
    const int kc = min(kRouterChunk, full - k0);
    __syncthreads();
    for (int i = tid; i < kRouterTokens * kc; i += 256) {
      const int r = i / kc, c = i % kc;
      const int tr = blockIdx.x * kRouterTokens + r;
      xs[r][c] = tr < T ? __ldg(x + static_cast<int64_t>(tr) * H + k0 + c) : 0.0f;
    }
    for (int i = tid; i < kRouterExperts * kc; i += 256) {
      const int r = i / kc, c = i % kc;
      ws[r][c] = r < ne ? __ldg(router + static_cast<int64_t>(e0 + r) * H + k0 + c) : 0.0f;
    }
    __syncthreads();
    for (int j = lane8; j < kc; j += 8) {
      const float xv = xs[tl][j];
#pragma unroll
      for (int i = 0; i < kRouterExperts; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(xv, ws[i][j]));
    }
  }
  // Combine the eight lanes of each (row, expert): lanes of a row are eight
  // consecutive threads of one warp.
  const int base = (tid & 31) & ~7;
#pragma unroll 1
  for (int i = 0; i < ne; ++i) {
    float a[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = __shfl_sync(0xffffffffu, acc[i], base + q);
    if (lane8 == 0 && t < T) {
      const int e = e0 + i;
      const float* xr = x + static_cast<int64_t>(t) * H;
      const float* wr = router + static_cast<int64_t>(e) * H;
      float tail = 0.0f;
      for (int c = full; c < H; ++c) tail = __fadd_rn(tail, __fmul_rn(__ldg(xr + c), __ldg(wr + c)));
      const float lo = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
      const float hi = __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7]));
      float s = __fadd_rn(__fadd_rn(lo, hi), tail);
      if (bias != nullptr) s = __fadd_rn(s, bias[e]);
      logits[static_cast<int64_t>(t) * E + e] = s;
    }
  }
}

__global__ void __launch_bounds__(256) topk_rows_i32_kernel(const float* __restrict__ logits, int T, int E, int K,
                                                            int renorm, int* ids, float* weights) {
  __shared__ float ebuf[8][kMaxExperts];
  const int warp = threadIdx.x >> 5;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (r >= T) return;
  softmax_topk_warp<int>(logits + r * E, E, K, renorm, ebuf[warp], ids + r * K, weights + r * K);
}

// Per block of 256 rows: how many selections each expert received.
__global__ void __launch_bounds__(kPermBlock) count_kernel(const int* __restrict__ ids, int T, int K, int E,
                                                           int* __restrict__ block_counts, ErrorWord* err) {
  __shared__ int cnt[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int t = blockIdx.x * kPermBlock + threadIdx.x;
  if (t < T)
    for (int j = 0; j < K; ++j) {
      const int e = ids[static_cast<int64_t>(t) * K + j];
      if (e >= 0 && e < E)
        atomicAdd(&cnt[e], 1);
      else
        raise_error(err, kDevBadIndex, 30, t, e);
    }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[static_cast<int64_t>(blockIdx.x) * E + e] = cnt[e];
}

// seg_count[e], seg_start[e] (exclusive scan over experts) and each block's
// first position inside every expert's segment.
__global__ void scan_kernel(const int* __restrict__ block_counts, int nblk, int E, int* __restrict__ seg_count,
                            int* __restrict__ seg_start, int* __restrict__ block_offset) {
  __shared__ int total[kMaxExperts];
  __shared__ int start[kMaxExperts];
  const int e = threadIdx.x;
  if (e < E) {
    int s = 0;
    for (int b = 0; b < nblk; ++b) s += block_counts[static_cast<int64_t>(b) * E + e];
    total[e] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      start[i] = acc;
      acc += total[i];
    }
  }
  __syncthreads();
  if (e < E) {
    seg_count[e] = total[e];
    seg_start[e] = start[e];
    int off = start[e];
    for (int b = 0; b < nblk; ++b) {
      block_offset[static_cast<int64_t>(b) * E + e] = off;
      off += block_counts[static_cast<int64_t>(b) * E + e];
    }
  }
}

// Positions of every selection (stable: token order inside each expert's
// segment), then the bf16 rows: x^ [T, H] for the shared expert and the
// permuted copies xperm [T*K, H] for the routed experts.
__global__ void __launch_bounds__(kPermBlock) scatter_kernel(const float* __restrict__ x, int T, int H, int K, int E,
                                                             const int* __restrict__ ids,
                                                             const int* __restrict__ block_offset,
                                                             int* __restrict__ pos_of, __nv_bfloat16* __restrict__ xhat,
                                                             __nv_bfloat16* __restrict__ xperm) {
  __shared__ int sid[kPermBlock][kMaxTopK];
  __shared__ int wcount[8][kMaxExperts];
  __shared__ int spos[kPermBlock][kMaxTopK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kPermBlock + threadIdx.x;
  for (int i = threadIdx.x; i < 8 * kMaxExperts; i += blockDim.x) (&wcount[0][0])[i] = 0;
  for (int j = 0; j < K; ++j) {
    int e = t < T ? ids[static_cast<int64_t>(t) * K + j] : -1;
    if (e < 0 || e >= E) e = -1;
    sid[threadIdx.x][j] = e;
  }
  __syncthreads();
  for (int j = 0; j < K; ++j) {
    const int e = sid[threadIdx.x][j];
    if (e >= 0) atomicAdd(&wcount[warp][e], 1);
  }
  __syncthreads();
  // Exclusive prefix over warps, per expert.
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int acc = 0;
    for (int w = 0; w < 8; ++w) {
      const int c = wcount[w][e];
      wcount[w][e] = acc;
      acc += c;
    }
  }
  __syncthreads();
  if (t < T) {
    for (int j = 0; j < K; ++j) {
      const int e = sid[threadIdx.x][j];
      if (e < 0) {
        spos[threadIdx.x][j] = -1;
        continue;
      }
      int rank = 0;  // earlier rows of this warp that chose e
      for (int r = warp * 32; r < static_cast<int>(threadIdx.x); ++r)
        for (int q = 0; q < K; ++q) rank += sid[r][q] == e;
      const int p = block_offset[static_cast<int64_t>(blockIdx.x) * E + e] + wcount[warp][e] + rank;
      spos[threadIdx.x][j] = p;
      pos_of[static_cast<int64_t>(t) * K + j] = p;
    }
  }
  __syncthreads();
  // Row copies: the warp streams its 32 rows one by one, 8 floats per lane step.
  for (int r = 0; r < 32; ++r) {
    const int lr = warp * 32 + r;
    const int tr = blockIdx.x * kPermBlock + lr;
    if (tr >= T) break;
    const float* src = x + static_cast<int64_t>(tr) * H;
    for (int c = lane * 8; c < H; c += 32 * 8) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src + c));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src + c + 4));
      uint4 pk;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      pk.z = *reinterpret_cast<uint32_t*>(&h2);
      pk.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(xhat + static_cast<int64_t>(tr) * H + c) = pk;
      for (int j = 0; j < K; ++j) {
        const int p = spos[lr][j];
        if (p >= 0) *reinterpret_cast<uint4*>(xperm + static_cast<int64_t>(p) * H + c) = pk;
      }
    }
  }
}

// y[t, c] = shared[t, c] + sum over t's experts in ascending id of w * yperm[pos, c]
// (+ resid[t, c] in the stack), the reference's addition order
// (src/model/feed_forward.cpp:65-76). One block per row, 8 columns per thread.
__global__ void __launch_bounds__(256) combine_kernel(int T, int H, int K, const int* __restrict__ ids,
                                                      const float* __restrict__ weights,
                                                      const int* __restrict__ pos_of,
                                                      const __nv_bfloat16* __restrict__ yperm,
                                                      const float* shared_out, const float* resid, float* y) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int eid[kMaxTopK], pos[kMaxTopK];
  float w[kMaxTopK];
  for (int j = 0; j < K; ++j) {
    eid[j] = ids[static_cast<int64_t>(t) * K + j];
    pos[j] = pos_of[static_cast<int64_t>(t) * K + j];
    w[j] = weights[static_cast<int64_t>(t) * K + j];
  }
  // Ascending expert id (insertion sort of at most 8).
  for (int a = 1; a < K; ++a)
    for (int b = a; b > 0 && eid[b] < eid[b - 1]; --b) {
      const int te = eid[b], tp = pos[b];
      const float tw = w[b];
      eid[b] = eid[b - 1];
      pos[b] = pos[b - 1];
      w[b] = w[b - 1];
      eid[b - 1] = te;
      pos[b - 1] = tp;
      w[b - 1] = tw;
    }
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float routed[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < K; ++j) {
      if (pos[j] < 0) continue;
      const uint4 pk = __ldg(reinterpret_cast<const uint4*>(yperm + static_cast<int64_t>(pos[j]) * H + c));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        routed[2 * q] = __fadd_rn(routed[2 * q], __fmul_rn(w[j], f.x));
        routed[2 * q + 1] = __fadd_rn(routed[2 * q + 1], __fmul_rn(w[j], f.y));
      }
    }
    const int64_t o = static_cast<int64_t>(t) * H + c;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float sh = shared_out != nullptr ? shared_out[o + q] : 0.0f;
      float out = __fadd_rn(sh, routed[q]);
      if (resid != nullptr) out = __fadd_rn(resid[o + q], out);
      y[o + q] = out;
    }
  }
}

}  // namespace

size_t prefill_scratch_bytes(const PrefillDims& d, bool routed_buffers) {
  PrefillScratch s{};
  carve_prefill_scratch(d, nullptr, &s, routed_buffers);
  return s.bytes;
}

void carve_prefill_scratch(const PrefillDims& d, void* base, PrefillScratch* s, bool routed_buffers) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    off = (off + 255) / 256 * 256;
    char* p = base == nullptr ? nullptr : static_cast<char*>(base) + off;
    off += bytes;
    return p;
  };
  const size_t T = static_cast<size_t>(d.max_rows), K = d.top_k, E = d.experts, H = d.hidden, F = d.ffn,
               S = d.shared_ffn;
  const size_t nblk = (T + kPermBlock - 1) / kPermBlock;
  *s = PrefillScratch{};
  s->block_counts = reinterpret_cast<int*>(take(nblk * E * 4));
  s->block_offset = reinterpret_cast<int*>(take(nblk * E * 4));
  s->pos_of = reinterpret_cast<int*>(take(T * K * 4));
  s->xhat = reinterpret_cast<__nv_bfloat16*>(take(T * H * 2));
  s->act_s = reinterpret_cast<__nv_bfloat16*>(take(T * (S > 0 ? S : 1) * 2));
  s->shared_out = reinterpret_cast<float*>(take(T * H * 4));
  if (routed_buffers) {
    s->seg_count = reinterpret_cast<int*>(take(E * 4));
    s->seg_start = reinterpret_cast<int*>(take(E * 4));
    s->xperm = reinterpret_cast<__nv_bfloat16*>(take(T * K * H * 2));
    s->act = reinterpret_cast<__nv_bfloat16*>(take(T * K * F * 2));
    s->yperm = reinterpret_cast<__nv_bfloat16*>(take(T * K * H * 2));
  }
  s->bytes = off;
}

cudaError_t launch_router_logits_rows(const float* x, int T, int H, const float* router, const float* bias, int E,
                                      float* logits, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const dim3 grid((T + kRouterTokens - 1) / kRouterTokens, (E + kRouterExperts - 1) / kRouterExperts);
  router_logits_rows_kernel<<<grid, 256, 0, stream>>>(x, T, H, router, bias, E, logits);
  return cudaGetLastError();
}

cudaError_t launch_prefill_route(const PrefillCall& c, cudaStream_t stream) {
  const PrefillDims& d = c.dims;
  const PrefillScratch& s = c.scratch;
  const int T = c.rows, H = d.hidden, E = d.experts, K = d.top_k;
  auto mark = [&](int i) { return c.events != nullptr ? cudaEventRecord(c.events[i], stream) : cudaSuccess; };
  if (T <= 0) {
    // An empty batch still publishes empty segments (expert-parallel peers read them).
    cudaError_t st = cudaMemsetAsync(s.seg_count, 0, static_cast<size_t>(E) * sizeof(int), stream);
    return st == cudaSuccess ? cudaMemsetAsync(s.seg_start, 0, static_cast<size_t>(E) * sizeof(int), stream) : st;
  }
  cudaError_t st = launch_router_logits_rows(c.x, T, H, c.router, c.bias, E, c.logits, stream);
  if (st != cudaSuccess || (st = mark(0)) != cudaSuccess) return st;
  topk_rows_i32_kernel<<<(T + 7) / 8, 256, 0, stream>>>(c.logits, T, E, K, d.renormalize, c.ids, c.weights);
  if ((st = cudaGetLastError()) != cudaSuccess || (st = mark(1)) != cudaSuccess) return st;
  const int nblk = (T + kPermBlock - 1) / kPermBlock;
  count_kernel<<<nblk, kPermBlock, 0, stream>>>(c.ids, T, K, E, s.block_counts, c.err);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  scan_kernel<<<1, kMaxExperts, 0, stream>>>(s.block_counts, nblk, E, s.seg_count, s.seg_start, s.block_offset);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  scatter_kernel<<<nblk, kPermBlock, 0, stream>>>(c.x, T, H, K, E, c.ids, s.block_offset, s.pos_of, s.xhat,
                                                  s.xperm);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  return mark(2);
}

GroupedGemm prefill_gate_up_gemm(const PrefillCall& c, bool routed, bool shared) {
  const PrefillDims& d = c.dims;
  const PrefillScratch& s = c.scratch;
  const int T = c.rows, H = d.hidden, E = d.experts, K = d.top_k, F = d.ffn, S = d.shared_ffn;
  GroupedGemm g{};
  g.mode = 0;
  g.experts = routed ? E : 0;
  g.seg_count = s.seg_count;
  g.seg_start = s.seg_start;
  g.a_routed = s.xperm;
  g.a_routed_rows = static_cast<int64_t>(T) * K;
  g.k_routed = H;
  g.b0_routed = c.gate;
  g.b1_routed = c.up;
  g.b_routed_rows = static_cast<int64_t>(E) * F;
  g.b_rows_per_expert = F;
  g.n_cols_routed = F;
  g.out_routed = s.act;
  g.ld_out_routed = F;
  g.shared_rows = shared && S > 0 ? T : 0;
  g.a_shared = s.xhat;
  g.k_shared = H;
  g.b0_shared = c.sgate;
  g.b1_shared = c.sup;
  g.b_shared_rows = S;
  g.n_cols_shared = S > 0 ? S : 128;
  g.out_shared = s.act_s;
  g.ld_out_shared = S;
  g.shared_out_f32 = false;
  g.err = c.err;
  g.blocks = c.sm_count;
  return g;
}

GroupedGemm prefill_down_gemm(const PrefillCall& c, bool routed, bool shared) {
  const PrefillDims& d = c.dims;
  const PrefillScratch& s = c.scratch;
  const int H = d.hidden, E = d.experts, F = d.ffn, S = d.shared_ffn;
  GroupedGemm g = prefill_gate_up_gemm(c, routed, shared);
  g.mode = 1;
  g.a_routed = s.act;
  g.k_routed = F;
  g.b0_routed = c.down;
  g.b1_routed = c.down;
  g.b_routed_rows = static_cast<int64_t>(E) * H;
  g.b_rows_per_expert = H;
  g.n_cols_routed = H;
  g.out_routed = s.yperm;
  g.ld_out_routed = H;
  g.a_shared = s.act_s;
  g.k_shared = S > 0 ? S : 64;
  g.b0_shared = c.sdown;
  g.b1_shared = c.sdown;
  g.b_shared_rows = H;
  g.n_cols_shared = H;
  g.out_shared = s.shared_out;
  g.ld_out_shared = H;
  g.shared_out_f32 = true;
  return g;
}

cudaError_t launch_prefill(const PrefillCall& c, cudaStream_t stream) {
  const PrefillDims& d = c.dims;
  const PrefillScratch& s = c.scratch;
  const int T = c.rows, H = d.hidden, K = d.top_k, S = d.shared_ffn;
  if (T <= 0) return cudaSuccess;
  // Optional per-kernel timing: an event after each stage of the path.
  auto mark = [&](int i) { return c.events != nullptr ? cudaEventRecord(c.events[i], stream) : cudaSuccess; };
  cudaError_t st = launch_prefill_route(c, stream);
  if (st != cudaSuccess) return st;
  if ((st = launch_grouped_gemm(prefill_gate_up_gemm(c, true, true), stream)) != cudaSuccess ||
      (st = mark(3)) != cudaSuccess)
    return st;
  if ((st = launch_grouped_gemm(prefill_down_gemm(c, true, true), stream)) != cudaSuccess ||
      (st = mark(4)) != cudaSuccess)
    return st;
  combine_kernel<<<T, 256, 0, stream>>>(T, H, K, c.ids, c.weights, s.pos_of, s.yperm, S > 0 ? s.shared_out : nullptr,
                                        c.resid, c.y);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  return mark(5);
}

}  // namespace uocr_b200
