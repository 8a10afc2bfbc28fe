// Prefill path (rows > 16): top-k, the token -> expert permutation, and the
// weighted combine. The router logits for many rows are router_rows.cu's; the
// expert GEMMs are the tcgen05 grouped GEMM (tc_gemm.cu).
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
#include "combine.cuh"
#include "route.cuh"

namespace uocr_b200 {
namespace {

constexpr int kPermBlock = 256;     // rows per permutation block (8 warps x 32)

__global__ void __launch_bounds__(256) topk_rows_i32_kernel(const float* __restrict__ logits, int T, int E, int K,
                                                            int renorm, int* ids, float* weights) {
  __shared__ __align__(16) float ebuf[8][kTopkScratch];
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
// segment). A row's rank among the earlier rows of its warp that chose the
// same expert is a population count over a per-warp, per-expert lane mask
// (a row's k ids are distinct, so each lane sets its bit once per expert).
__global__ void __launch_bounds__(kPermBlock) positions_kernel(int T, int K, int E, const int* __restrict__ ids,
                                                               const int* __restrict__ block_offset,
                                                               int* __restrict__ pos_of) {
  __shared__ int wcount[8][kMaxExperts];
  __shared__ unsigned lanes[8][kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kPermBlock + threadIdx.x;
  for (int i = threadIdx.x; i < 8 * kMaxExperts; i += blockDim.x) {
    (&wcount[0][0])[i] = 0;
    (&lanes[0][0])[i] = 0u;
  }
  __syncthreads();
  int sid[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    int e = (j < K && t < T) ? ids[static_cast<int64_t>(t) * K + j] : -1;
    if (e < 0 || e >= E) e = -1;
    sid[j] = e;
    if (e >= 0) {
      atomicAdd(&wcount[warp][e], 1);
      atomicOr(&lanes[warp][e], 1u << lane);
    }
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
  if (t >= T) return;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j >= K) break;
    const int e = sid[j];
    int p = -1;
    if (e >= 0)
      p = block_offset[static_cast<int64_t>(blockIdx.x) * E + e] + wcount[warp][e] +
          __popc(lanes[warp][e] & ((1u << lane) - 1u));
    pos_of[static_cast<int64_t>(t) * K + j] = p;
  }
}

// The bf16 rows: x^ [T, H] for the shared expert and the permuted copies
// xperm [T*K, H] for the routed experts (xperm null: x^ alone — the
// expert-parallel owners pull rows from x^). Grid-stride over (row, 8-column)
// items, two per thread per step with both loads issued first.
__global__ void __launch_bounds__(256) permute_copy_kernel(const float* __restrict__ x, int T, int H, int K,
                                                           const int* __restrict__ pos_of,
                                                           __nv_bfloat16* __restrict__ xhat,
                                                           __nv_bfloat16* __restrict__ xperm) {
  const int cpr = H / 8;  // 8-column items per row
  const int64_t n = static_cast<int64_t>(T) * cpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n; i0 += 2 * stride) {
    float4 v[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n) {
        const float4* src = reinterpret_cast<const float4*>(x + (i / cpr) * H + (i % cpr) * 8);
        v[u][0] = __ldg(src);
        v[u][1] = __ldg(src + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n) continue;
      const int64_t t = i / cpr, c = (i % cpr) * 8;
      uint4 pk;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(v[u][0].x, v[u][0].y), h1 = __floats2bfloat162_rn(v[u][0].z, v[u][0].w);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[u][1].x, v[u][1].y), h3 = __floats2bfloat162_rn(v[u][1].z, v[u][1].w);
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      pk.z = *reinterpret_cast<uint32_t*>(&h2);
      pk.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(xhat + t * H + c) = pk;
      if (xperm != nullptr)
        for (int j = 0; j < K; ++j) {
          const int p = __ldg(pos_of + t * K + j);
          if (p >= 0) *reinterpret_cast<uint4*>(xperm + static_cast<int64_t>(p) * H + c) = pk;
        }
    }
  }
}

// y[t, c] = shared[t, c] + sum over t's experts in ascending id of w * yperm[pos, c]
// (+ resid[t, c] in the stack), the reference's addition order
// (src/model/feed_forward.cpp:65-76). One block per row, 8 columns per thread.
__global__ void __launch_bounds__(256, 3) combine_kernel(int T, int H, int K, const int* __restrict__ ids,
                                                      const float* __restrict__ weights,
                                                      const int* __restrict__ pos_of,
                                                      const __nv_bfloat16* __restrict__ yperm,
                                                      const float* shared_out, const float* resid, float* y) {
  __shared__ CombineList list;
  const int t = blockIdx.x;
  if (t >= T) return;
  const int64_t b = static_cast<int64_t>(t) * K;
  order_selections(
      K, [&](int i) { return ids[b + i]; },
      [&](int j, int, float* w, const __nv_bfloat16** src) {
        *w = weights[b + j];
        const int p = pos_of[b + j];
        *src = p < 0 ? nullptr : yperm + static_cast<int64_t>(p) * H;
      },
      &list);
  const int64_t o = static_cast<int64_t>(t) * H;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
    combine_cols8(list, K, c, shared_out != nullptr ? shared_out + o : nullptr, resid != nullptr ? resid + o : nullptr,
                  y + o);
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
  positions_kernel<<<nblk, kPermBlock, 0, stream>>>(T, K, E, c.ids, s.block_offset, s.pos_of);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  permute_copy_kernel<<<c.sm_count * 8, 256, 0, stream>>>(c.x, T, H, K, s.pos_of, s.xhat, s.xperm);
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
  const int T = c.rows;
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
  if ((st = launch_prefill_combine(c, stream)) != cudaSuccess) return st;
  return mark(5);
}

cudaError_t launch_prefill_combine(const PrefillCall& c, cudaStream_t stream) {
  const PrefillDims& d = c.dims;
  const PrefillScratch& s = c.scratch;
  const int T = c.rows;
  if (T <= 0) return cudaSuccess;
  combine_kernel<<<T, 256, 0, stream>>>(T, d.hidden, d.top_k, c.ids, c.weights, s.pos_of, s.yperm,
                                        d.shared_ffn > 0 ? s.shared_out : nullptr, c.resid, c.y);
  return cudaGetLastError();
}

}  // namespace uocr_b200
