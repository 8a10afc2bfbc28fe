// Router gate, softmax and top-k selection.
//
// The logits are computed in fp32 with exactly the reference's summation
// order — eight lane partial sums over i = 8j + lane, a fixed combine tree,
// then the tail and the bias (src/backend/reference/ops.cpp:25-38, :91-109) —
// with every product and sum separately rounded. So the device logits are
// bit-identical to the oracle's, and the selected expert ids differ from the
// reference only where its float exp and CUDA's expf round a near-tie apart.
// Selection follows src/model/feed_forward.cpp:43-48 and
// src/backend/cuda/ops.cu:598-645: softmax with a double-precision total in
// index order, then k rounds of "best remaining", lower id on a tie.
#include "moe_kernels.h"

namespace uocr_b200 {
namespace {

// Softmax + top-k of one row by one warp. `ebuf` is per-warp shared scratch
// of kMaxExperts floats. Lane 0 returns the results through ids/weights.
template <typename IdT>
__device__ void softmax_topk_warp(const float* logits, int E, int K, int renorm, float* ebuf, IdT* ids,
                                  float* weights) {
  const int lane = threadIdx.x & 31;
  float v[4];
  float peak = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __ldcg(logits + e) : -INFINITY;
    peak = fmaxf(peak, v[i]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
  if (peak == -INFINITY) {
    // A fully masked row softmaxes to zeros (ops.cpp:175-177).
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = lane + 32 * i < E ? 0.0f : -INFINITY;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        v[i] = expf(v[i] - peak);
        ebuf[e] = v[i];
      }
    }
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      double total = 0.0;
      for (int e = 0; e < E; ++e) total += static_cast<double>(ebuf[e]);
      inv = static_cast<float>(1.0 / total);
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < E) v[i] = v[i] * inv;
    __syncwarp();
  }
  float sum = 0.0f;
  float chosen[kMaxTopK];
  int chosen_id[kMaxTopK];
  for (int j = 0; j < K; ++j) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < best_e))) {
        best = v[i];
        best_e = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    // Remove the winner from its owner lane (a removed slot can never win again).
    if ((best_e & 31) == lane) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i == (best_e >> 5)) v[i] = -INFINITY;
    }
    chosen[j] = best;
    chosen_id[j] = best_e;
    sum += best;
  }
  if (lane == 0) {
    for (int j = 0; j < K; ++j) {
      ids[j] = static_cast<IdT>(chosen_id[j]);
      weights[j] = renorm ? chosen[j] / sum : chosen[j];
    }
  }
}

// One block per expert row of the router: logits[t, e] for every row t of
// the decode batch, in the reference's dot order. The last block to finish
// runs softmax/top-k for every row and writes the decode routing table.
__global__ void __launch_bounds__(256) router_decode_kernel(const float* __restrict__ x, int T, int H,
                                                            const float* __restrict__ router,
                                                            const float* __restrict__ bias, int E, int K,
                                                            int renorm, float* logits, int* ids, float* weights,
                                                            DecodeRoute* route, unsigned* counter,
                                                            ErrorWord* err) {
  extern __shared__ float smem[];
  const int e = blockIdx.x;
  const int xstride = H + 8;  // rows 8 floats apart: the four rows a warp reads sit in different banks
  float* ws = smem;
  float* xs = smem + H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) ws[i] = router[static_cast<int64_t>(e) * H + i];
  for (int i = threadIdx.x; i < T * H; i += blockDim.x) xs[(i / H) * xstride + (i % H)] = x[i];
  __syncthreads();

  const int lane8 = threadIdx.x & 7;
  const int groups = blockDim.x >> 3;
  const int full = H & ~7;
  for (int t0 = 0; t0 < T; t0 += groups) {
    const int t = t0 + (threadIdx.x >> 3);
    float acc = 0.0f, tail = 0.0f;
    if (t < T) {
      const float* xr = xs + t * xstride;
#pragma unroll 8
      for (int i = lane8; i < full; i += 8) acc = __fadd_rn(acc, __fmul_rn(xr[i], ws[i]));
      if (lane8 == 0)
        for (int i = full; i < H; ++i) tail = __fadd_rn(tail, __fmul_rn(xr[i], ws[i]));
    }
    float a[8];
    const int base = (threadIdx.x & 31) & ~7;
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = __shfl_sync(0xffffffffu, acc, base + q);
    if (t < T && lane8 == 0) {
      const float lo = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
      const float hi = __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7]));
      float s = __fadd_rn(__fadd_rn(lo, hi), tail);
      if (bias != nullptr) s = __fadd_rn(s, bias[e]);
      logits[static_cast<int64_t>(t) * E + e] = s;
    }
  }

  __shared__ bool is_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  __shared__ float ebuf[8][kMaxExperts];
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  for (int t = warp; t < T; t += nwarps)
    softmax_topk_warp<int>(logits + static_cast<int64_t>(t) * E, E, K, renorm, ebuf[warp], ids + t * K,
                           weights + t * K);
  __threadfence();
  __syncthreads();

  if (threadIdx.x == 0) {
    // Experts in ascending id order, each with its rows in row order: the
    // order the reference adds routed contributions (feed_forward.cpp:66-75).
    __shared__ int slot_of[kMaxExperts];
    for (int i = 0; i < E; ++i) slot_of[i] = -1;
    for (int i = 0; i < T * K; ++i) {
      const int id = __ldcg(ids + i);
      if (id < 0 || id >= E) {
        raise_error(err, kDevBadIndex, 1, i, id);
        continue;
      }
      slot_of[id] = 0;
    }
    int U = 0;
    for (int i = 0; i < E; ++i)
      if (slot_of[i] == 0) {
        route->active_expert[U] = i;
        route->tok_count[U] = 0;
        slot_of[i] = U++;
      }
    route->active_count = U;
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < K; ++j) {
        const int id = __ldcg(ids + t * K + j);
        if (id < 0 || id >= E) continue;
        const int u = slot_of[id];
        const int s = route->tok_count[u]++;
        route->tok_index[u][s] = t;
        route->tok_weight[u][s] = __ldcg(weights + t * K + j);
      }
    int base = 0;
    for (int u = 0; u < U; ++u) {
      route->slot_base[u] = base;
      base += route->tok_count[u];
    }
    route->slot_total = base;
    __threadfence();
    *counter = 0u;  // ready for the next launch (and graph replays)
  }
}

// Standalone softmax/top-k over logits rows: one warp per row (the op-level
// mirror of expert_topk, int64 ids like the reference).
__global__ void __launch_bounds__(256) topk_rows_kernel(const float* __restrict__ logits, int64_t rows, int E,
                                                        int K, int renorm, int64_t* ids, float* weights) {
  __shared__ float ebuf[8][kMaxExperts];
  const int warp = threadIdx.x >> 5;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (r >= rows) return;
  softmax_topk_warp<int64_t>(logits + r * E, E, K, renorm, ebuf[warp], ids + r * K, weights + r * K);
}

// Routing table for the expert_ffn_one mirror: the k ids of one row in rank
// order (the reference sums expert contributions in j order, gemv_ops.cu:204).
__global__ void route_from_ids_kernel(const int64_t* ids, const float* weights, int K, int E, DecodeRoute* route,
                                      ErrorWord* err) {
  if (threadIdx.x != 0) return;
  route->active_count = K;
  route->slot_total = K;
  for (int j = 0; j < K; ++j) {
    int64_t id = ids[j];
    if (id < 0 || id >= E) {
      raise_error(err, kDevBadIndex, 2, j, static_cast<int>(id));
      id = 0;
    }
    route->active_expert[j] = static_cast<int>(id);
    route->tok_count[j] = 1;
    route->slot_base[j] = j;
    route->tok_index[j][0] = 0;
    route->tok_weight[j][0] = weights[j];
  }
}

}  // namespace

cudaError_t prepare_router_decode() {
  static bool raised[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < kMaxDevices && !raised[dev]) {
    st = allow_max_dynamic_smem(router_decode_kernel);
    if (st != cudaSuccess) return st;
    raised[dev] = true;
  }
  return cudaSuccess;
}

cudaError_t launch_router_decode(const float* x, int T, int H, const float* router, const float* bias, int E, int K,
                                 int renorm, float* logits, int* ids, float* weights, DecodeRoute* route,
                                 unsigned* counter, ErrorWord* err, cudaStream_t stream) {
  const size_t smem = (static_cast<size_t>(H) + static_cast<size_t>(T) * (H + 8)) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t st = prepare_router_decode();
    if (st != cudaSuccess) return st;
  }
  router_decode_kernel<<<E, 256, smem, stream>>>(x, T, H, router, bias, E, K, renorm, logits, ids, weights, route,
                                                 counter, err);
  return cudaGetLastError();
}

cudaError_t launch_topk_rows(const float* logits, int64_t rows, int E, int K, int renorm, int64_t* ids,
                             float* weights, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  topk_rows_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(logits, rows, E, K, renorm, ids,
                                                                              weights);
  return cudaGetLastError();
}

cudaError_t launch_route_from_ids(const int64_t* ids, const float* weights, int K, int E, DecodeRoute* route,
                                  ErrorWord* err, cudaStream_t stream) {
  route_from_ids_kernel<<<1, 32, 0, stream>>>(ids, weights, K, E, route, err);
  return cudaGetLastError();
}

}  // namespace uocr_b200
