// Router gate logits, and the standalone top-k op.
//
// The logits are computed in fp32 with exactly the reference's summation
// order — eight lane partial sums over i = 8j + lane, a fixed combine tree,
// then the tail and the bias (src/backend/reference/ops.cpp:25-38, :91-109) —
// with every product and sum separately rounded. So the device logits are
// bit-identical to the oracle's, and the selected expert ids differ from the
// reference only where its float exp and CUDA's expf round a near-tie apart.
// Softmax and top-k selection live in route.cuh (each expert-kernel block
// runs them on these logits).
#include <mutex>

#include "moe_kernels.h"
#include "ptx.cuh"
#include "rms_norm.cuh"
#include "route.cuh"

namespace uocr_b200 {
namespace {

constexpr int kStageUnroll = 4;  // float4 loads in flight per thread while staging

// Normalises the T staged x rows (row stride `stride`, 16-byte aligned) in
// place with the gain staged at gs; every thread of the block (8 warps or
// more) calls it.
__device__ void normalize_staged_rows(float* xs, int T, int H, int stride, const float* gs, float eps) {
  __shared__ double s_part[kDecodeMaxRows * kNormWarps];
  __shared__ float s_inv[kDecodeMaxRows];
  rms_inv_rows(
      T, H, eps, [&](int t, int q) { return reinterpret_cast<const float4*>(xs + static_cast<size_t>(t) * stride)[q]; },
      s_part, s_inv);
  const int n4 = H / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gs);
  for (int t = 0; t < T; ++t) {
    float4* r4 = reinterpret_cast<float4*>(xs + static_cast<size_t>(t) * stride);
    const float inv = s_inv[t];
    for (int q = threadIdx.x; q < n4; q += blockDim.x) {
      const float4 v = r4[q], g = g4[q];
      r4[q] = make_float4(rms_apply(v.x, inv, g.x), rms_apply(v.y, inv, g.y), rms_apply(v.z, inv, g.z),
                          rms_apply(v.w, inv, g.w));
    }
  }
  __syncthreads();
}

// One block per expert row of the router: logits[t, e] for every row t of
// the batch, in the reference's dot order. Launched with programmatic
// dependent launch: the router row is staged before waiting for the previous
// grid (which writes x).
__global__ void __launch_bounds__(256) router_logits_kernel(const float* __restrict__ x, int T, int H,
                                                            const float* __restrict__ router,
                                                            const float* __restrict__ bias, int E,
                                                            float* __restrict__ logits, RouteOut ro, RowNorm norm) {
  extern __shared__ float smem[];
  const int e = blockIdx.x;
  const int tid = threadIdx.x;
  const int xstride = H + 8;  // rows 8 floats apart: the four rows a warp reads sit in different banks
  float* ws = smem;
  float* xs = smem + H;
  float* gs = xs + static_cast<size_t>(T) * xstride;  // [H] norm gain (norm.on)
  // 16-byte loads, all of a thread's issued before any is stored: one DRAM
  // round trip for the row instead of one per element step.
  const int h4 = H / 4;
  {
    const float4* src = reinterpret_cast<const float4*>(router + static_cast<int64_t>(e) * H);
    float4 v[kStageUnroll];
    for (int i0 = tid; i0 < h4; i0 += blockDim.x * kStageUnroll) {
#pragma unroll
      for (int u = 0; u < kStageUnroll; ++u)
        if (i0 + u * static_cast<int>(blockDim.x) < h4) v[u] = __ldg(src + i0 + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < kStageUnroll; ++u)
        if (i0 + u * static_cast<int>(blockDim.x) < h4) reinterpret_cast<float4*>(ws)[i0 + u * blockDim.x] = v[u];
    }
    if (norm.on)
      for (int i = tid; i < h4; i += blockDim.x)
        reinterpret_cast<float4*>(gs)[i] = __ldg(reinterpret_cast<const float4*>(norm.gain) + i);
  }
  pdl_wait();  // x is written by the previous grid
  pdl_launch_dependents();
  for (int i0 = tid; i0 < T * h4; i0 += blockDim.x * kStageUnroll) {
    float4 v[kStageUnroll];
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < T * h4) v[u] = __ldcg(reinterpret_cast<const float4*>(x) + i);
    }
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < T * h4) reinterpret_cast<float4*>(xs + (i / h4) * xstride)[i % h4] = v[u];
    }
  }
  __syncthreads();
  if (norm.on) normalize_staged_rows(xs, T, H, xstride, gs, norm.eps);

  const int lane8 = tid & 7;
  const int groups = blockDim.x >> 3;
  const int full = H & ~7;
  for (int t0 = 0; t0 < T; t0 += groups) {
    const int t = t0 + (tid >> 3);
    float acc = 0.0f, tail = 0.0f;
    if (t < T) {
      const float* xr = xs + t * xstride;
      // Sixteen elements of the chain loaded before they are added: the
      // shared-memory latency is paid once per sixteen dependent adds.
      int i = lane8;
      for (; i + 120 < full; i += 128) {
        float xv[16], wv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          xv[u] = xr[i + 8 * u];
          wv[u] = ws[i + 8 * u];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, __fmul_rn(xv[u], wv[u]));
      }
      for (; i < full; i += 8) acc = __fadd_rn(acc, __fmul_rn(xr[i], ws[i]));
      if (lane8 == 0)
        for (int i = full; i < H; ++i) tail = __fadd_rn(tail, __fmul_rn(xr[i], ws[i]));
    }
    float a[8];
    const int base = (tid & 31) & ~7;
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
  if (ro.table == nullptr) return;
  // The last block to finish builds the batch's routing table once, with all
  // of its threads, for the expert kernels to copy.
  __shared__ int s_last;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(ro.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ SmemRoute r;
  route_from_logits(logits, T, E, ro.top_k, ro.renorm, &r, tid, blockDim.x, 1, ro.ids_out, ro.w_out);
  route_to_table(&r, ro.table, tid, blockDim.x);
  if (tid == 0) *ro.ticket = 0;
}

constexpr int kRouterCluster = 8;  // CTAs of the decode router's cluster (portable size)

// The decode router as one 8-CTA thread-block cluster: CTA c stages the router
// rows of experts c, c+8, ... into shared memory (before waiting for the grid
// that writes x), computes their logits for every batch row in the exact dot
// order — into global memory and into CTA 0's shared memory (distributed
// shared memory) — and after a cluster barrier (release/acquire: the other
// CTAs' logits are visible) CTA 0 builds the routing table from its own shared
// memory. No global ticket, no last-block handshake.
__global__ void __launch_bounds__(256) router_cluster_kernel(const float* __restrict__ x, int T, int H,
                                                             const float* __restrict__ router,
                                                             const float* __restrict__ bias, int E,
                                                             float* __restrict__ logits, RouteOut ro,
                                                             RowNorm norm) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = blockIdx.x;
  const int per = (E + kRouterCluster - 1) / kRouterCluster;  // expert rows per CTA (layout stride)
  const int ne = cta < E ? (E - cta + kRouterCluster - 1) / kRouterCluster : 0;
  // Rows 8 floats longer than H: the router rows (and the x rows) that the
  // lanes of a warp read at the same offset fall in different banks.
  const int xstride = H + 8;
  float* ws = smem;                                       // [per][H + 8]
  float* xs = smem + static_cast<size_t>(per) * xstride;  // [T][H + 8]
  float* gs = xs + static_cast<size_t>(T) * xstride;     // [H] norm gain (norm.on)
  // The batch's logits [T, E], gathered in CTA 0's copy of this array.
  __shared__ __align__(16) float cl_logits[kDecodeMaxRows * kMaxExperts];
  // Bulk copies (TMA engine, one thread issues them all): the CTA's router
  // rows before the wait for x — one round trip for all of them — then the x rows.
  __shared__ __align__(8) uint64_t bars[2];
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    const uint32_t rows_bytes = static_cast<uint32_t>(ne + (norm.on ? 1 : 0)) * H * 4;
    if (rows_bytes > 0) {
      mbar_arrive_expect_tx(&bars[0], rows_bytes);
      for (int i = 0; i < ne; ++i)
        bulk_g2s(ws + static_cast<size_t>(i) * xstride, router + static_cast<int64_t>(cta + kRouterCluster * i) * H,
                 static_cast<uint32_t>(H) * 4, &bars[0]);
      if (norm.on) bulk_g2s(gs, norm.gain, static_cast<uint32_t>(H) * 4, &bars[0]);
    } else {
      mbar_arrive(&bars[0]);
    }
  }
  // Every CTA of the cluster has started before any writes another's shared
  // memory: this arrive pairs with the wait before the chains.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  pdl_wait();  // x is written by the previous grid
  pdl_launch_dependents();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[1], static_cast<uint32_t>(T) * H * 4);
    for (int t = 0; t < T; ++t)
      bulk_g2s(xs + static_cast<size_t>(t) * xstride, x + static_cast<int64_t>(t) * H, static_cast<uint32_t>(H) * 4,
               &bars[1]);
  }
  __syncthreads();  // the barriers are initialised before anyone waits on them
  const bool ok = mbar_wait(&bars[0], 0) & mbar_wait(&bars[1], 0);
  if (!ok && tid == 0 && ro.err != nullptr) raise_error(ro.err, kDevWaitTimeout, 40, cta, 0);
  if (norm.on) normalize_staged_rows(xs, T, H, xstride, gs, norm.eps);
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // This thread's address of CTA 0's cl_logits.
  uint32_t cl0;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(cl0) : "r"(smem_addr(cl_logits)));
  // Chains (expert i, row t, lane l8): the eight lanes of a chain group are
  // eight consecutive threads of one warp.
  const int n_items = ne * T * 8;
  const int full = H & ~7;
  for (int b = warp * 32; b < n_items; b += blockDim.x) {
    const int item = b + lane;
    const bool valid = item < n_items;
    const int i = valid ? item / (T * 8) : 0, t = valid ? (item / 8) % T : 0, l8 = item & 7;
    const float* xr = xs + t * xstride;
    const float* wr = ws + static_cast<size_t>(i) * xstride;
    float acc = 0.0f, tail = 0.0f;
    if (valid) {
      int k = l8;
      for (; k + 120 < full; k += 128) {
        float xv[16], wv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          xv[u] = xr[k + 8 * u];
          wv[u] = wr[k + 8 * u];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, __fmul_rn(xv[u], wv[u]));
      }
      for (; k < full; k += 8) acc = __fadd_rn(acc, __fmul_rn(xr[k], wr[k]));
      if (l8 == 0)
        for (int q = full; q < H; ++q) tail = __fadd_rn(tail, __fmul_rn(xr[q], wr[q]));
    }
    float a[8];
    const int gbase = lane & ~7;
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = __shfl_sync(0xffffffffu, acc, gbase + q);
    if (valid && l8 == 0) {
      const int e = cta + kRouterCluster * i;
      const float lo = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
      const float hi = __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7]));
      float sum = __fadd_rn(__fadd_rn(lo, hi), tail);
      if (bias != nullptr) sum = __fadd_rn(sum, bias[e]);
      logits[static_cast<int64_t>(t) * E + e] = sum;
      if (ro.table != nullptr)
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cl0 + static_cast<uint32_t>(t * E + e) * 4u), "f"(sum)
                     : "memory");
    }
  }
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (cta != 0 || ro.table == nullptr) return;
  __shared__ SmemRoute r;
  route_from_logits<true>(cl_logits, T, E, ro.top_k, ro.renorm, &r, tid, blockDim.x, 1, ro.ids_out, ro.w_out);
  route_to_table(&r, ro.table, tid, blockDim.x);
}

size_t router_cluster_smem(int T, int H, int E, bool norm) {
  const size_t per = static_cast<size_t>((E + kRouterCluster - 1) / kRouterCluster);
  return ((per + static_cast<size_t>(T)) * (H + 8) + (norm ? H : 0)) * sizeof(float);
}

size_t router_fallback_smem(int T, int H, bool norm) {
  return (static_cast<size_t>(H) + static_cast<size_t>(T) * (H + 8) + (norm ? H : 0)) * sizeof(float);
}

// Standalone softmax/top-k over logits rows: one warp per row (the op-level
// mirror of expert_topk, int64 ids like the reference).
__global__ void __launch_bounds__(256) topk_rows_kernel(const float* __restrict__ logits, int64_t rows, int E,
                                                        int K, int renorm, int64_t* ids, float* weights) {
  __shared__ __align__(16) float ebuf[8][kTopkScratch];
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
    float w = weights[j];
    if (id < 0 || id >= E) {
      // Recorded in the op-level error word (uocr_ops_check reports it);
      // the slot reads expert 0's rows with weight 0, so nothing outside
      // the stacks is touched and the bad id adds nothing to the output.
      raise_error(err, kDevBadIndex, 2, j, static_cast<int>(id));
      id = 0;
      w = 0.0f;
    }
    route->active_expert[j] = static_cast<int>(id);
    route->tok_count[j] = 1;
    route->slot_base[j] = j;
    route->slot_tok[j] = 0;
    route->slot_w[j] = w;
  }
}

}  // namespace

size_t g_cluster_dyn_limit[kMaxDevices] = {};

cudaError_t prepare_router_decode() {
  static bool raised[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < kMaxDevices && !raised[dev]) {
    st = allow_max_dynamic_smem(router_logits_kernel);
    if (st == cudaSuccess) st = allow_max_dynamic_smem(router_cluster_kernel);
    if (st != cudaSuccess) return st;
    cudaFuncAttributes a{};
    int optin = 0;
    if ((st = cudaFuncGetAttributes(&a, router_cluster_kernel)) != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return st;
    g_cluster_dyn_limit[dev] = static_cast<size_t>(optin) - a.sharedSizeBytes;
    raised[dev] = true;
  }
  return cudaSuccess;
}

cudaError_t launch_router_logits(const float* x, int T, int H, const float* router, const float* bias, int E,
                                 float* logits, cudaStream_t stream, bool pdl, const RouteOut* route, RowNorm norm) {
  RouteOut ro = route != nullptr ? *route : RouteOut{nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if ((st = prepare_router_decode()) != cudaSuccess) return st;
  const size_t csmem = router_cluster_smem(T, H, E, norm.on != 0);
  if (route != nullptr && T <= kDecodeMaxRows && E <= kMaxExperts && dev < kMaxDevices &&
      csmem <= g_cluster_dyn_limit[dev]) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kRouterCluster);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = csmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kRouterCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    void* args[] = {&x, &T, &H, &router, &bias, &E, &logits, &ro, &norm};
    return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(router_cluster_kernel), args);
  }
  const size_t smem = router_fallback_smem(T, H, norm.on != 0);
  void* args[] = {&x, &T, &H, &router, &bias, &E, &logits, &ro, &norm};
  return launch_maybe_pdl(reinterpret_cast<const void*>(router_logits_kernel), dim3(E), dim3(256), smem, stream, args,
                          pdl);
}

size_t router_decode_smem(int T, int H, int E, bool norm) {
  return router_fallback_smem(T, H, norm);
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

// The op-level mirrors' error word: one per device, in module memory (zero
// at load), never cleared by a call, so the first bad index since the last
// uocr_ops_check stays recorded until that check reads and clears it.
static __device__ ErrorWord g_ops_error;

cudaError_t ops_error_word(ErrorWord** out) {
  static std::mutex mu;
  static ErrorWord* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if ((st = cudaGetSymbolAddress(&p, g_ops_error)) != cudaSuccess) return st;
    addr[dev] = static_cast<ErrorWord*>(p);
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace uocr_b200
