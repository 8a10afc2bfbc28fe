// The page decoder around the MoE: attention, the final norm with lm_head and
// greedy selection, and the prefill's row kernels.
//
// What the reference computes (src/model/cuda/cuda_decode_step.cpp:47-70,
// src/backend/cuda/decode_ops.cu:112-200, src/runtime/generator.cpp:41-84):
// per layer h = rms_norm(x); x += o(attend(rope(q h), rope(k h), v h));
// x += moe(rms_norm(x)); then logits = lm_head(rms_norm(x)) and the greedy
// token. The reference runs one kernel per operation over fp32 activations
// and an fp32 KV cache, with multi-head attention. Here a decode layer is
// three kernels before the MoE — norm + q/k/v GEMV + RoPE + cache append in
// one weight stream, split-key GQA attention, and the output GEMV that first
// merges the splits and ends with the residual add —
// and the lm_head GEMV carries the greedy argmax. Weights stream once with
// 128-bit loads (bf16, or int8 with per-row scales converted in the load);
// the KV cache is bf16, head-major ([kv][pos][128]), so a split reads
// contiguous keys. Every length-dependent value comes from DecState in device
// memory, so one captured decode step replays for every position.
#include <climits>

#include "decode_fmt.cuh"
#include "decoder.h"
#include "moe_kernels.h"
#include "ptx.cuh"
#include "rms_norm.cuh"

namespace uocr_b200 {
namespace {

constexpr int kGemvThreads = 512;  // 16 warps, one block per SM
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kCpl = 8;            // 16-byte chunks of a row a lane keeps in flight
constexpr int kHalf = kDecHeadDim / 2;
constexpr int kPartStride = kDecHeadDim + 2;  // [max, sum, acc[128]] per (head, split)

// Where element e of a GEMV input row sits in the conflict-free layout the
// chunk dot products read: quad Q = e / 4 of chunk Q / kQuads goes to
// quad slot (Q % kQuads) * qs + Q / kQuads (qs = chunks per row).
template <typename Rows>
__device__ __forceinline__ int quad_slot(int e, int qs) {
  using F = Fmt<Rows>;
  const int Q = e >> 2;
  return (((Q % F::kQuads) * qs + Q / F::kQuads) << 2) + (e & 3);
}

// Two weight rows against the staged input: all of a row's chunks in a batch
// (kCpl per lane, 16 bytes each) are loaded before the first product, both
// rows at once. load_rows2 issues a batch; finish_rows2 takes the first batch
// already loaded (a warp issues it before waiting for the previous kernel,
// since weights do not depend on it), loads any further batches and reduces.
template <typename Rows>
__device__ __forceinline__ void load_rows2(const Rows& w, int64_t r0, int64_t r1, int base, int nchunks, int lane,
                                           uint4 (&u0)[kCpl], uint4 (&u1)[kCpl]) {
  using F = Fmt<Rows>;
  const uint4* p0 = F::row(w, r0);
  const uint4* p1 = F::row(w, r1);
#pragma unroll
  for (int u = 0; u < kCpl; ++u) {
    const int c = base + lane + 32 * u;
    if (c < nchunks) {
      u0[u] = ld_stream(p0 + c);
      u1[u] = ld_stream(p1 + c);
    } else {
      u0[u] = make_uint4(0, 0, 0, 0);
      u1[u] = u0[u];
    }
  }
}

template <typename Rows>
__device__ __forceinline__ void finish_rows2(const Rows& w, int64_t r0, int64_t r1, int nchunks, const float4* xs4,
                                             int qs, int lane, uint4 (&u0)[kCpl], uint4 (&u1)[kCpl], float& d0,
                                             float& d1) {
  using F = Fmt<Rows>;
  float a0 = 0.0f, a1 = 0.0f;
  for (int base = 0; base < nchunks; base += 32 * kCpl) {
    if (base > 0) load_rows2(w, r0, r1, base, nchunks, lane, u0, u1);
#pragma unroll
    for (int u = 0; u < kCpl; ++u) {
      const int c = base + lane + 32 * u;
      if (c < nchunks) {
        a0 += F::dot_xq(u0[u], xs4 + c, qs);
        a1 += F::dot_xq(u1[u], xs4 + c, qs);
      }
    }
  }
  d0 = warp_sum(a0) * F::scale(w, r0);
  d1 = warp_sum(a1) * F::scale(w, r1);
}

// RMSNorm(row) * gain rounded to bf16, into the quad layout at xs (the raw
// row is in xr). Every thread of the block calls it; it ends with a barrier.
template <typename Rows>
__device__ __forceinline__ void stage_normed(const float* xr, int H, float eps, const float* gain, float* xs,
                                             double* part, float* inv) {
  rms_inv_rows(1, H, eps, [&](int, int q) { return reinterpret_cast<const float4*>(xr)[q]; }, part, inv);
  const int qs = H / Fmt<Rows>::kPerChunk;
  const float iv = inv[0];
  for (int e4 = threadIdx.x; e4 < H / 4; e4 += blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(xr)[e4];
    const float4 gn = gain != nullptr ? __ldg(reinterpret_cast<const float4*>(gain) + e4)
                                      : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    xs[quad_slot<Rows>(4 * e4, qs)] = bf16_round(rms_apply(v.x, iv, gn.x));
    xs[quad_slot<Rows>(4 * e4 + 1, qs)] = bf16_round(rms_apply(v.y, iv, gn.y));
    xs[quad_slot<Rows>(4 * e4 + 2, qs)] = bf16_round(rms_apply(v.z, iv, gn.z));
    xs[quad_slot<Rows>(4 * e4 + 3, qs)] = bf16_round(rms_apply(v.w, iv, gn.w));
  }
  __syncthreads();
}

// (a, b) -> (a cos - b sin, b cos + a sin), each product and sum rounded on
// its own as PageRope::apply writes it (src/model/page_rope.cpp:49-53).
__device__ __forceinline__ void rotate(float a, float b, float angle, float& o0, float& o1) {
  const float c = cosf(angle), s = sinf(angle);
  o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  o1 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

template <typename Rows>
__global__ void __launch_bounds__(kGemvThreads, 1)
    dec_qkv_kernel(DecShape s, float* x, const __nv_bfloat16* __restrict__ embed, const float* __restrict__ norm,
                   Rows w, const float* __restrict__ inv_freq, const DecState* st, float* q_out,
                   __nv_bfloat16* kc, __nv_bfloat16* vc) {
  extern __shared__ __align__(16) float dsm[];
  float* xr = dsm;
  float* xs = dsm + s.H;
  __shared__ double part[kNormWarps];
  __shared__ float inv[1];
  const int H = s.H;
  const int qs = H / Fmt<Rows>::kPerChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jobs = (s.heads + 2 * s.kv) * kHalf;
  int j = blockIdx.x * kGemvWarps + warp;
  uint4 u0[kCpl], u1[kCpl];
  if (j < jobs) {
    const int64_t r0 = static_cast<int64_t>(j / kHalf) * kDecHeadDim + j % kHalf;
    load_rows2(w, r0, r0 + kHalf, 0, qs, lane, u0, u1);
  }
  pdl_wait();
  pdl_launch_dependents();  // the attention may start staging the cache's earlier rows
  const int pos = st->pos;
  if (embed != nullptr) {
    const uint2* row = reinterpret_cast<const uint2*>(embed + static_cast<int64_t>(st->token) * H);
    for (int e4 = threadIdx.x; e4 < H / 4; e4 += blockDim.x) {
      const uint2 b = __ldg(row + e4);
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.x));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.y));
      reinterpret_cast<float4*>(xr)[e4] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
  } else {
    for (int e4 = threadIdx.x; e4 < H / 4; e4 += blockDim.x)
      reinterpret_cast<float4*>(xr)[e4] = __ldcg(reinterpret_cast<const float4*>(x) + e4);
  }
  __syncthreads();
  if (embed != nullptr && blockIdx.x == 0)
    for (int e4 = threadIdx.x; e4 < H / 4; e4 += blockDim.x)
      reinterpret_cast<float4*>(x)[e4] = reinterpret_cast<const float4*>(xr)[e4];
  stage_normed<Rows>(xr, H, s.eps, norm, xs, part, inv);
  for (bool first = true; j < jobs; j += gridDim.x * kGemvWarps, first = false) {
    const int hh = j / kHalf, i = j % kHalf;
    const int64_t r0 = static_cast<int64_t>(hh) * kDecHeadDim + i, r1 = r0 + kHalf;
    if (!first) load_rows2(w, r0, r1, 0, qs, lane, u0, u1);
    float d0, d1;
    finish_rows2(w, r0, r1, qs, reinterpret_cast<const float4*>(xs), qs, lane, u0, u1, d0, d1);
    if (lane != 0) continue;
    if (hh < s.heads + s.kv) {
      float o0, o1;
      rotate(d0, d1, __fmul_rn(static_cast<float>(pos), inv_freq[i]), o0, o1);
      if (hh < s.heads) {
        q_out[r0] = bf16_round(o0);
        q_out[r1] = bf16_round(o1);
      } else {
        const int64_t base = (static_cast<int64_t>(hh - s.heads) * s.max_pos + pos) * kDecHeadDim;
        kc[base + i] = __float2bfloat16_rn(o0);
        kc[base + i + kHalf] = __float2bfloat16_rn(o1);
      }
    } else {
      const int64_t base = (static_cast<int64_t>(hh - s.heads - s.kv) * s.max_pos + pos) * kDecHeadDim;
      vc[base + i] = __float2bfloat16_rn(d0);
      vc[base + i + kHalf] = __float2bfloat16_rn(d1);
    }
  }
}


constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kKeyGroups = 8;  // groups of four keys a warp scores at once (32 keys in flight)

__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The cluster's splits merged through distributed shared memory, after every
// block of the cluster wrote its hmax[G], hsum[G] (max and exp sum per head)
// and accs[G][128] (p . V with p = exp(s - hmax)): this block takes dims
// [split * D, split * D + D) of every head (D = 128 / splits), tpi threads per
// (head, dim) item sharing the splits; weights exp(m_s - m), then the
// weighted sum over the weighted exp-sum total, rounded to bf16. Every thread
// of the block calls it.
template <int G>
__device__ __forceinline__ void cluster_merge(const float* hmax, const float* hsum, const float* accs, int split,
                                              int splits, int qh0, float* merged) {
  cluster_sync_all();  // every split's hmax, hsum and accs are written
  const int D = kDecHeadDim / splits;
  const int items = G * D;
  const int tpi = kAttnThreads / items;  // a power of two, 2..32
  const int item = threadIdx.x / tpi, li = threadIdx.x % tpi;
  const int a = item / D, d = split * D + item % D;
  float m = -INFINITY;
  for (int r = li; r < splits; r += tpi) m = fmaxf(m, ld_cluster(cluster_addr(&hmax[a], r)));
  for (int off = tpi / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float tot = 0.0f, o = 0.0f;
  for (int r = li; r < splits; r += tpi) {
    const float ms = ld_cluster(cluster_addr(&hmax[a], r));
    if (ms == -INFINITY) continue;
    const float w = expf(ms - m);
    tot = fmaf(w, ld_cluster(cluster_addr(&hsum[a], r)), tot);
    o = fmaf(w, ld_cluster(cluster_addr(accs + a * kDecHeadDim + d, r)), o);
  }
  for (int off = tpi / 2; off > 0; off >>= 1) {
    tot += __shfl_xor_sync(0xffffffffu, tot, off);
    o += __shfl_xor_sync(0xffffffffu, o, off);
  }
  if (li == 0) merged[(qh0 + a) * kDecHeadDim + d] = bf16_round(o / tot);
  cluster_sync_all();  // no block leaves while others read its shared memory
}

// Split-key attention, one thread-block cluster per key/value head: block
// (g, split) takes a contiguous share of keys 0..pos for the G query heads
// that read head g (one cluster per query head, 4x the blocks, measured
// slower: 0.89 against 0.53 ms of attention per 24-layer step). Its V rows go to shared memory by cp.async (when they
// fit; else phase 3 reads them from global memory) while the scores are
// formed — q in registers, 8 lanes per key (16 dims each), 32 keys in flight
// per warp, the partial dots of all keys and heads first and then their lane
// reductions, so the shuffles pipeline. Then the split's max and exp sum per
// head, p . V with the keys spread over the warps (four dims of every head per
// lane), summed across warps. After a cluster barrier each block merges a
// slice of the dims over all the cluster's splits through distributed shared
// memory (weights exp(m_s - m), then the weighted sum over the exp-sum total)
// and writes merged rows (bf16 values, the output projection's input).
template <int G>
__global__ void __launch_bounds__(kAttnThreads) dec_attn_kernel(DecShape s, const float* __restrict__ q,
                                                                const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                                                                const DecState* st, float* merged, int cap,
                                                                int v_smem, float scale) {
  extern __shared__ __align__(16) unsigned char sraw[];
  const int capr = (cap + 3) & ~3;
  float* sc = reinterpret_cast<float*>(sraw);        // [G][capr] scores, then exp values
  float* red = sc + G * capr;                        // [warps][G * 128]
  float* accs = red + kAttnWarps * G * kDecHeadDim;  // [G][128] this split's p . V
  __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(accs + G * kDecHeadDim);  // [cap][128] when v_smem
  __shared__ float hmax[G], hsum[G];
  pdl_wait();
  pdl_launch_dependents();
  const int qh0 = blockIdx.x * G, split = blockIdx.y, splits = gridDim.y;
  const int g = qh0 / (s.heads / s.kv);  // the key/value head these query heads read
  const int keys = st->pos + 1;
  const int chunk = (keys + splits - 1) / splits;
  const int first = split * chunk;
  const int n = max(0, min(keys, first + chunk) - first);
  const __nv_bfloat16* kh = kc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  const __nv_bfloat16* vh = vc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  if (v_smem)
    for (int c = threadIdx.x; c < n * (kDecHeadDim / 8); c += kAttnThreads) cp_async16(vs + c * 8, vh + c * 8);
  cp_async_commit();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane >> 3, sl = lane & 7;  // key of a group of four, lane within the key
  float qr[G][16];
#pragma unroll
  for (int a = 0; a < G; ++a) {
    const float4* qp = reinterpret_cast<const float4*>(q + (qh0 + a) * kDecHeadDim + sl * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldcg(qp + i);
      qr[a][4 * i] = v.x;
      qr[a][4 * i + 1] = v.y;
      qr[a][4 * i + 2] = v.z;
      qr[a][4 * i + 3] = v.w;
    }
  }
  for (int j0 = warp * 4 * kKeyGroups; j0 < n; j0 += kAttnWarps * 4 * kKeyGroups) {
    uint4 kk[kKeyGroups][2];
#pragma unroll
    for (int u = 0; u < kKeyGroups; ++u) {
      const int jj = j0 + 4 * u + sub;
      if (jj < n) {
        const uint4* p = reinterpret_cast<const uint4*>(kh + static_cast<int64_t>(jj) * kDecHeadDim + sl * 16);
        kk[u][0] = __ldcg(p);
        kk[u][1] = __ldcg(p + 1);
      } else {
        kk[u][0] = make_uint4(0, 0, 0, 0);
        kk[u][1] = kk[u][0];
      }
    }
    float pd[kKeyGroups][G];
#pragma unroll
    for (int u = 0; u < kKeyGroups; ++u) {
      float kf[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&kk[u][h]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(b[i]);
          kf[8 * h + 2 * i] = f.x;
          kf[8 * h + 2 * i + 1] = f.y;
        }
      }
#pragma unroll
      for (int a = 0; a < G; ++a) {
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          d0 = fmaf(qr[a][i], kf[i], d0);
          d1 = fmaf(qr[a][i + 1], kf[i + 1], d1);
        }
        pd[u][a] = d0 + d1;
      }
    }
#pragma unroll
    for (int off = 4; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < kKeyGroups; ++u)
#pragma unroll
        for (int a = 0; a < G; ++a) pd[u][a] += __shfl_xor_sync(0xffffffffu, pd[u][a], off);
    if (sl == 0) {
#pragma unroll
      for (int u = 0; u < kKeyGroups; ++u) {
        const int jj = j0 + 4 * u + sub;
        if (jj < n)
#pragma unroll
          for (int a = 0; a < G; ++a) sc[a * capr + jj] = pd[u][a] * scale;
      }
    }
  }
  __syncthreads();
  if (warp < G) {  // warp a: head a's max and exp sum over the split
    float* row = sc + warp * capr;
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, row[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(row[j] - m);
      row[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      hmax[warp] = m;
      hsum[warp] = sum;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  float acc[G][4];
#pragma unroll
  for (int a = 0; a < G; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.0f;
  const __nv_bfloat16* vsrc = v_smem ? vs : vh;
#pragma unroll 4
  for (int j = warp; j < n; j += kAttnWarps) {
    const uint2 v = *reinterpret_cast<const uint2*>(vsrc + static_cast<int64_t>(j) * kDecHeadDim + lane * 4);
    const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
    const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
#pragma unroll
    for (int a = 0; a < G; ++a) {
      const float p = sc[a * capr + j];
      acc[a][0] = fmaf(p, v01.x, acc[a][0]);
      acc[a][1] = fmaf(p, v01.y, acc[a][1]);
      acc[a][2] = fmaf(p, v23.x, acc[a][2]);
      acc[a][3] = fmaf(p, v23.y, acc[a][3]);
    }
  }
#pragma unroll
  for (int a = 0; a < G; ++a)
    *reinterpret_cast<float4*>(red + warp * G * kDecHeadDim + a * kDecHeadDim + lane * 4) =
        make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
  __syncthreads();
  for (int it = threadIdx.x; it < G * kDecHeadDim; it += kAttnThreads) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) v += red[w * G * kDecHeadDim + it];
    accs[it] = v;
  }
  cluster_merge<G>(hmax, hsum, accs, split, splits, qh0, merged);
}

// x += wo . merged (the attention's merged rows, bf16 values), the weight
// rows of a warp's first job issued before the wait for the previous kernel.
template <typename Rows>
__global__ void __launch_bounds__(kGemvThreads, 1)
    dec_oproj_kernel(DecShape s, const float* merged, Rows w, float* x) {
  extern __shared__ __align__(16) float xs[];
  const int K = s.heads * kDecHeadDim;
  const int qs = K / Fmt<Rows>::kPerChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = s.H / 2;
  int j = blockIdx.x * kGemvWarps + warp;
  uint4 u0[kCpl], u1[kCpl];
  if (j < half) load_rows2(w, j, j + half, 0, qs, lane, u0, u1);
  pdl_wait();
  pdl_launch_dependents();
  for (int e4 = threadIdx.x; e4 < K / 4; e4 += blockDim.x) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(merged) + e4);
    xs[quad_slot<Rows>(4 * e4, qs)] = v.x;
    xs[quad_slot<Rows>(4 * e4 + 1, qs)] = v.y;
    xs[quad_slot<Rows>(4 * e4 + 2, qs)] = v.z;
    xs[quad_slot<Rows>(4 * e4 + 3, qs)] = v.w;
  }
  __syncthreads();
  for (bool first = true; j < half; j += gridDim.x * kGemvWarps, first = false) {
    if (!first) load_rows2(w, j, j + half, 0, qs, lane, u0, u1);
    float d0, d1;
    finish_rows2(w, j, j + half, qs, reinterpret_cast<const float4*>(xs), qs, lane, u0, u1, d0, d1);
    if (lane == 0) {
      x[j] += d0;
      x[j + half] += d1;
    }
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

template <typename Rows>
__global__ void __launch_bounds__(kGemvThreads, 1)
    dec_lmhead_kernel(DecShape s, const float* x, const float* __restrict__ norm, Rows w, float* logits, DecState* st,
                      int2* part, unsigned* counter, int* tokens, int advance, int set_pos) {
  extern __shared__ __align__(16) float dsm[];
  float* xr = dsm;
  float* xs = dsm + s.H;
  __shared__ double npart[kNormWarps];
  __shared__ float inv[1];
  __shared__ float wv[kGemvWarps];
  __shared__ int wi[kGemvWarps];
  __shared__ int is_last;
  const int H = s.H;
  const int qs = H / Fmt<Rows>::kPerChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = (s.vocab + 1) / 2;
  int j = blockIdx.x * kGemvWarps + warp;
  uint4 u0[kCpl], u1[kCpl];
  if (j < half) load_rows2(w, j, j + half < s.vocab ? j + half : j, 0, qs, lane, u0, u1);
  pdl_wait();
  pdl_launch_dependents();
  for (int e4 = threadIdx.x; e4 < H / 4; e4 += blockDim.x)
    reinterpret_cast<float4*>(xr)[e4] = __ldcg(reinterpret_cast<const float4*>(x) + e4);
  __syncthreads();
  stage_normed<Rows>(xr, H, s.eps, norm, xs, npart, inv);
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (bool first = true; j < half; j += gridDim.x * kGemvWarps, first = false) {
    const int r1 = j + half < s.vocab ? j + half : j;
    if (!first) load_rows2(w, j, r1, 0, qs, lane, u0, u1);
    float d0, d1;
    finish_rows2(w, j, r1, qs, reinterpret_cast<const float4*>(xs), qs, lane, u0, u1, d0, d1);
    if (lane == 0) {
      if (logits != nullptr) {
        logits[j] = d0;
        if (r1 != j) logits[r1] = d1;
      }
      if (better(d0, j, bv, bi)) {
        bv = d0;
        bi = j;
      }
      if (r1 != j && better(d1, r1, bv, bi)) {
        bv = d1;
        bi = r1;
      }
    }
  }
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kGemvWarps; ++k)
      if (better(wv[k], wi[k], bv, bi)) {
        bv = wv[k];
        bi = wi[k];
      }
    part[blockIdx.x] = make_int2(__float_as_int(bv), bi);
    __threadfence();
    is_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last || threadIdx.x != 0) return;
  __threadfence();
  float best = -INFINITY;
  int id = INT_MAX;
  for (unsigned b = 0; b < gridDim.x; ++b) {
    const int2 p = __ldcg(part + b);
    if (better(__int_as_float(p.x), p.y, best, id)) {
      best = __int_as_float(p.x);
      id = p.y;
    }
  }
  if (id == INT_MAX) id = 0;
  st->token = id;
  if (advance) {
    tokens[st->step] = id;
    st->step += 1;
    st->pos += 1;
  } else {
    tokens[0] = id;
    st->step = 1;
    st->pos = set_pos;
  }
  *counter = 0;
}

__global__ void __launch_bounds__(256) norm_rows_bf16_kernel(const float* x, int H, const float* gain, float eps,
                                                             __nv_bfloat16* out) {
  __shared__ double part[kNormWarps];
  __shared__ float inv[1];
  const float* row = x + static_cast<int64_t>(blockIdx.x) * H;
  rms_inv_rows(1, H, eps, [&](int, int q) { return __ldg(reinterpret_cast<const float4*>(row) + q); }, part, inv);
  __nv_bfloat16* o = out + static_cast<int64_t>(blockIdx.x) * H;
  for (int e = threadIdx.x; e < H; e += blockDim.x)
    o[e] = __float2bfloat16_rn(rms_apply(row[e], inv[0], gain != nullptr ? gain[e] : 1.0f));
}

__global__ void __launch_bounds__(256) rope_rows_kernel(DecShape s, const float* __restrict__ qkv,
                                                        const float* __restrict__ inv_freq, __nv_bfloat16* q,
                                                        __nv_bfloat16* kc, __nv_bfloat16* vc) {
  const int t = blockIdx.x;
  const int width = (s.heads + 2 * s.kv) * kDecHeadDim;
  const float* row = qkv + static_cast<int64_t>(t) * width;
  for (int p = threadIdx.x; p < (s.heads + 2 * s.kv) * kHalf; p += blockDim.x) {
    const int hh = p / kHalf, i = p % kHalf;
    const float a = row[hh * kDecHeadDim + i], b = row[hh * kDecHeadDim + i + kHalf];
    if (hh < s.heads + s.kv) {
      float o0, o1;
      rotate(a, b, __fmul_rn(static_cast<float>(t), inv_freq[i]), o0, o1);
      if (hh < s.heads) {
        __nv_bfloat16* qr = q + static_cast<int64_t>(t) * s.heads * kDecHeadDim + hh * kDecHeadDim;
        qr[i] = __float2bfloat16_rn(o0);
        qr[i + kHalf] = __float2bfloat16_rn(o1);
      } else {
        const int64_t base = (static_cast<int64_t>(hh - s.heads) * s.max_pos + t) * kDecHeadDim;
        kc[base + i] = __float2bfloat16_rn(o0);
        kc[base + i + kHalf] = __float2bfloat16_rn(o1);
      }
    } else {
      const int64_t base = (static_cast<int64_t>(hh - s.heads - s.kv) * s.max_pos + t) * kDecHeadDim;
      vc[base + i] = __float2bfloat16_rn(a);
      vc[base + i + kHalf] = __float2bfloat16_rn(b);
    }
  }
}

// ---- prefill attention: mma.sync m16n8k16 tiles, online softmax -----------

constexpr int kAttnRows = 64;      // query rows per block (16 per warp)
constexpr int kAttnKeys = 64;      // keys per tile
constexpr int kKStride = kDecHeadDim + 8;  // padded bf16 row of the K tile (conflict-free B loads)
constexpr int kVStride = kAttnKeys + 8;    // padded bf16 row of the transposed V tile

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(128) prefill_attn_kernel(DecShape s, const __nv_bfloat16* __restrict__ q, int rows,
                                                           const __nv_bfloat16* __restrict__ kc,
                                                           const __nv_bfloat16* __restrict__ vc,
                                                           __nv_bfloat16* out, float scale) {
  __shared__ __align__(16) __nv_bfloat16 ks[kAttnKeys * kKStride];
  __shared__ __align__(16) __nv_bfloat16 vt[kDecHeadDim * kVStride];
  const int tile = blockIdx.x, h = blockIdx.y;
  const int g = h / (s.heads / s.kv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int q0 = tile * kAttnRows + warp * 16;  // this warp's first query row
  const int ldq = s.heads * kDecHeadDim;
  // Q fragments for the warp's 16 rows, 8 chunks of 16 dims.
  uint32_t qa[8][4];
  {
    const int ra = q0 + gr, rb = q0 + gr + 8;
    const __nv_bfloat16* pa = q + static_cast<int64_t>(ra) * ldq + h * kDecHeadDim;
    const __nv_bfloat16* pb = q + static_cast<int64_t>(rb) * ldq + h * kDecHeadDim;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + 2 * tq;
      qa[kk][0] = ra < rows ? *reinterpret_cast<const uint32_t*>(pa + c) : 0u;
      qa[kk][1] = rb < rows ? *reinterpret_cast<const uint32_t*>(pb + c) : 0u;
      qa[kk][2] = ra < rows ? *reinterpret_cast<const uint32_t*>(pa + c + 8) : 0u;
      qa[kk][3] = rb < rows ? *reinterpret_cast<const uint32_t*>(pb + c + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  const __nv_bfloat16* kh = kc + static_cast<int64_t>(g) * s.max_pos * kDecHeadDim;
  const __nv_bfloat16* vh = vc + static_cast<int64_t>(g) * s.max_pos * kDecHeadDim;
  const int last_tile = min(tile, (rows - 1) / kAttnKeys);
  for (int kt = 0; kt <= last_tile; ++kt) {
    __syncthreads();  // the previous tile's readers are done
    for (int idx = threadIdx.x; idx < kAttnKeys * (kDecHeadDim / 8); idx += blockDim.x) {
      const int key = idx / (kDecHeadDim / 8), c8 = idx % (kDecHeadDim / 8);
      const int kidx = kt * kAttnKeys + key;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (kidx < rows) {
        kv = *reinterpret_cast<const uint4*>(kh + static_cast<int64_t>(kidx) * kDecHeadDim + c8 * 8);
        vv = *reinterpret_cast<const uint4*>(vh + static_cast<int64_t>(kidx) * kDecHeadDim + c8 * 8);
      }
      *reinterpret_cast<uint4*>(ks + key * kKStride + c8 * 8) = kv;
      const __nv_bfloat16* ve = reinterpret_cast<const __nv_bfloat16*>(&vv);
#pragma unroll
      for (int i = 0; i < 8; ++i) vt[(c8 * 8 + i) * kVStride + key] = ve[i];
    }
    __syncthreads();
    float sfr[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sfr[nt][0] = sfr[nt][1] = sfr[nt][2] = sfr[nt][3] = 0.0f;
      const __nv_bfloat16* kr = ks + (nt * 8 + gr) * kKStride;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + kk * 16 + 2 * tq);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + kk * 16 + 8 + 2 * tq);
        mma_bf16_16816(sfr[nt], qa[kk], b0, b1);
      }
    }
    // scale, causal mask, running max
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kidx = kt * kAttnKeys + nt * 8 + 2 * tq + (e & 1);
        const int qidx = q0 + gr + (e >> 1) * 8;
        const float v = (kidx <= qidx && kidx < rows) ? sfr[nt][e] * scale : -INFINITY;
        sfr[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      alpha[r] = m_new == -INFINITY ? 1.0f : expf(m_run[r] - m_new);  // exp(-inf) = 0 for a first tile
      m_run[r] = m_new;
      l_run[r] *= alpha[r];
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float p = sfr[nt][e] == -INFINITY ? 0.0f : expf(sfr[nt][e] - m_run[r]);
        sfr[nt][e] = p;
        l_run[r] += p;
      }
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= alpha[0];
      o[d][1] *= alpha[0];
      o[d][2] *= alpha[1];
      o[d][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(sfr[2 * kk][0], sfr[2 * kk][1]);
      pa[1] = pack_bf16(sfr[2 * kk][2], sfr[2 * kk][3]);
      pa[2] = pack_bf16(sfr[2 * kk + 1][0], sfr[2 * kk + 1][1]);
      pa[3] = pack_bf16(sfr[2 * kk + 1][2], sfr[2 * kk + 1][3]);
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        const __nv_bfloat16* vr = vt + (d * 8 + gr) * kVStride + kk * 16;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(vr + 2 * tq);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(vr + 8 + 2 * tq);
        mma_bf16_16816(o[d], pa, b0, b1);
      }
    }
  }
  float l[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] = l_run[r] + __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + gr + 8 * r;
    if (row >= rows) continue;
    __nv_bfloat16* orow = out + static_cast<int64_t>(row) * ldq + h * kDecHeadDim;
    const float il = 1.0f / l[r];
#pragma unroll
    for (int d = 0; d < 16; ++d)
      *reinterpret_cast<uint32_t*>(orow + d * 8 + 2 * tq) = pack_bf16(o[d][2 * r] * il, o[d][2 * r + 1] * il);
  }
}

const void* attn_fn(int G) {
  switch (G) {
    case 1: return reinterpret_cast<const void*>(dec_attn_kernel<1>);
    case 2: return reinterpret_cast<const void*>(dec_attn_kernel<2>);
    case 4: return reinterpret_cast<const void*>(dec_attn_kernel<4>);
    case 8: return reinterpret_cast<const void*>(dec_attn_kernel<8>);
    default: return nullptr;
  }
}

// ---- decode attention on the tensor cores --------------------------------

constexpr int kTcKeysPerWarp = 48;  // keys a warp scores per round (6 tiles of 8, 3 chunks of 16 for p . V)
constexpr int kTcRound = kTcKeysPerWarp * kAttnWarps;
constexpr int kKvStride = kDecHeadDim + 8;  // padded bf16 row of the staged K and V (conflict-free fragments)

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_addr(row_addr)));
}

// The same split-key attention as dec_attn_kernel with the products on the
// tensor cores: the G query heads are the rows of 16-row mma tiles (the other
// rows zero), the split's K and V rows staged in shared memory by cp.async
// (K and V rows padded to 136 bf16, so every fragment load is conflict-free;
// V's fragments come transposed from ldmatrix). Warp w takes 48 keys a round
// (s = q . k as 6 tiles of 8 keys x 8 chunks of 16 dims, then an online
// softmax per head: running max, rescale, exp; p rounded to bf16 as the A
// operand of p . V, 3 chunks of 16 keys x 16 tiles of 8 dims). The warps'
// (max, sum, p . V) per head are merged in shared memory, then the cluster
// merges its splits as dec_attn_kernel does.
template <int G>
__global__ void __launch_bounds__(kAttnThreads) dec_attn_tc_kernel(DecShape s, const float* __restrict__ q,
                                                                   const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                                                                   const DecState* st, float* merged, int cap,
                                                                   float scale) {
  extern __shared__ __align__(16) unsigned char sraw[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(sraw);            // [cap][136]
  __nv_bfloat16* vs = ks + static_cast<size_t>(cap) * kKvStride;         // [cap][136]
  float* wo = reinterpret_cast<float*>(vs + static_cast<size_t>(cap) * kKvStride);  // [warps][G][128]
  float* accs = wo + kAttnWarps * G * kDecHeadDim;                        // [G][128]
  __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
  __shared__ float hmax[G], hsum[G];
  // The position comes from the state the previous step's lm_head advanced
  // (complete before this step's first kernel); the cache rows before it
  // were written by earlier steps, so they are staged before the wait for
  // the q/k/v grid, which writes only row pos.
  const int qh0 = blockIdx.x * G, split = blockIdx.y, splits = gridDim.y;
  const int g = qh0 / (s.heads / s.kv);
  const int pos = st->pos;
  const int keys = pos + 1;
  const int chunk = (keys + splits - 1) / splits;
  const int first = split * chunk;
  const int n = max(0, min(keys, first + chunk) - first);
  const int n_old = max(0, min(n, pos - first));  // this split's rows before pos
  const __nv_bfloat16* kh = kc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  const __nv_bfloat16* vh = vc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  auto stage_rows = [&](int k0, int k1) {
    for (int c = k0 * (kDecHeadDim / 8) + static_cast<int>(threadIdx.x); c < k1 * (kDecHeadDim / 8);
         c += kAttnThreads) {
      const int key = c / (kDecHeadDim / 8), c8 = c % (kDecHeadDim / 8);
      cp_async16(ks + key * kKvStride + c8 * 8, kh + c * 8);
      cp_async16(vs + key * kKvStride + c8 * 8, vh + c * 8);
    }
  };
  stage_rows(0, n_old);
  pdl_wait();
  pdl_launch_dependents();
  stage_rows(n_old, n);  // row pos, written by the q/k/v grid
  cp_async_commit();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gr = lane >> 2, tq = lane & 3;
  // Q as the A operand: row gr < G is query head qh0 + gr, other rows zero.
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    if (gr < G) {
      const float* qr = q + (qh0 + gr) * kDecHeadDim + kk * 16 + 2 * tq;
      const float2 lo = __ldcg(reinterpret_cast<const float2*>(qr));
      const float2 hi = __ldcg(reinterpret_cast<const float2*>(qr + 8));
      qa[kk][0] = pack_bf16(lo.x, lo.y);
      qa[kk][1] = pack_bf16(hi.x, hi.y);
    } else {
      qa[kk][0] = qa[kk][1] = 0u;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;  // for row gr (valid when gr < G)
  for (int base = warp * kTcKeysPerWarp; base < n; base += kTcRound) {
    float sc[6][4];
#pragma unroll
    for (int nt = 0; nt < 6; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
      const int key = base + nt * 8 + gr;
      const __nv_bfloat16* kr = ks + min(key, n - 1) * kKvStride;  // keys past n: a staged row, masked below
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + kk * 16 + 2 * tq);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + kk * 16 + 8 + 2 * tq);
        const uint32_t a[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
        mma_bf16_16816(sc[nt], a, b0, b1);
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 6; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = base + nt * 8 + 2 * tq + e;
        const float v = key < n ? sc[nt][e] * scale : -INFINITY;
        sc[nt][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_new == -INFINITY ? 1.0f : expf(m_run - m_new);
    m_run = m_new;
    l_run *= alpha;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= alpha;
      o[d][1] *= alpha;
    }
#pragma unroll
    for (int nt = 0; nt < 6; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p = sc[nt][e] == -INFINITY ? 0.0f : expf(sc[nt][e] - m_run);
        sc[nt][e] = p;
        l_run += p;
      }
#pragma unroll
    for (int kc2 = 0; kc2 < 3; ++kc2) {
      const uint32_t pa[4] = {pack_bf16(sc[2 * kc2][0], sc[2 * kc2][1]), 0u,
                              pack_bf16(sc[2 * kc2 + 1][0], sc[2 * kc2 + 1][1]), 0u};
      // rows of the 16-key chunk; keys past n read a staged (finite) row with p = 0
      const int krow = min(base + kc2 * 16 + (lane & 15), n - 1);
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        uint32_t b0, b1;
        ldmatrix_x2_trans(b0, b1, vs + krow * kKvStride + d * 8);
        mma_bf16_16816(o[d], pa, b0, b1);
      }
    }
  }
  // this warp's row sum (the four lanes of a row hold parts of it)
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (gr < G) {
    if (tq == 0) {
      wm[warp][gr] = m_run;
      wl[warp][gr] = l_run;
    }
#pragma unroll
    for (int d = 0; d < 16; ++d)
      *reinterpret_cast<float2*>(wo + (warp * G + gr) * kDecHeadDim + d * 8 + 2 * tq) = make_float2(o[d][0], o[d][1]);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int a = threadIdx.x;
    float m = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) m = fmaxf(m, wm[w][a]);
    float l = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w)
      if (wm[w][a] != -INFINITY) l = fmaf(expf(wm[w][a] - m), wl[w][a], l);
    hmax[a] = m;
    hsum[a] = l;
  }
  __syncthreads();
  for (int it = threadIdx.x; it < G * kDecHeadDim; it += kAttnThreads) {
    const int a = it / kDecHeadDim;
    float v = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w)
      if (wm[w][a] != -INFINITY) v = fmaf(expf(wm[w][a] - hmax[a]), wo[(w * G) * kDecHeadDim + it], v);
    accs[it] = v;
  }
  cluster_merge<G>(hmax, hsum, accs, split, splits, qh0, merged);
}

const void* attn_tc_fn(int G) {
  switch (G) {
    case 1: return reinterpret_cast<const void*>(dec_attn_tc_kernel<1>);
    case 2: return reinterpret_cast<const void*>(dec_attn_tc_kernel<2>);
    case 4: return reinterpret_cast<const void*>(dec_attn_tc_kernel<4>);
    case 8: return reinterpret_cast<const void*>(dec_attn_tc_kernel<8>);
    default: return nullptr;
  }
}

template <typename Rows>
void* qkv_fn() {
  return reinterpret_cast<void*>(dec_qkv_kernel<Rows>);
}
template <typename Rows>
void* oproj_fn() {
  return reinterpret_cast<void*>(dec_oproj_kernel<Rows>);
}
template <typename Rows>
void* lmhead_fn() {
  return reinterpret_cast<void*>(dec_lmhead_kernel<Rows>);
}

}  // namespace

cudaError_t prepare_decoder_kernels() {
  static bool done[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (done[dev]) return cudaSuccess;
  if ((st = allow_max_dynamic_smem(dec_qkv_kernel<Bf16Rows>)) != cudaSuccess) return st;
  if ((st = allow_max_dynamic_smem(dec_qkv_kernel<Q8Rows>)) != cudaSuccess) return st;
  if ((st = allow_max_dynamic_smem(dec_oproj_kernel<Bf16Rows>)) != cudaSuccess) return st;
  if ((st = allow_max_dynamic_smem(dec_oproj_kernel<Q8Rows>)) != cudaSuccess) return st;
  if ((st = allow_max_dynamic_smem(dec_lmhead_kernel<Bf16Rows>)) != cudaSuccess) return st;
  if ((st = allow_max_dynamic_smem(dec_lmhead_kernel<Q8Rows>)) != cudaSuccess) return st;
  for (int i = 0; i < 8; ++i) {
    const int G = 1 << (i % 4);
    const void* fn = i < 4 ? attn_fn(G) : attn_tc_fn(G);
    int optin = 0;
    cudaFuncAttributes a{};
    if ((st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return st;
    if ((st = cudaFuncGetAttributes(&a, fn)) != cudaSuccess) return st;
    if ((st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   optin - static_cast<int>(a.sharedSizeBytes))) != cudaSuccess)
      return st;
    if ((st = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess) return st;
  }
  done[dev] = true;
  return cudaSuccess;
}

cudaError_t launch_dec_qkv(const DecShape& s, bool int8, float* x, const __nv_bfloat16* embed, const float* norm,
                           DecMatrix wqkv, const float* inv_freq, const DecState* st, float* q_out,
                           __nv_bfloat16* kcache, __nv_bfloat16* vcache, int sm_count, cudaStream_t stream, bool pdl) {
  DecShape sh = s;
  const size_t smem = static_cast<size_t>(2 * s.H) * sizeof(float);
  if (int8) {
    Q8Rows w{static_cast<const int8_t*>(wqkv.w), wqkv.scale, s.H};
    void* args[] = {&sh, &x, &embed, &norm, &w, &inv_freq, &st, &q_out, &kcache, &vcache};
    return launch_maybe_pdl(qkv_fn<Q8Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
  }
  Bf16Rows w{static_cast<const __nv_bfloat16*>(wqkv.w), s.H};
  void* args[] = {&sh, &x, &embed, &norm, &w, &inv_freq, &st, &q_out, &kcache, &vcache};
  return launch_maybe_pdl(qkv_fn<Bf16Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
}

size_t dec_attn_smem(const DecShape& s, int splits, bool v_smem) {
  const size_t G = static_cast<size_t>(s.heads / s.kv);  // query heads per block
  const size_t cap = static_cast<size_t>((s.max_pos + splits - 1) / splits);
  const size_t capr = (cap + 3) & ~size_t{3};
  return (G * capr + kAttnWarps * G * kDecHeadDim + G * kDecHeadDim) * 4 + (v_smem ? cap * kDecHeadDim * 2 : 0);
}

size_t dec_attn_tc_smem(const DecShape& s, int splits) {
  const size_t G = static_cast<size_t>(s.heads / s.kv);
  const size_t cap = static_cast<size_t>((s.max_pos + splits - 1) / splits);
  return 2 * cap * kKvStride * 2 + (kAttnWarps * G * kDecHeadDim + G * kDecHeadDim) * 4;
}

namespace {
// Whether a cluster of c blocks of fn with smem bytes can be placed.
bool cluster_fits(const void* fn, const DecShape& s, int c, size_t smem) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(s.kv, c);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = c;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return clusters >= 1;
}
}  // namespace

cudaError_t plan_dec_attn(const DecShape& s, bool cuda_cores, int* splits, int* mode) {
  const int G = s.heads / s.kv;
  const void* fn = attn_fn(G);
  const void* tc = attn_tc_fn(G);
  if (fn == nullptr || tc == nullptr) return cudaErrorInvalidValue;
  int dev = 0, optin = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (st != cudaSuccess) return st;
  const size_t limit = static_cast<size_t>(optin) - 1024;
  for (int c : {16, 8}) {
    if (!cuda_cores && dec_attn_tc_smem(s, c) <= limit && cluster_fits(tc, s, c, dec_attn_tc_smem(s, c))) {
      *splits = c;
      *mode = kAttnTensorCores;
      return cudaSuccess;
    }
    for (int vsm : {1, 0}) {
      const size_t smem = dec_attn_smem(s, c, vsm != 0);
      if (smem <= limit && cluster_fits(fn, s, c, smem)) {
        *splits = c;
        *mode = vsm ? kAttnCudaCoresSmemV : kAttnCudaCores;
        return cudaSuccess;
      }
    }
  }
  return cudaErrorNotSupported;
}

cudaError_t launch_dec_attn(const DecShape& s, const float* q, const __nv_bfloat16* kcache,
                            const __nv_bfloat16* vcache, const DecState* st, float* merged, int splits, int mode,
                            cudaStream_t stream, bool pdl) {
  const int G = s.heads / s.kv;
  const bool tc = mode == kAttnTensorCores;
  const void* fn = tc ? attn_tc_fn(G) : attn_fn(G);
  if (fn == nullptr) return cudaErrorInvalidValue;
  DecShape sh = s;
  int cap = (s.max_pos + splits - 1) / splits;
  int vsm = mode == kAttnCudaCoresSmemV ? 1 : 0;
  float scale = 1.0f / sqrtf(static_cast<float>(kDecHeadDim));
  void* args_cc[] = {&sh, &q, &kcache, &vcache, &st, &merged, &cap, &vsm, &scale};
  void* args_tc[] = {&sh, &q, &kcache, &vcache, &st, &merged, &cap, &scale};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(s.kv, splits);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = tc ? dec_attn_tc_smem(s, splits) : dec_attn_smem(s, splits, vsm != 0);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelExC(&cfg, fn, tc ? args_tc : args_cc);
}

cudaError_t launch_dec_oproj(const DecShape& s, bool int8, const float* merged, DecMatrix wo, float* x, int sm_count,
                             cudaStream_t stream, bool pdl) {
  DecShape sh = s;
  const int K = s.heads * kDecHeadDim;
  const size_t smem = static_cast<size_t>(K) * sizeof(float);
  if (int8) {
    Q8Rows w{static_cast<const int8_t*>(wo.w), wo.scale, K};
    void* args[] = {&sh, &merged, &w, &x};
    return launch_maybe_pdl(oproj_fn<Q8Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
  }
  Bf16Rows w{static_cast<const __nv_bfloat16*>(wo.w), K};
  void* args[] = {&sh, &merged, &w, &x};
  return launch_maybe_pdl(oproj_fn<Bf16Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
}

cudaError_t launch_dec_lmhead(const DecShape& s, bool int8, const float* x, const float* norm, DecMatrix lm_head,
                              float* logits, DecState* st, int2* part, unsigned* counter, int* tokens, int advance,
                              int set_pos, int sm_count, cudaStream_t stream, bool pdl) {
  DecShape sh = s;
  const size_t smem = static_cast<size_t>(2 * s.H) * sizeof(float);
  if (int8) {
    Q8Rows w{static_cast<const int8_t*>(lm_head.w), lm_head.scale, s.H};
    void* args[] = {&sh, &x, &norm, &w, &logits, &st, &part, &counter, &tokens, &advance, &set_pos};
    return launch_maybe_pdl(lmhead_fn<Q8Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
  }
  Bf16Rows w{static_cast<const __nv_bfloat16*>(lm_head.w), s.H};
  void* args[] = {&sh, &x, &norm, &w, &logits, &st, &part, &counter, &tokens, &advance, &set_pos};
  return launch_maybe_pdl(lmhead_fn<Bf16Rows>(), dim3(sm_count), dim3(kGemvThreads), smem, stream, args, pdl);
}

cudaError_t launch_norm_rows_bf16(const float* x, int64_t rows, int H, const float* gain, float eps,
                                  __nv_bfloat16* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  norm_rows_bf16_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(x, H, gain, eps, out);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows(const DecShape& s, const float* qkv, int64_t rows, const float* inv_freq,
                             __nv_bfloat16* q, __nv_bfloat16* kcache, __nv_bfloat16* vcache, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  rope_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(s, qkv, inv_freq, q, kcache, vcache);
  return cudaGetLastError();
}

cudaError_t launch_prefill_attn(const DecShape& s, const __nv_bfloat16* q, int64_t rows, const __nv_bfloat16* kcache,
                                const __nv_bfloat16* vcache, __nv_bfloat16* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((rows + kAttnRows - 1) / kAttnRows), static_cast<unsigned>(s.heads));
  prefill_attn_kernel<<<grid, 128, 0, stream>>>(s, q, static_cast<int>(rows), kcache, vcache, out,
                                                1.0f / sqrtf(static_cast<float>(kDecHeadDim)));
  return cudaGetLastError();
}

}  // namespace uocr_b200
