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
// one weight stream, split-key GQA attention whose last block per key/value
// head merges the splits, and the output GEMV with the residual add fused —
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

// Two weight rows against the staged input: all of a row's chunks are loaded
// before the first product (kCpl per lane, 16 bytes each), both rows at once.
template <typename Rows>
__device__ __forceinline__ void dot_rows2(const Rows& w, int64_t r0, int64_t r1, int nchunks, const float4* xs4,
                                          int qs, int lane, float& d0, float& d1) {
  using F = Fmt<Rows>;
  const uint4* p0 = F::row(w, r0);
  const uint4* p1 = F::row(w, r1);
  float a0 = 0.0f, a1 = 0.0f;
  for (int base = 0; base < nchunks; base += 32 * kCpl) {
    uint4 u0[kCpl], u1[kCpl];
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
  for (int e = threadIdx.x; e < H; e += blockDim.x)
    xs[quad_slot<Rows>(e, qs)] = bf16_round(rms_apply(xr[e], iv, gain != nullptr ? gain[e] : 1.0f));
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
  pdl_wait();
  const int H = s.H;
  const int pos = st->pos;
  if (embed != nullptr) {
    const __nv_bfloat16* row = embed + static_cast<int64_t>(st->token) * H;
    for (int e = threadIdx.x; e < H; e += blockDim.x) xr[e] = __bfloat162float(row[e]);
  } else {
    for (int e = threadIdx.x; e < H; e += blockDim.x) xr[e] = x[e];
  }
  __syncthreads();
  if (embed != nullptr && blockIdx.x == 0)
    for (int e = threadIdx.x; e < H; e += blockDim.x) x[e] = xr[e];
  stage_normed<Rows>(xr, H, s.eps, norm, xs, part, inv);
  const int qs = H / Fmt<Rows>::kPerChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jobs = (s.heads + 2 * s.kv) * kHalf;
  for (int j = blockIdx.x * kGemvWarps + warp; j < jobs; j += gridDim.x * kGemvWarps) {
    const int hh = j / kHalf, i = j % kHalf;
    const int64_t r0 = static_cast<int64_t>(hh) * kDecHeadDim + i, r1 = r0 + kHalf;
    float d0, d1;
    dot_rows2(w, r0, r1, qs, reinterpret_cast<const float4*>(xs), qs, lane, d0, d1);
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

// Split-key attention: block (kv head g, split). Scores of the split's keys
// for the g's query heads (8 lanes per key, two groups of four keys in flight
// per warp), the split's max and exp sum per head, p . V, and the partials;
// the last block of head g (a ticket) merges its splits.
__global__ void __launch_bounds__(256) dec_attn_kernel(DecShape s, const float* __restrict__ q,
                                                       const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                                                       const DecState* st, float* part, unsigned* counters,
                                                       float* merged, int splits, int cap, float scale) {
  extern __shared__ __align__(16) float dsm[];
  const int G = s.heads / s.kv;
  float* qsm = dsm;               // [G][128]
  float* sc = dsm + G * kDecHeadDim;  // [G][cap]
  __shared__ float hmax[kDecMaxGroup], hsum[kDecMaxGroup];
  __shared__ int is_last;
  pdl_wait();
  const int g = blockIdx.x, split = blockIdx.y;
  const int keys = st->pos + 1;
  const int chunk = (keys + splits - 1) / splits;
  const int first = split * chunk;
  const int n = max(0, min(keys, first + chunk) - first);
  for (int t = threadIdx.x; t < G * kDecHeadDim; t += blockDim.x) qsm[t] = q[g * G * kDecHeadDim + t];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane >> 3, sl = lane & 7;  // key of the group of four, lane within the key
  const __nv_bfloat16* kh = kc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  const __nv_bfloat16* vh = vc + (static_cast<int64_t>(g) * s.max_pos + first) * kDecHeadDim;
  for (int j0 = warp * 8; j0 < n; j0 += 64) {
    uint4 k0[2], k1[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int jj = j0 + 4 * u + sub;
      if (jj < n) {
        const uint4* p = reinterpret_cast<const uint4*>(kh + static_cast<int64_t>(jj) * kDecHeadDim + sl * 16);
        k0[u] = p[0];
        k1[u] = p[1];
      } else {
        k0[u] = make_uint4(0, 0, 0, 0);
        k1[u] = k0[u];
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int jj = j0 + 4 * u + sub;
      for (int a = 0; a < G; ++a) {
        const float4* qv = reinterpret_cast<const float4*>(qsm + a * kDecHeadDim + sl * 16);
        float d = dot8_bf16(k0[u], qv[0], qv[1]) + dot8_bf16(k1[u], qv[2], qv[3]);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        if (sl == 0 && jj < n) sc[a * cap + jj] = d * scale;
      }
    }
  }
  __syncthreads();
  // Warp a: head a's max and exp sum over the split (exp overwrites the scores).
  if (warp < G) {
    float* row = sc + warp * cap;
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
  __syncthreads();
  // p . V: item (head a, dim pair dp).
  for (int it = threadIdx.x; it < G * kHalf; it += blockDim.x) {
    const int a = it / kHalf, dp = it % kHalf;
    const float* pr = sc + a * cap;
    float acc0 = 0.0f, acc1 = 0.0f;
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      __nv_bfloat162 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = *reinterpret_cast<const __nv_bfloat162*>(vh + static_cast<int64_t>(j + u) * kDecHeadDim + 2 * dp);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __bfloat1622float2(v[u]);
        acc0 = fmaf(pr[j + u], f.x, acc0);
        acc1 = fmaf(pr[j + u], f.y, acc1);
      }
    }
    for (; j < n; ++j) {
      const float2 f =
          __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vh + static_cast<int64_t>(j) * kDecHeadDim + 2 * dp));
      acc0 = fmaf(pr[j], f.x, acc0);
      acc1 = fmaf(pr[j], f.y, acc1);
    }
    float* out = part + (static_cast<int64_t>(g * G + a) * splits + split) * kPartStride;
    out[2 + 2 * dp] = acc0;
    out[3 + 2 * dp] = acc1;
    if (dp == 0) {
      out[0] = hmax[a];
      out[1] = hsum[a];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    is_last = atomicAdd(counters + g, 1u) == static_cast<unsigned>(splits - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int it = threadIdx.x; it < G * kDecHeadDim; it += blockDim.x) {
    const int a = it / kDecHeadDim, d = it % kDecHeadDim;
    const float* ph = part + static_cast<int64_t>(g * G + a) * splits * kPartStride;
    float m = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) m = fmaxf(m, __ldcg(ph + sp * kPartStride));
    float tot = 0.0f, o = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const float ms = __ldcg(ph + sp * kPartStride);
      if (ms == -INFINITY) continue;
      const float wgt = expf(ms - m);
      tot = fmaf(wgt, __ldcg(ph + sp * kPartStride + 1), tot);
      o = fmaf(wgt, __ldcg(ph + sp * kPartStride + 2 + d), o);
    }
    merged[(g * G + a) * kDecHeadDim + d] = bf16_round(o / tot);
  }
  if (threadIdx.x == 0) counters[g] = 0;
}

template <typename Rows>
__global__ void __launch_bounds__(kGemvThreads, 1)
    dec_oproj_kernel(DecShape s, const float* __restrict__ merged, Rows w, float* x) {
  extern __shared__ __align__(16) float xs[];
  pdl_wait();
  const int K = s.heads * kDecHeadDim;
  const int qs = K / Fmt<Rows>::kPerChunk;
  for (int e = threadIdx.x; e < K; e += blockDim.x) xs[quad_slot<Rows>(e, qs)] = merged[e];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = s.H / 2;
  for (int j = blockIdx.x * kGemvWarps + warp; j < half; j += gridDim.x * kGemvWarps) {
    float d0, d1;
    dot_rows2(w, j, j + half, qs, reinterpret_cast<const float4*>(xs), qs, lane, d0, d1);
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
  pdl_wait();
  const int H = s.H;
  for (int e = threadIdx.x; e < H; e += blockDim.x) xr[e] = x[e];
  __syncthreads();
  stage_normed<Rows>(xr, H, s.eps, norm, xs, npart, inv);
  const int qs = H / Fmt<Rows>::kPerChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = (s.vocab + 1) / 2;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int j = blockIdx.x * kGemvWarps + warp; j < half; j += gridDim.x * kGemvWarps) {
    const int r1 = j + half < s.vocab ? j + half : j;
    float d0, d1;
    dot_rows2(w, j, r1, qs, reinterpret_cast<const float4*>(xs), qs, lane, d0, d1);
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
  if ((st = allow_max_dynamic_smem(dec_attn_kernel)) != cudaSuccess) return st;
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

size_t dec_attn_smem(const DecShape& s, int splits) {
  const int G = s.heads / s.kv;
  const int cap = (s.max_pos + splits - 1) / splits;
  return static_cast<size_t>(G) * (kDecHeadDim + cap) * sizeof(float);
}

cudaError_t launch_dec_attn(const DecShape& s, const float* q, const __nv_bfloat16* kcache,
                            const __nv_bfloat16* vcache, const DecState* st, float* part, unsigned* counters,
                            float* merged, int splits, cudaStream_t stream, bool pdl) {
  DecShape sh = s;
  int cap = (s.max_pos + splits - 1) / splits;
  float scale = 1.0f / sqrtf(static_cast<float>(kDecHeadDim));
  void* args[] = {&sh, &q, &kcache, &vcache, &st, &part, &counters, &merged, &splits, &cap, &scale};
  return launch_maybe_pdl(reinterpret_cast<void*>(dec_attn_kernel), dim3(s.kv, splits), dim3(256),
                          dec_attn_smem(s, splits), stream, args, pdl);
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
