// The decoder's pre-feed-forward RMSNorm (src/model/decoder.cpp:180,200;
// ref::rms_norm, src/backend/reference/ops.cpp:129-141) as device functions,
// applied to a layer's input rows where they are read: the decode router and
// gate/up kernels normalise the rows they stage, the prefill path normalises
// its rows once into a scratch copy. Every site uses rms_inv_rows (one
// summation order), so all of them see the same bits.
#pragma once

#include "moe_common.cuh"

namespace uocr_b200 {

// Inverse RMS of a row (H % 4 == 0, rows 16-byte aligned):
// float(1 / sqrt(ss / H + eps)) in double, with ss = the sum of double(v) * v
// (each product exact in double, so a fused multiply-add rounds only the sum).
// The sum is split over eight warps: the row's 16-byte words come in blocks of
// 32 (one word a lane), block j goes to warp j % 8, and a lane keeps one
// double accumulator per word component; a warp's partial is its lanes'
// (a0 + a1) + (a2 + a3) reduced by a butterfly, and the total is the fixed
// tree ((P0 + P1) + (P2 + P3)) + ((P4 + P5) + (P6 + P7)). Every site that
// normalises rows (the decode router and gate/up kernels, the prefill copy)
// uses this order, so all of them see the same bits. The reference adds in
// index order; the totals can differ only by rounding in the last bits of a
// 53-bit sum (about H * 2^-53 relative), which changes the float result only
// when its exact value lies that close to a rounding boundary.
constexpr int kNormWarps = 8;

// Warp w's partial of a row whose word q load(q) returns (elements 4q .. 4q+3).
template <typename Load>
__device__ __forceinline__ double rms_partial(int H, int w, Load load) {
  constexpr int kBatch = 4;
  const int lane = threadIdx.x & 31;
  const int n4 = H / 4;
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  for (int j0 = w; j0 * 32 < n4; j0 += kNormWarps * kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int q = (j0 + kNormWarps * b) * 32 + lane;
      v[b] = q < n4 ? load(q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      a0 = fma(static_cast<double>(v[b].x), static_cast<double>(v[b].x), a0);
      a1 = fma(static_cast<double>(v[b].y), static_cast<double>(v[b].y), a1);
      a2 = fma(static_cast<double>(v[b].z), static_cast<double>(v[b].z), a2);
      a3 = fma(static_cast<double>(v[b].w), static_cast<double>(v[b].w), a3);
    }
  }
  double s = (a0 + a1) + (a2 + a3);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

// The inverse RMS from the eight partials of a row.
__device__ __forceinline__ float rms_inv_from(const double* p, int H, float eps) {
  const double ss = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  return static_cast<float>(1.0 / sqrt(ss / static_cast<double>(H) + static_cast<double>(eps)));
}

// The inverse RMS of rows t = 0..T-1 into inv[t] (shared memory): the
// block's warps take the (row, partial) pairs in turn (part: shared,
// [T][8]) and threads t < T the totals. Every thread of the block calls it;
// it ends with a barrier. word(t, q) returns word q of row t.
template <typename Word>
__device__ __forceinline__ void rms_inv_rows(int T, int H, float eps, Word word, double* part, float* inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int pi = warp; pi < T * kNormWarps; pi += nwarps) {
    const int t = pi / kNormWarps;
    const double p = rms_partial(H, pi % kNormWarps, [&](int q) { return word(t, q); });
    if (lane == 0) part[pi] = p;
  }
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < T) inv[threadIdx.x] = rms_inv_from(part + threadIdx.x * kNormWarps, H, eps);
  __syncthreads();
}

// gain * (v * inv), the reference's order of the two float products.
__device__ __forceinline__ float rms_apply(float v, float inv, float gain) { return __fmul_rn(gain, __fmul_rn(v, inv)); }

}  // namespace uocr_b200
