// Shared device-side pieces of the MoE path: limits, the error word, the
// decode routing table, weight row views and small numeric helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace uocr_b200 {

constexpr int kWarp = 32;
constexpr int kMaxExperts = 128;     // the reference's expert_topk limit (ops.cu:653)
constexpr int kMaxTopK = 8;
constexpr int kDecodeMaxRows = 16;   // rows at or below this take the weight-streaming decode path
constexpr int kMaxActive = kDecodeMaxRows * kMaxTopK;  // distinct experts one decode batch can touch
constexpr int kMaxDevices = 64;

// A kernel that meets a bad index, a capacity overflow or a wait that ran out
// records it here instead of touching memory it should not; the host reads
// it through uocr_moe_check. The first error wins.
enum DeviceErrorCode : int {
  kDevOk = 0,
  kDevBadIndex = 1,
  kDevCapacity = 2,
  kDevWaitTimeout = 3,
};
struct ErrorWord {
  int code;
  int where;
  int a;
  int b;
};
__device__ inline void raise_error(ErrorWord* e, int code, int where, int a, int b) {
  if (atomicCAS(&e->code, 0, code) == 0) {
    e->where = where;
    e->a = a;
    e->b = b;
  }
}

// Routing of one decode batch (rows <= kDecodeMaxRows), written by the
// router. Experts appear once each, in ascending id order (for the op-level
// mirror of expert_ffn_one: in rank order). Expert u owns the slots
// slot_base[u] .. slot_base[u] + tok_count[u] - 1, its batch rows in row
// order; slot s names batch row slot_tok[s] with combine weight slot_w[s] and
// indexes the [slots, F] activation scratch.
struct DecodeRoute {
  int active_count;
  int slot_total;
  int reserved[2];
  int active_expert[kMaxActive];
  int tok_count[kMaxActive];
  int slot_base[kMaxActive];
  int slot_tok[kMaxActive];
  float slot_w[kMaxActive];
};

// Shared-memory floats one warp's softmax/top-k needs: the row's 64-bit keys,
// then the selected weights and ids in rank order.
constexpr int kTopkScratch = 2 * kMaxExperts + 2 * kMaxTopK;

// The decoder's pre-feed-forward RMSNorm on a layer's input rows (rms_norm.cuh);
// `on` = 0 leaves the rows as they are.
struct RowNorm {
  const float* gain;  // [H]
  float eps;
  int on;
};

// A stack of weight rows: bf16, or int8 with one fp32 scale per row.
struct Bf16Rows {
  const __nv_bfloat16* w;
  int64_t cols;
};
struct Q8Rows {
  const int8_t* q;
  const float* scale;
  int64_t cols;
};

// Opts a kernel into the largest dynamic shared memory the current device
// allows next to the kernel's own static shared memory.
template <typename Kernel>
inline cudaError_t allow_max_dynamic_smem(Kernel kernel) {
  int dev = 0, optin = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes attr{};
  if (st == cudaSuccess) st = cudaFuncGetAttributes(&attr, kernel);
  if (st == cudaSuccess)
    st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              optin - static_cast<int>(attr.sharedSizeBytes));
  return st;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// silu(g) * u as the reference backend writes it: v * (1 / (1 + exp(-v)))
// (src/backend/reference/ops.cpp:40,163-167), then times the up projection.
__device__ __forceinline__ float swiglu(float g, float u) {
  const float s = 1.0f / (1.0f + expf(-g));
  return (g * s) * u;
}

// Eight bf16 weights (one 128-bit load) dotted with eight fp32 inputs.
__device__ __forceinline__ float dot8_bf16(const uint4& w, const float4& x0, const float4& x1) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&w);
  const float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
  const float2 c = __bfloat1622float2(p[2]), d = __bfloat1622float2(p[3]);
  float s = a.x * x0.x;
  s = fmaf(a.y, x0.y, s);
  s = fmaf(b.x, x0.z, s);
  s = fmaf(b.y, x0.w, s);
  s = fmaf(c.x, x1.x, s);
  s = fmaf(c.y, x1.y, s);
  s = fmaf(d.x, x1.z, s);
  s = fmaf(d.y, x1.w, s);
  return s;
}

// Four int8 weights packed in a word, as fp32, exactly. Integer-to-float
// conversions issue at a fraction of the fp32 rate, which an int8 weight
// stream at HBM speed would exceed; instead each byte, offset to b + 128 by
// flipping its sign bit, becomes the low mantissa byte of 2^23 (a byte
// permute), and subtracting 2^23 + 128 leaves b exactly (both operands lie in
// [2^23, 2^24), where every integer is a float).
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& a, float& b, float& c, float& d) {
  const uint32_t u = w ^ 0x80808080u;
  constexpr float kBias = 8388736.0f;  // 2^23 + 128
  a = __uint_as_float(__byte_perm(u, 0x4b000000u, 0x7540u)) - kBias;
  b = __uint_as_float(__byte_perm(u, 0x4b000000u, 0x7541u)) - kBias;
  c = __uint_as_float(__byte_perm(u, 0x4b000000u, 0x7542u)) - kBias;
  d = __uint_as_float(__byte_perm(u, 0x4b000000u, 0x7543u)) - kBias;
}

}  // namespace uocr_b200
