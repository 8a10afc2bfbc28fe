// Weight-row access of the decode kernels (decode.cu): streaming 16-byte
// loads and the dot products of one
// chunk of bf16 or per-channel int8 weights against fp32 or bf16 inputs.
#pragma once

#include "moe_common.cuh"

namespace uocr_b200 {

// Weights are read once per step and never reused from L1.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Asks the TMA unit to bring `bytes` (a multiple of 16, 16-byte aligned
// address) from HBM into L2: no registers or shared memory held, so a warp can
// keep many rows on their way while it works on earlier ones.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Activation loads: 0 read-only global path, 1 through L2 only (written
// earlier in the same kernel), 2 generic (shared or global memory).
template <int Mode>
__device__ __forceinline__ uint4 ld_act(const uint4* p) {
  if constexpr (Mode == 1)
    return __ldcg(p);
  else if constexpr (Mode == 2)
    return *p;
  else
    return __ldg(p);
}

// How the decode kernels read one weight format: rows of 16-byte chunks
// (8 bf16 or 16 int8 weights) and the per-row scale.
template <typename Rows>
struct Fmt;

// Packed fp32 pairs for the decode dots (sm_100 f32x2): two weights per
// instruction; each element rounds as the scalar fmaf / fsub would.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_sum(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Bytes 2p and 2p+1 of the sign-flipped word u as an fp32 pair of their int8
// values: each byte under the bits of 2^23 + 128, minus that bias (exact).
__device__ __forceinline__ uint64_t i8_pair(uint32_t u, int p) {
  constexpr uint64_t kBias2 = 0x4B0000804B000080ull;  // (2^23 + 128, 2^23 + 128)
  const uint32_t lo = __byte_perm(u, 0x4b000000u, p == 0 ? 0x7540u : 0x7542u);
  const uint32_t hi = __byte_perm(u, 0x4b000000u, p == 0 ? 0x7541u : 0x7543u);
  uint64_t v, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo), "r"(hi));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(v), "l"(kBias2));
  return d;
}

// The two bf16 weights of word v as an fp32 pair (exact: a bf16 is the top
// half of an fp32).
__device__ __forceinline__ uint64_t bf16_pair(uint32_t v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(v << 16), "r"(v & 0xffff0000u));
  return r;
}

template <>
struct Fmt<Bf16Rows> {
  static constexpr int kElemBytes = 2;
  static constexpr int kPerChunk = 8;  // weights per 16 bytes
  __device__ static const uint4* row(const Bf16Rows& r, int64_t i) {
    return reinterpret_cast<const uint4*>(r.w + i * r.cols);
  }
  __device__ static float scale(const Bf16Rows&, int64_t) { return 1.0f; }
  // 16 bytes of weights against fp32 inputs in shared memory
  __device__ static float dot_x(const uint4& w, const float* x) {
    const float4 x0 = reinterpret_cast<const float4*>(x)[0];
    const float4 x1 = reinterpret_cast<const float4*>(x)[1];
    return dot8_bf16(w, x0, x1);
  }
  // The same product with the chunk's inputs stored as kQuads float4s
  // `qs` float4s apart (the conflict-free shared layout of the gate/up kernel).
  static constexpr int kQuads = 2;
  // Even and odd weights accumulate in the two halves of a packed pair.
  __device__ static float dot_xq(const uint4& w, const float4* x, int qs) {
    const float4 x0 = x[0], x1 = x[qs];
    uint64_t s = 0;
    s = f2_fma(bf16_pair(w.x), f2_pack(x0.x, x0.y), s);
    s = f2_fma(bf16_pair(w.y), f2_pack(x0.z, x0.w), s);
    s = f2_fma(bf16_pair(w.z), f2_pack(x1.x, x1.y), s);
    s = f2_fma(bf16_pair(w.w), f2_pack(x1.z, x1.w), s);
    return f2_sum(s);
  }
  // 16 bytes of weights against bf16 activations (load mode as ld_act).
  // Even and odd weights in the two halves of an f32x2 accumulator (Packed
  // selects the packed form for int8 rows; bf16 rows always use it).
  template <int Cg = 0, bool Packed = false>
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    const uint4 a = ld_act<Cg>(reinterpret_cast<const uint4*>(act));
    uint64_t s = 0;
    s = f2_fma(bf16_pair(w.x), bf16_pair(a.x), s);
    s = f2_fma(bf16_pair(w.y), bf16_pair(a.y), s);
    s = f2_fma(bf16_pair(w.z), bf16_pair(a.z), s);
    s = f2_fma(bf16_pair(w.w), bf16_pair(a.w), s);
    return f2_sum(s);
  }
};

template <>
struct Fmt<Q8Rows> {
  static constexpr int kElemBytes = 1;
  static constexpr int kPerChunk = 16;
  __device__ static const uint4* row(const Q8Rows& r, int64_t i) {
    return reinterpret_cast<const uint4*>(r.q + i * r.cols);
  }
  __device__ static float scale(const Q8Rows& r, int64_t i) { return __ldg(r.scale + i); }
  __device__ static float dot_x(const uint4& w, const float* x) {
    return dot_xq(w, reinterpret_cast<const float4*>(x), 1);
  }
  static constexpr int kQuads = 4;
  // Even and odd weights accumulate in the two halves of a packed pair.
  __device__ static float dot_xq(const uint4& w, const float4* x, int qs) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint64_t s = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t u = words[q] ^ 0x80808080u;
      const float4 xv = x[q * qs];
      s = f2_fma(i8_pair(u, 0), f2_pack(xv.x, xv.y), s);
      s = f2_fma(i8_pair(u, 1), f2_pack(xv.z, xv.w), s);
    }
    return f2_sum(s);
  }
  // Packed: even and odd weights in the two halves of an f32x2 accumulator
  // (fewer instructions; the batch-1 down kernel keeps the scalar form, which
  // needs fewer registers there).
  template <int Cg = 0, bool Packed = false>
  __device__ static float dot_act(const uint4& w, const __nv_bfloat16* act) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    const uint4 a0 = ld_act<Cg>(reinterpret_cast<const uint4*>(act));
    const uint4 a1 = ld_act<Cg>(reinterpret_cast<const uint4*>(act) + 1);
    const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&a0);
    const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&a1);
    if constexpr (Packed) {
      uint64_t s2 = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t u = words[q] ^ 0x80808080u;
        const __nv_bfloat162* p = q < 2 ? p0 : p1;
        const float2 f0 = __bfloat1622float2(p[(q & 1) * 2]);
        const float2 f1 = __bfloat1622float2(p[(q & 1) * 2 + 1]);
        s2 = f2_fma(i8_pair(u, 0), f2_pack(f0.x, f0.y), s2);
        s2 = f2_fma(i8_pair(u, 1), f2_pack(f1.x, f1.y), s2);
      }
      return f2_sum(s2);
    }
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

}  // namespace uocr_b200
