// The weighted combine of one output row, shared by the single-GPU prefill
// (prefill.cu) and the expert-parallel one (ep.cu), so both add in the same
// order: y = resid + (shared + sum over the row's selections in ascending
// expert id of w * expert_out) — the order of src/model/feed_forward.cpp:65-76
// (shared first, then the routed sum built expert by expert from 0).
#pragma once

#include "moe_common.cuh"

namespace uocr_b200 {

// A row's selections: expert id, weight and the expert output row (bf16).
struct CombineRow {
  int n;
  int eid[kMaxTopK];
  float w[kMaxTopK];
  const __nv_bfloat16* src[kMaxTopK];
};

// Ascending expert id; a fully unrolled exchange network, so the arrays stay
// in registers.
__device__ __forceinline__ void sort_selections(CombineRow& r) {
#pragma unroll
  for (int a = 0; a < kMaxTopK - 1; ++a) {
#pragma unroll
    for (int b = 0; b < kMaxTopK - 1 - a; ++b) {
      if (b + 1 < r.n && r.eid[b + 1] < r.eid[b]) {
        const int te = r.eid[b];
        r.eid[b] = r.eid[b + 1];
        r.eid[b + 1] = te;
        const float tw = r.w[b];
        r.w[b] = r.w[b + 1];
        r.w[b + 1] = tw;
        const __nv_bfloat16* ts = r.src[b];
        r.src[b] = r.src[b + 1];
        r.src[b + 1] = ts;
      }
    }
  }
}

// Columns c .. c+7 of the row: every selection's 16 bytes are loaded before
// any is added (src[j] null: a dropped selection).
__device__ __forceinline__ void combine_cols8(const CombineRow& r, int64_t c, const float* shared_row,
                                              const float* resid_row, float* y_row) {
  // Every load of the 8 columns first (expert rows, shared output, residual),
  // then the arithmetic.
  uint4 pk[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j)
    if (j < r.n && r.src[j] != nullptr) pk[j] = __ldcg(reinterpret_cast<const uint4*>(r.src[j] + c));
  float4 sa = make_float4(0, 0, 0, 0), sb = sa, ra = sa, rb = sa;
  if (shared_row != nullptr) {
    sa = __ldcg(reinterpret_cast<const float4*>(shared_row + c));
    sb = __ldcg(reinterpret_cast<const float4*>(shared_row + c) + 1);
  }
  if (resid_row != nullptr) {
    ra = __ldcg(reinterpret_cast<const float4*>(resid_row + c));
    rb = __ldcg(reinterpret_cast<const float4*>(resid_row + c) + 1);
  }
  float routed[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j >= r.n || r.src[j] == nullptr) continue;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk[j]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(h[q]);
      routed[2 * q] = __fadd_rn(routed[2 * q], __fmul_rn(r.w[j], f.x));
      routed[2 * q + 1] = __fadd_rn(routed[2 * q + 1], __fmul_rn(r.w[j], f.y));
    }
  }
  const float sh[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
  const float rs[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
  float out[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    out[q] = __fadd_rn(sh[q], routed[q]);
    if (resid_row != nullptr) out[q] = __fadd_rn(rs[q], out[q]);
  }
  reinterpret_cast<float4*>(y_row + c)[0] = make_float4(out[0], out[1], out[2], out[3]);
  reinterpret_cast<float4*>(y_row + c)[1] = make_float4(out[4], out[5], out[6], out[7]);
}

}  // namespace uocr_b200
