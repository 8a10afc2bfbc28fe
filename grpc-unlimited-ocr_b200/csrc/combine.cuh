// The weighted combine of one output row, shared by the single-GPU prefill
// (prefill.cu) and the expert-parallel one (ep.cu), so both add in the same
// order: y = resid + (shared + sum over the row's selections in ascending
// expert id of w * expert_out) — the order of src/model/feed_forward.cpp:65-76
// (shared first, then the routed sum built expert by expert from 0).
#pragma once

#include "moe_common.cuh"

namespace uocr_b200 {

// The selections of the block's row in ascending expert id (a stable
// order: equal ids keep their slot order): weight and expert output row
// (bf16; null for a dropped selection). Thread j < n fetches selection j and
// counts the selections ahead of it; the ranked weight and row pointer go to
// shared memory, which every thread then reads — one rank per selection
// instead of a sorting network in every thread, and no per-thread copy of the
// list in registers.
struct CombineList {
  float w[kMaxTopK];
  const __nv_bfloat16* src[kMaxTopK];
};

// id_of(i): selection i's expert id; fetch(j, id, &w, &src): its weight and
// expert output row (null for a dropped selection). Every thread of the block
// calls this (it holds a barrier).
template <class IdOf, class Fetch>
__device__ __forceinline__ void order_selections(int n, IdOf id_of, Fetch fetch, CombineList* list) {
  const int j = threadIdx.x;
  if (j < n) {
    const int e = id_of(j);
    int rank = 0;
    for (int i = 0; i < n; ++i) {
      const int ei = id_of(i);
      rank += (ei < e || (ei == e && i < j)) ? 1 : 0;
    }
    float w;
    const __nv_bfloat16* src;
    fetch(j, e, &w, &src);
    list->w[rank] = w;
    list->src[rank] = src;
  }
  __syncthreads();
}

// Columns c .. c+7 of the row (its n ordered selections in r): every
// selection's 16 bytes are loaded before any is added.
__device__ __forceinline__ void combine_cols8(const CombineList& r, int n, int64_t c, const float* shared_row,
                                              const float* resid_row, float* y_row) {
  // Every load of the 8 columns first (expert rows, shared output, residual),
  // then the arithmetic.
  uint4 pk[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j)
    if (j < n && r.src[j] != nullptr) pk[j] = __ldcg(reinterpret_cast<const uint4*>(r.src[j] + c));
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
    if (j >= n || r.src[j] == nullptr) continue;
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
