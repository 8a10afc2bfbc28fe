// Host interface of the prefill path (prefill.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

#include "moe_common.cuh"
#include "tc_gemm.h"

namespace uocr_b200 {

struct PrefillDims {
  int max_rows;
  int hidden;
  int experts;
  int top_k;
  int ffn;
  int shared_ffn;
  int renormalize;
};

// Scratch carved from the plan arena, sized for max_rows.
struct PrefillScratch {
  int* block_counts;            // [blocks, E]
  int* block_offset;            // [blocks, E]
  int* seg_count;               // [E]
  int* seg_start;               // [E]
  int* pos_of;                  // [T, k] position of each selection in the permuted rows
  __nv_bfloat16* xhat;          // [T, H] bf16 rows (shared expert input)
  __nv_bfloat16* xperm;         // [T*k, H] rows grouped by expert, token order inside
  __nv_bfloat16* act;           // [T*k, F] routed SwiGLU activations
  __nv_bfloat16* act_s;         // [T, S] shared SwiGLU activations
  __nv_bfloat16* yperm;         // [T*k, H] routed expert outputs
  float* shared_out;            // [T, H] shared expert output
  size_t bytes;
};

// The shapes the prefill path takes (tile multiples of the grouped GEMM).
inline bool prefill_shapes_ok(int hidden, int ffn, int shared_ffn) {
  return hidden % 256 == 0 && ffn % 128 == 0 && shared_ffn % 128 == 0;
}

// routed_buffers = false leaves seg_count, seg_start, xperm, act and yperm
// null: the expert-parallel path keeps those in its exchange region.
size_t prefill_scratch_bytes(const PrefillDims& d, bool routed_buffers = true);
void carve_prefill_scratch(const PrefillDims& d, void* base, PrefillScratch* s, bool routed_buffers = true);

struct PrefillCall {
  PrefillDims dims;
  PrefillScratch scratch;
  int rows;
  const float* x;           // [T, H] fp32
  const float* router;      // [E, H] fp32
  const float* bias;        // [E] or null
  const __nv_bfloat16* gate, *up, *down, *sgate, *sup, *sdown;
  float* logits;            // [T, E]
  int* ids;                 // [T, k]
  float* weights;           // [T, k]
  const float* resid;       // [T, H] or null
  float* y;                 // [T, H]
  ErrorWord* err;
  int sm_count;
  // Optional: 6 events recorded after router, top-k, permutation, gate/up
  // GEMM, down GEMM and combine (null: none).
  cudaEvent_t* events;
};

// The weighted combine alone (c.scratch.yperm holds the routed outputs at the
// positions pos_of gives).
cudaError_t launch_prefill_combine(const PrefillCall& c, cudaStream_t stream);
cudaError_t launch_router_logits_rows(const float* x, int T, int H, const float* router, const float* bias, int E,
                                      float* logits, cudaStream_t stream);
cudaError_t launch_prefill(const PrefillCall& c, cudaStream_t stream);

// The stages of launch_prefill, for the expert-parallel path (ep.cu):
// router + top-k + permutation (an empty batch writes empty segments), and
// the two grouped GEMM descriptions with the routed and/or shared groups.
cudaError_t launch_prefill_route(const PrefillCall& c, cudaStream_t stream);
GroupedGemm prefill_gate_up_gemm(const PrefillCall& c, bool routed, bool shared);
GroupedGemm prefill_down_gemm(const PrefillCall& c, bool routed, bool shared);

}  // namespace uocr_b200
