// Host interface of the tcgen05 grouped GEMM (tc_gemm.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_common.cuh"

namespace uocr_b200 {

// out = A . B^T per group, bf16 inputs, fp32 accumulation.
//   routed group e (e < experts): A rows seg_start[e] .. + seg_count[e] of
//     a_routed [a_routed_rows, k_routed]; B rows e * b_rows_per_expert + ...
//     of b0_routed / b1_routed [b_routed_rows, k_routed]; output rows
//     seg_start[e] + i of out_routed (ld_out_routed elements per row).
//   shared group (shared_rows > 0): A rows 0 .. shared_rows of a_shared
//     [shared_rows, k_shared]; B rows of b0_shared / b1_shared; output
//     out_shared (bf16, or fp32 with shared_out_f32 in mode 1).
// mode 0 (gate/up + SwiGLU): b0 = gate stack, b1 = up stack; output column
//   j < n_cols = bf16(silu(A.gate[j]) * (A.up[j])), n_cols a multiple of 128.
// mode 1 (down): b0 = b1 = the down stack; output columns A.B[j], n_cols a
//   multiple of 256.
// k_* are multiples of 64; every matrix is row-major with 16-byte aligned rows.
//
// Routed output rows sent to other GPUs' memory (expert parallelism, mode 1):
// with world > 0, routed output row R (a group's rows arrive source after
// source) belongs to segment (group g, source s), the last s with
// seg_dst[g * world + s] <= R (an empty segment starts where the next one
// does), and is stored as row seg_src[g * world + s] + R - seg_dst[g * world + s]
// of base[s] (ld_out_routed elements per row) instead of out_routed: each
// tile's rows go straight from the epilogue to the GPU they came from.
constexpr int kMaxScatterRanks = 8;
struct RowScatter {
  int world;
  const int* seg_dst;
  const int* seg_src;
  void* base[kMaxScatterRanks];
};

struct GroupedGemm {
  int mode;
  int experts;
  const int* seg_count;
  const int* seg_start;
  const __nv_bfloat16* a_routed;
  int64_t a_routed_rows;
  int k_routed;
  const __nv_bfloat16* b0_routed;
  const __nv_bfloat16* b1_routed;
  int64_t b_routed_rows;
  int b_rows_per_expert;
  int n_cols_routed;
  void* out_routed;
  int64_t ld_out_routed;
  int shared_rows;
  const __nv_bfloat16* a_shared;
  int k_shared;
  const __nv_bfloat16* b0_shared;
  const __nv_bfloat16* b1_shared;
  int64_t b_shared_rows;
  int n_cols_shared;
  void* out_shared;
  int64_t ld_out_shared;
  bool shared_out_f32;
  bool shared_accumulate;  // with shared_out_f32: out_shared += A.B^T (a residual add)
  ErrorWord* err;
  int blocks;  // persistent grid size (the SM count)
  RowScatter scatter;  // world 0: routed rows to out_routed
};

size_t grouped_gemm_smem_bytes();
cudaError_t launch_grouped_gemm(const GroupedGemm& g, cudaStream_t stream);

}  // namespace uocr_b200
