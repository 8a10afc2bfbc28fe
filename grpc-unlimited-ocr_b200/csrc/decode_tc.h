// Host interface of the tensor-core decode experts (decode_tc.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

#include "moe_kernels.h"

namespace uocr_b200 {

// Most work items one launch may split into (bounds the partial-sum scratch).
constexpr int kDecodeTcMaxItems = 8192;

struct DecodeTcScratch {
  __nv_bfloat16* act;    // [kMaxActive][16][F] routed activations, every batch row
  __nv_bfloat16* act_s;  // [16][S] shared activations
  float* partial;        // [kDecodeTcMaxItems][2][16][128] K-split partial sums
  unsigned* tickets_gu;  // [S/128 + kMaxActive * F/128] last-arriver tickets (zeroed once)
  unsigned* tickets_dn;  // [H/128]
  int max_items;
  size_t bytes;
};

size_t decode_tc_scratch_bytes(int H, int F, int S);
void carve_decode_tc_scratch(int H, int F, int S, void* base, DecodeTcScratch* s);
bool decode_tc_shapes_ok(int H, int F, int S);

struct DecodeTcCall {
  const float* x;  // [T, H]
  int T, H, F, S, E;
  const __nv_bfloat16 *gate, *up, *down, *sgate, *sup, *sdown;
  DecodeRouting routing;
  const float* resid;
  float* y;
  DecodeTcScratch scratch;
  ErrorWord* err;
  int sm_count;
  bool pdl;
  cudaEvent_t between;  // optional, recorded between the two kernels
};

// Launches the gate/up and the down kernels.
cudaError_t launch_decode_tc(const DecodeTcCall& c, cudaStream_t stream);

}  // namespace uocr_b200
