// Library-internal entry into a MoE plan (capi.cu) for the decoder
// (decoder_capi.cu), which runs the MoE block inside its own steps.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/uocr_moe.h"

namespace uocr_b200 {

// h <- h + MoE_layer(RMSNorm(h)) in place for a plan made with
// UOCR_PLAN_PRE_NORM: the decoder's whole feed-forward block. Rows up to 16
// take the PDL-chained decode kernels, more rows the prefill path. Checks
// nothing the caller has checked (layer loaded, rows <= max_rows).
int moe_layer_inplace(uocr_moe_plan* p, int64_t layer, float* h, int64_t rows, cudaStream_t stream);

}  // namespace uocr_b200
