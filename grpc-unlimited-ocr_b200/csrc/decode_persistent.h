// Host interface of the persistent decode kernel (decode_persistent.cu): a
// whole decode stack (or one layer) of rows <= 16 in ONE cooperative launch.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

#include "moe_common.cuh"

namespace uocr_b200 {

// One layer's weights on the device (bf16, or int8 with per-row scales).
struct DecodeLayerW {
  const float* router;  // [E, H] fp32
  const float* bias;    // [E] or null
  const void* gate;     // [E*F, H]
  const void* up;       // [E*F, H]
  const void* down;     // [E*H, F]
  const void* sgate;    // [S, H]
  const void* sup;      // [S, H]
  const void* sdown;    // [H, S]
  const float* gate_s, *up_s, *down_s, *sgate_s, *sup_s, *sdown_s;  // int8 scales (null for bf16)
};

// Grid-wide barrier state: arrivals of the current round and its generation.
struct GridBarrier {
  unsigned count;
  unsigned gen;
};

struct PersistentDecodeCall {
  const DecodeLayerW* layers;  // device array, n_layers entries
  int n_layers;
  const float* x;  // [T, H] input of the first layer
  float* y;        // [T, H] output of the last layer; may equal x when residual
  int residual;    // 1: every layer adds its input (the stack); 0: one layer, y = MoE(x)
  int T, H, E, K, F, S, renorm, int8;
  float* logits;   // [T, E] scratch
  int* ids_out;    // optional: the last layer's rank-order ids [T, K] and weights
  float* w_out;
  __nv_bfloat16* act;    // [T*K, F]
  __nv_bfloat16* act_s;  // [T, S]
  GridBarrier* barrier;  // cleared by the launcher
  ErrorWord* err;
  int sm_count;
};

// Whether the persistent kernel takes these shapes on this device (shared
// memory for the staged rows and the down partials), and its set-up.
bool persistent_decode_fits(int T, int H, int E, int K, int S, int sm_count, size_t smem_optin);
cudaError_t prepare_persistent_decode();
cudaError_t launch_persistent_decode(const PersistentDecodeCall& c, cudaStream_t stream);

}  // namespace uocr_b200
