// Host interface of the page-decoder kernels around the MoE (decoder.cu):
// attention (RMSNorm, q/k/v with the rotate-half RoPE, GQA over a bf16 KV
// cache, the output projection with its residual add), the final norm with
// lm_head and greedy selection, and the prefill's row kernels. The MoE block
// itself runs through a uocr_moe_plan.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_common.cuh"

namespace uocr_b200 {

constexpr int kDecHeadDim = 128;  // the only head width the kernels take
constexpr int kDecMaxGroup = 8;   // query heads per key/value head

// Where the sequence stands, in device memory so that a captured decode step
// replays unchanged: pos = position the next step processes, token = the
// token it consumes, step = how many tokens have been generated.
struct DecState {
  int pos;
  int token;
  int step;
  int reserved;
};

struct DecShape {
  int H;        // model width
  int heads;    // query heads
  int kv;       // key/value heads
  int vocab;
  int max_pos;  // KV cache length
  float eps;    // RMSNorm epsilon
};

// A weight matrix in the decoder's format: bf16, or int8 with one fp32 scale
// per row (scale null for bf16).
struct DecMatrix {
  const void* w;
  const float* scale;
};

// Decode step, layer part 1: RMSNorm(x) -> q, k, v (one matrix of
// (heads + 2 kv) * 128 rows), RoPE on q and k at state.pos, k and v into the
// cache at pos, q (bf16 values, fp32 storage) into q_out. With embed non-null
// the input row is embed[state.token] (written to x as the residual stream).
cudaError_t launch_dec_qkv(const DecShape& s, bool int8, float* x, const __nv_bfloat16* embed, const float* norm,
                           DecMatrix wqkv, const float* inv_freq, const DecState* st, float* q_out,
                           __nv_bfloat16* kcache, __nv_bfloat16* vcache, int sm_count, cudaStream_t stream, bool pdl);

// Decode step, layer part 2: split-key GQA attention of q over keys 0..pos,
// one thread-block cluster of `splits` blocks per key/value head; the blocks
// merge their partials through distributed shared memory into merged
// ([heads * 128], bf16 values). plan_dec_attn picks the split count (16, or
// 8 where a 16-block cluster cannot be placed) and the mode.
// Modes: the products on the tensor cores (a split's K and V rows staged in
// shared memory; the default where they fit), or on the CUDA cores with the V
// rows in shared memory or read from global memory.
enum DecAttnMode : int { kAttnCudaCores = 0, kAttnCudaCoresSmemV = 1, kAttnTensorCores = 2 };
size_t dec_attn_smem(const DecShape& s, int splits, bool v_smem);
size_t dec_attn_tc_smem(const DecShape& s, int splits);
cudaError_t plan_dec_attn(const DecShape& s, bool cuda_cores, int* splits, int* mode);
cudaError_t launch_dec_attn(const DecShape& s, const float* q, const __nv_bfloat16* kcache,
                            const __nv_bfloat16* vcache, const DecState* st, float* merged, int splits, int mode,
                            cudaStream_t stream, bool pdl);

// Decode step, layer part 3: x += wo . merged.
cudaError_t launch_dec_oproj(const DecShape& s, bool int8, const float* merged, DecMatrix wo, float* x, int sm_count,
                             cudaStream_t stream, bool pdl);

// Final RMSNorm of row x, logits = lm_head . x (written when logits is
// non-null), greedy argmax (lowest id on a tie) over the blocks' partials by
// the last block: state.token = the choice. advance = 1 (a decode step):
// tokens[state.step] = choice, step + 1, pos + 1; advance = 0 (after a
// prefill of set_pos rows): tokens[0] = choice, step = 1, pos = set_pos.
// part: [grid] int2 partials; counter zero between launches.
cudaError_t launch_dec_lmhead(const DecShape& s, bool int8, const float* x, const float* norm, DecMatrix lm_head,
                              float* logits, DecState* st, int2* part, unsigned* counter, int* tokens, int advance,
                              int set_pos, int sm_count, cudaStream_t stream, bool pdl);

// Prefill rows: out[t] = bf16(RMSNorm(x[t]) * gain).
cudaError_t launch_norm_rows_bf16(const float* x, int64_t rows, int H, const float* gain, float eps,
                                  __nv_bfloat16* out, cudaStream_t stream);
// Prefill rows: qkv [rows, (heads + 2 kv) * 128] fp32 -> q (rotated, bf16
// [rows, heads * 128]) and the cache rows 0..rows-1 (k rotated).
cudaError_t launch_rope_rows(const DecShape& s, const float* qkv, int64_t rows, const float* inv_freq,
                             __nv_bfloat16* q, __nv_bfloat16* kcache, __nv_bfloat16* vcache, cudaStream_t stream);
// Prefill causal GQA attention over the cache rows 0..rows-1 (tensor-core
// mma.sync tiles, online softmax): out [rows, heads * 128] bf16.
cudaError_t launch_prefill_attn(const DecShape& s, const __nv_bfloat16* q, int64_t rows, const __nv_bfloat16* kcache,
                                const __nv_bfloat16* vcache, __nv_bfloat16* out, cudaStream_t stream);
// One-time per-device set-up of the decoder kernels' shared-memory limits.
cudaError_t prepare_decoder_kernels();

}  // namespace uocr_b200
