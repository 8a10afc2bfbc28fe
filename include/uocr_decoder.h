/* uocr_decoder.h — C ABI of the synthetic page decoder around the B200 MoE.
 *
 * A decoder stack on one GPU: per layer RMSNorm, grouped-query attention
 * (head dim 128, rotate-half RoPE, a bf16 KV cache), and the MoE
 * feed-forward block of uocr_moe.h behind its own RMSNorm; then the final
 * norm, lm_head and greedy token selection. It stands for the reference's
 * CudaDecoder (src/model/cuda/cuda_decoder.h:25-104) with its decode body
 * (src/model/cuda/cuda_decode_step.cpp:47-70, captured as one CUDA graph as
 * in src/model/cuda/cuda_decoder.cpp:300-329) and prefill, driven the way
 * generate_from_embeddings drives it (src/runtime/generator.cpp:41-84): a
 * prefill of embedding rows gives the first token, then each decode step
 * consumes the last token and yields the next (greedy, lowest id on a tie).
 * The reference decoder uses multi-head attention with its own block router
 * and a two-axis PageRope; this one has the grouped-query attention and plain
 * RoPE the benchmark configuration names, and no block router.
 *
 * Conventions are uocr_moe.h's: plain pointers, a cudaStream_t passed as
 * void*, status codes with uocr_last_error(), nothing synchronises the stream
 * except uocr_decoder_check and the measurement call
 * uocr_decoder_profile_decode.
 */
#ifndef UOCR_DECODER_H
#define UOCR_DECODER_H

#include <stdint.h>

#include "uocr_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct uocr_decoder uocr_decoder;

typedef struct uocr_decoder_desc {
  int64_t hidden;            /* model width H (a multiple of 256) */
  int64_t layers;
  int64_t heads;             /* query heads; heads * head_dim == hidden */
  int64_t kv_heads;          /* key/value heads: heads % kv_heads == 0, at most 8 query heads per kv head */
  int64_t head_dim;          /* 128 */
  int64_t vocab;
  int64_t max_positions;     /* KV cache length: prefill rows + decode steps of one sequence */
  int64_t max_prefill;       /* rows of one prefill call */
  int64_t routed_experts;    /* MoE block: as uocr_moe_desc */
  int64_t experts_per_token;
  int64_t expert_ffn;
  int64_t shared_ffn;
  float rope_theta;          /* RoPE base (1e4) */
  float rms_norm_eps;
  int32_t weight_format;     /* uocr_weight_format: bf16, or per-output-channel int8 for every projection */
  int32_t renormalize;       /* MoE top-k weights divided by their sum */
  int32_t device;
  int32_t flags;             /* UOCR_DECODER_* bits */
} uocr_decoder_desc;

/* The decode attention's products on the CUDA cores instead of the tensor
 * cores (the default wherever a split's K and V rows fit in shared memory). */
#define UOCR_DECODER_CUDA_CORE_ATTENTION 1

/* One layer's weights, fp32 or bf16 (dtype), host or device (memory); the
 * norm gains and the router are fp32. They are converted on the device to
 * the decoder's format (bf16, or int8 with one fp32 scale per row). */
typedef struct uocr_decoder_layer_src {
  int32_t memory;            /* uocr_memory of every pointer below */
  int32_t dtype;             /* uocr_dtype of the matrices */
  const float* input_norm;   /* [H] gain of the norm in front of attention */
  const void* wq;            /* [heads * 128, H] */
  const void* wk;            /* [kv_heads * 128, H] */
  const void* wv;            /* [kv_heads * 128, H] */
  const void* wo;            /* [H, heads * 128] */
  const float* post_norm;    /* [H] gain of the norm in front of the MoE block */
  const float* router;       /* [E, H] */
  const void* gate;          /* [E * F, H] */
  const void* up;            /* [E * F, H] */
  const void* down;          /* [E * H, F] */
  const void* shared_gate;   /* [S, H] */
  const void* shared_up;     /* [S, H] */
  const void* shared_down;   /* [H, S] */
} uocr_decoder_layer_src;

int uocr_decoder_create(const uocr_decoder_desc* desc, uocr_decoder** out);
int uocr_decoder_destroy(uocr_decoder* dec);
/* Bytes of device memory held: weights, KV cache and scratch. */
int uocr_decoder_bytes(const uocr_decoder* dec, int64_t* weight_bytes, int64_t* other_bytes);

int uocr_decoder_set_layer(uocr_decoder* dec, int64_t layer, const uocr_decoder_layer_src* src, void* stream);
/* The token embedding [vocab, H] (kept in bf16), the final norm gain [H]
 * (fp32) and lm_head [vocab, H] (in the decoder's format). */
int uocr_decoder_set_head(uocr_decoder* dec, int32_t memory, int32_t dtype, const void* embed,
                          const float* final_norm, const void* lm_head, void* stream);

/* Starts a sequence: rows fp32 embedding rows [rows, H] (device memory) at
 * positions 0..rows-1 fill the KV cache; the last row's logits pick the
 * first token. logits (device [vocab]) and token (device int32) receive
 * them when non-null. */
int uocr_decoder_prefill(uocr_decoder* dec, const float* embeds, int64_t rows, float* logits, int32_t* token,
                         void* stream);
/* `steps` greedy decode steps, each consuming the current token at the next
 * position: tokens (device int32 [steps]) receives the tokens they produce,
 * logits (device fp32 [steps, vocab]) each step's logits when non-null. The
 * step replays a CUDA graph captured on the first call for the stream (plain
 * launches on a capturing or legacy stream). UOCR_ERR_INVALID_ARGUMENT when
 * the sequence would pass max_positions or no prefill started it. */
int uocr_decoder_decode(uocr_decoder* dec, int64_t steps, int32_t* tokens, float* logits, void* stream);
/* Measurement: `steps` decode steps with plain launches and events between
 * the phases (synchronises after each step); ms[0..4] receive the mean time
 * per step of the q/k/v kernels, attention, the output projections, the MoE
 * blocks (all layers summed) and lm_head. Advances the sequence like
 * uocr_decoder_decode. */
int uocr_decoder_profile_decode(uocr_decoder* dec, int64_t steps, float* ms, void* stream);
/* Synchronises the stream and reports device errors recorded by the
 * decoder's kernels or its MoE block (UOCR_ERR_DEVICE / UOCR_ERR_TIMEOUT). */
int uocr_decoder_check(uocr_decoder* dec, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* UOCR_DECODER_H */
