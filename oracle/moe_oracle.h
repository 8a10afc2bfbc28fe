/* TEST INFRASTRUCTURE ONLY: the CPU oracle for the decoder MoE hot path.
 *
 * Plain-C restatement of the reference's fp32 mixture-of-experts
 * (src/model/feed_forward.cpp:36-78 over src/backend/reference/ops.cpp),
 * extended with the three switches the synthetic configurations need:
 * top-k weight renormalisation, an additive router bias, and int8
 * per-output-channel weights (run as their dequantised fp32 values).
 * Only tests, the smoke check and bench.py's CPU baseline may load it; the
 * product library never links or calls it.
 *
 * Pinning: with renormalize = 0 and no bias the output is bit-identical to
 * the reference's own MixtureOfExperts::forward compiled from its sources
 * (oracle/_ref, tests/test_oracle.py), and the committed golden vectors in
 * tests/golden/ were produced by that reference build. */
#ifndef UOCR_MOE_ORACLE_H
#define UOCR_MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int64_t hidden, experts, top_k, ffn, shared_ffn;
  int32_t renormalize;        /* 0: raw softmax probabilities (reference); 1: divided by their top-k sum */
  const float* router;        /* [E, H] */
  const float* router_bias;   /* [E] or NULL */
  const float* gate;          /* [E*F, H] */
  const float* up;            /* [E*F, H] */
  const float* down;          /* [E*H, F] */
  const float* shared_gate;   /* [S, H] (unused when shared_ffn == 0) */
  const float* shared_up;     /* [S, H] */
  const float* shared_down;   /* [H, S] */
} oracle_moe_layer;

/* y [T,H] = MoE(x [T,H]). Optional outputs (NULL to skip):
 *   ids [T,k] int32 in rank order (descending score, lower id on a tie),
 *   weights [T,k] the combine weights in the same order,
 *   logits [T,E] the router logits (bias included) before the softmax,
 *   margin [T] logit(k-th selected) - max logit over the unselected experts,
 *   order_margin [T] the smallest logit gap between adjacent ranks 1..k+1.
 * threads <= 0 uses every core. Returns 0, or 1 on a bad argument. */
int oracle_moe_forward(const oracle_moe_layer* layer, const float* x, int64_t tokens, float* y, int32_t* ids,
                       float* weights, float* logits, float* margin, float* order_margin, int threads);

/* Reference fp32 `linear` (ops.cpp:91-109): y[m,n] = x[m,k] . w[n,k] (+ bias[n]). */
void oracle_linear(const float* x, int64_t m, int64_t k, const float* w, int64_t n, const float* bias, float* y,
                   int threads);

/* Symmetric round-to-nearest int8 with one fp32 scale per `group` inputs of a
 * row (device_weight.cpp:11-26 restated with a free group size; group = cols
 * is per-output-channel). scales [rows, cols/group]. Returns 1 on a bad group. */
int oracle_quantize_q8(const float* w, int64_t rows, int64_t cols, int64_t group, int8_t* q, float* scales);

/* Dequantised weights q*scale, as the reference test builds them
 * (tests/cuda_decoder_test.cpp:61-87). */
void oracle_dequantize_q8(const int8_t* q, const float* scales, int64_t rows, int64_t cols, int64_t group,
                          float* w);

/* fp32 -> bf16 -> fp32 round trip, round to nearest even, NaN kept quiet
 * (src/tensor/dtype.h:39-46 then :33-35). */
void oracle_round_bf16(float* v, int64_t n);

/* The synthetic generator the configurations use: a counter-based stream,
 * value(i) = sigma * (sum of twelve 16-bit uniforms, centred), identical on
 * host and device. stream() names one tensor of one layer. */
uint64_t oracle_synth_stream(uint64_t layer, uint64_t kind, uint64_t index);
void oracle_synth_fill(uint64_t seed, uint64_t stream, float sigma, int64_t offset, int64_t n, float* out,
                       int threads);

#ifdef __cplusplus
}
#endif
#endif
