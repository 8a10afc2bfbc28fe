/* TEST INFRASTRUCTURE ONLY: CPU oracle for the decoder MoE hot path.
 * Every function cites the reference code it restates (paths are inside the
 * reference project). Build with -ffp-contract=off: the reference computes
 * every product and sum as a separately rounded IEEE operation. */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int pick_threads(int threads) {
#ifdef _OPENMP
  return threads > 0 ? threads : omp_get_num_procs();
#else
  (void)threads;
  return 1;
#endif
}

/* src/backend/reference/ops.cpp:25-38 — eight partial sums in a fixed order,
 * a tail, combined as a fixed tree. */
static float ref_dot(const float* a, const float* b, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    for (int lane = 0; lane < 8; ++lane) acc[lane] += a[i + lane] * b[i + lane];
  }
  float tail = 0.0f;
  for (; i < n; ++i) tail += a[i] * b[i];
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7])) + tail;
}

/* src/backend/reference/ops.cpp:91-109 (one row per task, like parallel_for over m). */
static void linear_rows(const float* x, int64_t m, int64_t k, const float* w, int64_t n, const float* bias, float* y,
                        int threads) {
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1 && m > 1)
  for (int64_t r = 0; r < m; ++r) {
    const float* xr = x + r * k;
    float* o = y + r * n;
    for (int64_t c = 0; c < n; ++c) {
      const float sum = ref_dot(xr, w + c * k, k);
      o[c] = bias != NULL ? sum + bias[c] : sum;
    }
  }
}

void oracle_linear(const float* x, int64_t m, int64_t k, const float* w, int64_t n, const float* bias, float* y,
                   int threads) {
  linear_rows(x, m, k, w, n, bias, y, pick_threads(threads));
}

/* src/backend/reference/ops.cpp:40 and :163-167: v * (1 / (1 + exp(-v))). */
static float ref_silu(float v) {
  const float s = 1.0f / (1.0f + expf(-v));
  return v * s;
}

/* src/model/feed_forward.cpp:18-24 — GatedMlp::forward on n rows. */
static void gated_mlp(const float* in, int64_t n, int64_t hidden, int64_t width, const float* gate, const float* up,
                      const float* down, float* out, int threads) {
  float* g = (float*)malloc(sizeof(float) * (size_t)(n * width));
  float* u = (float*)malloc(sizeof(float) * (size_t)(n * width));
  linear_rows(in, n, hidden, gate, width, NULL, g, threads);
  linear_rows(in, n, hidden, up, width, NULL, u, threads);
  for (int64_t i = 0; i < n * width; ++i) g[i] = ref_silu(g[i]);
  for (int64_t i = 0; i < n * width; ++i) g[i] *= u[i];
  linear_rows(g, n, width, down, hidden, NULL, out, threads);
  free(g);
  free(u);
}

/* src/backend/reference/ops.cpp:169-187 — max shift, float exp, double total,
 * multiply by float(1/total); an all -inf row becomes zeros. */
static void ref_softmax_row(float* v, int64_t c) {
  float peak = -INFINITY;
  for (int64_t i = 0; i < c; ++i) peak = peak < v[i] ? v[i] : peak; /* std::max(peak, v[i]) */
  if (peak == -INFINITY) {
    for (int64_t i = 0; i < c; ++i) v[i] = 0.0f;
    return;
  }
  double total = 0.0;
  for (int64_t i = 0; i < c; ++i) {
    v[i] = expf(v[i] - peak);
    total += v[i];
  }
  const float inv = (float)(1.0 / total);
  for (int64_t i = 0; i < c; ++i) v[i] *= inv;
}

/* src/model/feed_forward.cpp:43-48 — partial_sort by descending score, lower
 * index on a tie; the comparator is a total order, so k rounds of "best
 * remaining" give the same sequence. */
static void ref_topk(const float* s, int64_t e_count, int64_t k, int32_t* out) {
  for (int64_t j = 0; j < k; ++j) {
    int64_t best = -1;
    for (int64_t e = 0; e < e_count; ++e) {
      int taken = 0;
      for (int64_t q = 0; q < j; ++q) taken |= out[q] == e;
      if (taken) continue;
      if (best < 0 || s[e] > s[best]) best = e;  /* ties keep the lower index */
    }
    out[j] = (int32_t)best;
  }
}

int oracle_moe_forward(const oracle_moe_layer* L, const float* x, int64_t tokens, float* y, int32_t* ids_out,
                       float* weights_out, float* logits_out, float* margin_out, float* order_margin_out,
                       int threads) {
  if (L == NULL || x == NULL || y == NULL || tokens < 0 || L->hidden <= 0 || L->experts <= 0 || L->top_k <= 0 ||
      L->top_k > L->experts || L->ffn <= 0 || L->shared_ffn < 0)
    return 1;
  threads = pick_threads(threads);
  const int64_t H = L->hidden, E = L->experts, K = L->top_k, F = L->ffn, S = L->shared_ffn;

  /* feed_forward.cpp:38-39: scores = softmax(linear(x, gate)). */
  float* logits = (float*)malloc(sizeof(float) * (size_t)(tokens * E));
  float* scores = (float*)malloc(sizeof(float) * (size_t)(tokens * E));
  linear_rows(x, tokens, H, L->router, E, L->router_bias, logits, threads);
  memcpy(scores, logits, sizeof(float) * (size_t)(tokens * E));
  for (int64_t t = 0; t < tokens; ++t) ref_softmax_row(scores + t * E, E);

  /* feed_forward.cpp:41-54: per token its top-k experts and gate weights. */
  int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)(tokens * K));
  float* wsel = (float*)malloc(sizeof(float) * (size_t)(tokens * K));
  for (int64_t t = 0; t < tokens; ++t) {
    ref_topk(scores + t * E, E, K, sel + t * K);
    float sum = 0.0f;
    for (int64_t j = 0; j < K; ++j) {
      wsel[t * K + j] = scores[t * E + sel[t * K + j]];
      sum += wsel[t * K + j];
    }
    /* Renormalisation (absent in the reference, feed_forward.cpp:40): each
     * selected weight divided by the rank-order float sum of the k weights. */
    if (L->renormalize)
      for (int64_t j = 0; j < K; ++j) wsel[t * K + j] = wsel[t * K + j] / sum;
  }

  /* Routing lists in token order per expert (feed_forward.cpp:49-53). */
  int64_t* count = (int64_t*)calloc((size_t)E, sizeof(int64_t));
  for (int64_t i = 0; i < tokens * K; ++i) count[sel[i]]++;
  int64_t* start = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
  start[0] = 0;
  for (int64_t e = 0; e < E; ++e) start[e + 1] = start[e] + count[e];
  int64_t* tok_of = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tokens * K + 1));
  float* w_of = (float*)malloc(sizeof(float) * (size_t)(tokens * K + 1));
  int64_t* fill = (int64_t*)calloc((size_t)E, sizeof(int64_t));
  for (int64_t t = 0; t < tokens; ++t)
    for (int64_t j = 0; j < K; ++j) {
      const int64_t e = sel[t * K + j];
      const int64_t p = start[e] + fill[e]++;
      tok_of[p] = t;
      w_of[p] = wsel[t * K + j];
    }

  /* feed_forward.cpp:57-64: each expert over its rows, experts in parallel,
   * the linears inside an expert serial (parallel.h:26-31). */
  float* outs = (float*)malloc(sizeof(float) * (size_t)((tokens * K + 1) * H));
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads) if (threads > 1)
  for (int64_t e = 0; e < E; ++e) {
    const int64_t n = count[e];
    if (n == 0) continue;
    float* in = (float*)malloc(sizeof(float) * (size_t)(n * H));
    for (int64_t i = 0; i < n; ++i) memcpy(in + i * H, x + tok_of[start[e] + i] * H, sizeof(float) * (size_t)H);
    gated_mlp(in, n, H, F, L->gate + e * F * H, L->up + e * F * H, L->down + e * H * F, outs + start[e] * H, 1);
    free(in);
  }

  /* feed_forward.cpp:65-76: shared expert, routed sum in expert order, add. */
  if (S > 0) {
    gated_mlp(x, tokens, H, S, L->shared_gate, L->shared_up, L->shared_down, y, threads);
  } else {
    memset(y, 0, sizeof(float) * (size_t)(tokens * H));
  }
  float* routed = (float*)calloc((size_t)(tokens * H), sizeof(float));
  for (int64_t e = 0; e < E; ++e)
    for (int64_t i = 0; i < count[e]; ++i) {
      const float w = w_of[start[e] + i];
      const float* src = outs + (start[e] + i) * H;
      float* dst = routed + tok_of[start[e] + i] * H;
      for (int64_t c = 0; c < H; ++c) dst[c] += w * src[c];
    }
  for (int64_t i = 0; i < tokens * H; ++i) y[i] += routed[i];

  for (int64_t t = 0; t < tokens; ++t) {
    const float* lg = logits + t * E;
    const int32_t* s = sel + t * K;
    float best_rest = -INFINITY;
    for (int64_t e = 0; e < E; ++e) {
      int taken = 0;
      for (int64_t j = 0; j < K; ++j) taken |= s[j] == e;
      if (!taken && lg[e] > best_rest) best_rest = lg[e];
    }
    const float m = lg[s[K - 1]] - best_rest;
    float om = m;
    for (int64_t j = 0; j + 1 < K; ++j) {
      const float gap = lg[s[j]] - lg[s[j + 1]];
      if (gap < om) om = gap;
    }
    if (margin_out) margin_out[t] = m;
    if (order_margin_out) order_margin_out[t] = om;
  }
  if (ids_out) memcpy(ids_out, sel, sizeof(int32_t) * (size_t)(tokens * K));
  if (weights_out) memcpy(weights_out, wsel, sizeof(float) * (size_t)(tokens * K));
  if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)(tokens * E));

  free(logits);
  free(scores);
  free(sel);
  free(wsel);
  free(count);
  free(start);
  free(tok_of);
  free(w_of);
  free(fill);
  free(outs);
  free(routed);
  return 0;
}

/* src/model/cuda/device_weight.cpp:11-26 with the group size free. */
int oracle_quantize_q8(const float* w, int64_t rows, int64_t cols, int64_t group, int8_t* q, float* scales) {
  if (group <= 0 || cols % group != 0) return 1;
  const int64_t groups = cols / group;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      const float* src = w + r * cols + g * group;
      float peak = 0.0f;
      for (int64_t i = 0; i < group; ++i) peak = fabsf(src[i]) > peak ? fabsf(src[i]) : peak;
      const float scale = peak > 0.0f ? peak / 127.0f : 1.0f;
      scales[r * groups + g] = scale;
      for (int64_t i = 0; i < group; ++i) {
        float v = nearbyintf(src[i] / scale);
        v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
        q[r * cols + g * group + i] = (int8_t)v;
      }
    }
  return 0;
}

void oracle_dequantize_q8(const int8_t* q, const float* scales, int64_t rows, int64_t cols, int64_t group,
                          float* w) {
  const int64_t groups = cols / group;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) w[r * cols + c] = (float)q[r * cols + c] * scales[r * groups + c / group];
}

/* src/tensor/dtype.h:39-46 (f32_to_bf16) followed by :33-35 (bf16_to_f32). */
void oracle_round_bf16(float* v, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t bits;
    memcpy(&bits, &v[i], 4);
    uint16_t h;
    if ((bits & 0x7fffffffU) > 0x7f800000U) {
      h = (uint16_t)((bits >> 16) | 0x0040U);
    } else {
      const uint32_t rounding = 0x7fffU + ((bits >> 16) & 1U);
      h = (uint16_t)((bits + rounding) >> 16);
    }
    bits = (uint32_t)h << 16;
    memcpy(&v[i], &bits, 4);
  }
}

/* ---- synthetic inputs -------------------------------------------------- */

static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

uint64_t oracle_synth_stream(uint64_t layer, uint64_t kind, uint64_t index) {
  return (layer << 40) | (kind << 32) | index;
}

/* value(i) = sigma * ((S + 6) / 65536 - 6), S the sum of twelve 16-bit words
 * of three hashes of (stream key, i). (S + 6) / 65536 - 6 is exact in fp32
 * (fewer than 20 significant bits), so the only rounding is the product with
 * sigma: host and device produce the same bits. */
void oracle_synth_fill(uint64_t seed, uint64_t stream, float sigma, int64_t offset, int64_t n, float* out,
                       int threads) {
  const uint64_t golden = 0x9E3779B97F4A7C15ULL;
  const uint64_t key = mix64(seed * golden + stream);
  threads = pick_threads(threads);
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1 && n > 65536)
  for (int64_t j = 0; j < n; ++j) {
    const uint64_t i = (uint64_t)(offset + j);
    uint32_t s = 0;
    for (uint64_t w = 0; w < 3; ++w) {
      const uint64_t h = mix64(key + (3 * i + w + 1) * golden);
      s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) + (uint32_t)((h >> 32) & 0xffff) +
           (uint32_t)(h >> 48);
    }
    const float centred = (float)(s + 6u) * (1.0f / 65536.0f) - 6.0f;
    out[j] = centred * sigma;
  }
}
