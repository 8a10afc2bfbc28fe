// C ABI of the page decoder (include/uocr_decoder.h): weights, KV cache and
// scratch sized at creation; prefill and graph-replayed decode steps. Host
// code only; the kernels are in decoder.cu, the MoE block is a uocr_moe_plan.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "../../include/uocr_decoder.h"
#include "decoder.h"
#include "moe_kernels.h"
#include "plan_internal.h"
#include "tc_gemm.h"

using namespace uocr_b200;

namespace {

int dfail(int code, const std::string& what) { return set_last_error(code, what); }

int dcuda(cudaError_t st, const char* what) {
  return dfail(st == cudaErrorMemoryAllocation ? UOCR_ERR_OUT_OF_MEMORY : UOCR_ERR_CUDA,
               std::string(what) + ": " + cudaGetErrorString(st));
}

#define DEC_TRY(expr, what)                              \
  do {                                                   \
    cudaError_t st_ = (expr);                            \
    if (st_ != cudaSuccess) return dcuda(st_, what);     \
  } while (0)

#define DEC_RC(expr)                  \
  do {                                \
    int rc_ = (expr);                 \
    if (rc_ != UOCR_OK) return rc_;   \
  } while (0)

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

class Guard {
 public:
  explicit Guard(int device) {
    cudaGetDevice(&prev_);
    cudaSetDevice(device);
  }
  ~Guard() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

struct DecLayer {
  void* block = nullptr;
  float* input_norm = nullptr;
  void* wqkv = nullptr;
  float* wqkv_s = nullptr;
  void* wo = nullptr;
  float* wo_s = nullptr;
  bool loaded = false;
};

}  // namespace

struct uocr_decoder {
  uocr_decoder_desc d{};
  DecShape shape{};
  bool int8 = false;
  int sm_count = 1;
  int splits = 1;        // attention blocks (one cluster) per key/value head
  int attn_mode = 0;     // DecAttnMode of the decode attention
  int64_t qkv_rows = 0;  // (heads + 2 kv) * 128
  uocr_moe_plan* moe = nullptr;
  std::vector<DecLayer> layers;
  void* head_block = nullptr;
  __nv_bfloat16* embed = nullptr;
  float* final_norm = nullptr;
  void* lm_head = nullptr;
  float* lm_head_s = nullptr;
  bool head_loaded = false;
  // arena
  void* arena = nullptr;
  size_t arena_bytes = 0;
  size_t weight_bytes = 0;
  float* x = nullptr;             // [max_prefill, H] residual stream (a decode step uses row 0)
  float* q = nullptr;             // [heads * 128]
  float* merged = nullptr;        // [heads * 128] attention output (bf16 values)
  unsigned* counters = nullptr;   // the lm_head's ticket
  int2* lm_part = nullptr;        // [sm_count]
  float* logits = nullptr;        // [vocab]
  DecState* state = nullptr;
  int* tokens = nullptr;          // [max_positions]
  float* inv_freq = nullptr;      // [64]
  __nv_bfloat16* kcache = nullptr;  // [layers][kv][max_pos][128]
  __nv_bfloat16* vcache = nullptr;
  __nv_bfloat16* xn = nullptr;    // [max_prefill, H]
  float* qkv = nullptr;           // [max_prefill, qkv_rows]
  __nv_bfloat16* qb = nullptr;    // [max_prefill, heads * 128]
  __nv_bfloat16* attn = nullptr;  // [max_prefill, heads * 128]
  __nv_bfloat16* wexp = nullptr;  // int8 prefill: one projection expanded to bf16
  ErrorWord* err = nullptr;
  // host mirrors of the sequence
  int64_t length = 0;     // positions in the KV cache
  int64_t generated = 0;  // tokens chosen so far
  bool started = false;
  // the captured decode step
  cudaGraphExec_t graph = nullptr;
  cudaStream_t graph_stream = nullptr;
};

namespace {

__nv_bfloat16* kc_of(const uocr_decoder* p, int64_t layer) {
  return p->kcache + layer * p->d.kv_heads * p->d.max_positions * kDecHeadDim;
}
__nv_bfloat16* vc_of(const uocr_decoder* p, int64_t layer) {
  return p->vcache + layer * p->d.kv_heads * p->d.max_positions * kDecHeadDim;
}

// One matrix [rows, cols] from (memory, dtype) into bf16, or int8 with row
// scales: a host source goes through a staging buffer.
int convert_matrix(int32_t memory, int32_t dtype, const void* from, int64_t rows, int64_t cols, bool int8, void* dst,
                   float* scales, cudaStream_t stream, const char* name) {
  if (from == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, std::string("decoder: missing ") + name);
  if (dtype != UOCR_DTYPE_F32 && dtype != UOCR_DTYPE_BF16)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder: matrices must be fp32 or bf16");
  const size_t eb = dtype == UOCR_DTYPE_BF16 ? 2 : 4;
  const size_t n = static_cast<size_t>(rows * cols);
  const void* src = from;
  void* staging = nullptr;
  if (memory == UOCR_MEMORY_HOST) {
    DEC_TRY(cudaMallocAsync(&staging, n * eb, stream), "decoder: staging allocation");
    cudaError_t up = cudaMemcpyAsync(staging, from, n * eb, cudaMemcpyHostToDevice, stream);
    if (up != cudaSuccess) {
      cudaFreeAsync(staging, stream);
      return dcuda(up, "decoder: upload");
    }
    src = staging;
  }
  cudaError_t st;
  if (int8)
    st = launch_quantize_rows(src, dtype == UOCR_DTYPE_BF16, rows, cols, cols, static_cast<int8_t*>(dst), scales,
                              stream);
  else if (dtype == UOCR_DTYPE_BF16)
    st = cudaMemcpyAsync(dst, src, n * 2, cudaMemcpyDeviceToDevice, stream);
  else
    st = launch_f32_to_bf16(static_cast<const float*>(src), static_cast<__nv_bfloat16*>(dst),
                            static_cast<int64_t>(n), stream);
  if (staging != nullptr) cudaFreeAsync(staging, stream);
  if (st != cudaSuccess) return dcuda(st, "decoder: conversion");
  if (memory == UOCR_MEMORY_HOST) DEC_TRY(cudaStreamSynchronize(stream), "decoder: upload wait");
  return UOCR_OK;
}

int copy_gain(int32_t memory, const float* from, float* dst, int64_t n, cudaStream_t stream, const char* name) {
  if (from == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, std::string("decoder: missing ") + name);
  DEC_TRY(cudaMemcpyAsync(dst, from, static_cast<size_t>(n) * 4,
                          memory == UOCR_MEMORY_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, stream),
          "decoder: gain copy");
  return UOCR_OK;
}

size_t matrix_bytes(int64_t rows, int64_t cols, bool int8) {
  return up256(static_cast<size_t>(rows * cols) * (int8 ? 1 : 2)) + (int8 ? up256(static_cast<size_t>(rows) * 4) : 0);
}

// A plain GEMM on the tcgen05 grouped kernel (its shared group): out [m, n]
// fp32 = a [m, k] . b [n, k]^T, or out += that with accumulate.
cudaError_t gemm(const uocr_decoder* p, const __nv_bfloat16* a, int64_t m, int64_t k, const __nv_bfloat16* b,
                 int64_t n, float* out, bool accumulate, cudaStream_t stream) {
  GroupedGemm g{};
  g.mode = 1;
  g.experts = 0;
  g.k_routed = 64;
  g.n_cols_routed = 256;
  g.shared_rows = static_cast<int>(m);
  g.a_shared = a;
  g.k_shared = static_cast<int>(k);
  g.b0_shared = b;
  g.b1_shared = b;
  g.b_shared_rows = n;
  g.n_cols_shared = static_cast<int>(n);
  g.out_shared = out;
  g.ld_out_shared = n;
  g.shared_out_f32 = true;
  g.shared_accumulate = accumulate;
  g.err = p->err;
  g.blocks = p->sm_count;
  return launch_grouped_gemm(g, stream);
}

// The matrix as the prefill GEMM reads it: bf16 as stored, int8 expanded.
const __nv_bfloat16* gemm_operand(const uocr_decoder* p, const void* w, const float* s, int64_t rows, int64_t cols,
                                  cudaStream_t stream, cudaError_t* st) {
  if (!p->int8) return static_cast<const __nv_bfloat16*>(w);
  *st = launch_dequant_rows(static_cast<const int8_t*>(w), s, rows, cols, p->wexp, stream);
  return p->wexp;
}

// One decode step: every layer (norm + q/k/v + RoPE + cache, attention,
// output projection, the MoE block) and the head with the greedy choice. For
// measurement, ev (kProfilePhases + 1 events per layer slot) receives an event
// before the first kernel and after each phase, and the launches are plain
// (no programmatic overlap) so that the events bracket each phase.
constexpr int kProfilePhases = 4;  // q/k/v, attention, output projection, MoE block

int decode_step(uocr_decoder* p, cudaStream_t stream, cudaEvent_t* ev = nullptr) {
  const DecShape& s = p->shape;
  const bool pdl = ev == nullptr;
  auto mark = [&](int64_t l, int k) -> cudaError_t {
    return ev != nullptr ? cudaEventRecord(ev[l * (kProfilePhases + 1) + k], stream) : cudaSuccess;
  };
  for (int64_t l = 0; l < p->d.layers; ++l) {
    const DecLayer& L = p->layers[static_cast<size_t>(l)];
    DEC_TRY(mark(l, 0), "decode: event");
    DEC_TRY(launch_dec_qkv(s, p->int8, p->x, l == 0 ? p->embed : nullptr, L.input_norm, DecMatrix{L.wqkv, L.wqkv_s},
                           p->inv_freq, p->state, p->q, kc_of(p, l), vc_of(p, l), p->sm_count, stream, pdl),
            "decode: q/k/v");
    DEC_TRY(mark(l, 1), "decode: event");
    DEC_TRY(launch_dec_attn(s, p->q, kc_of(p, l), vc_of(p, l), p->state, p->merged, p->splits, p->attn_mode, stream,
                            pdl),
            "decode: attention");
    DEC_TRY(mark(l, 2), "decode: event");
    DEC_TRY(launch_dec_oproj(s, p->int8, p->merged, DecMatrix{L.wo, L.wo_s}, p->x, p->sm_count, stream, pdl),
            "decode: output projection");
    DEC_TRY(mark(l, 3), "decode: event");
    DEC_RC(moe_layer_inplace(p->moe, l, p->x, 1, stream));
    DEC_TRY(mark(l, 4), "decode: event");
  }
  DEC_TRY(launch_dec_lmhead(s, p->int8, p->x, p->final_norm, DecMatrix{p->lm_head, p->lm_head_s}, p->logits, p->state,
                            p->lm_part, p->counters, p->tokens, 1, 0, p->sm_count, stream, pdl),
          "decode: lm_head");
  if (ev != nullptr) DEC_TRY(cudaEventRecord(ev[p->d.layers * (kProfilePhases + 1)], stream), "decode: event");
  return UOCR_OK;
}

}  // namespace

extern "C" {

int uocr_decoder_create(const uocr_decoder_desc* desc, uocr_decoder** out) {
  if (desc == nullptr || out == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_create: null argument");
  *out = nullptr;
  const uocr_decoder_desc& d = *desc;
  if (d.head_dim != kDecHeadDim) return dfail(UOCR_ERR_UNSUPPORTED, "decoder_create: head_dim must be 128");
  if (d.heads <= 0 || d.kv_heads <= 0 || d.heads % d.kv_heads != 0 || d.heads / d.kv_heads > kDecMaxGroup)
    return dfail(UOCR_ERR_INVALID_ARGUMENT,
                 "decoder_create: heads must be a positive multiple of kv_heads, at most 8 per kv head");
  if (d.hidden != d.heads * d.head_dim || d.hidden % 256 != 0 || d.hidden > 8192)
    return dfail(UOCR_ERR_INVALID_ARGUMENT,
                 "decoder_create: hidden must equal heads * head_dim, be a multiple of 256 and at most 8192");
  if ((d.heads + 2 * d.kv_heads) % 2 != 0)
    return dfail(UOCR_ERR_UNSUPPORTED, "decoder_create: heads + 2 * kv_heads must be even");
  if (d.layers <= 0 || d.vocab <= 1 || d.vocab > (1 << 30) || d.max_prefill <= 0 ||
      d.max_positions <= d.max_prefill || d.max_positions > (1 << 24))
    return dfail(UOCR_ERR_INVALID_ARGUMENT,
                 "decoder_create: need layers > 0, vocab > 1, 0 < max_prefill < max_positions");
  if (d.weight_format != UOCR_WEIGHT_BF16 && d.weight_format != UOCR_WEIGHT_INT8)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_create: weight_format must be bf16 or int8");
  if (!(d.rope_theta > 0.0f) || !(d.rms_norm_eps >= 0.0f))
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_create: rope_theta > 0, rms_norm_eps >= 0");
  Guard guard(d.device);
  auto* p = new uocr_decoder;
  p->d = d;
  p->int8 = d.weight_format == UOCR_WEIGHT_INT8;
  p->shape = DecShape{static_cast<int>(d.hidden), static_cast<int>(d.heads), static_cast<int>(d.kv_heads),
                      static_cast<int>(d.vocab), static_cast<int>(d.max_positions), d.rms_norm_eps};
  p->qkv_rows = (d.heads + 2 * d.kv_heads) * kDecHeadDim;
  int sms = 0;
  cudaError_t st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d.device);
  if (st == cudaSuccess) st = prepare_decoder_kernels();
  if (st == cudaSuccess)
    st = plan_dec_attn(p->shape, (d.flags & UOCR_DECODER_CUDA_CORE_ATTENTION) != 0, &p->splits, &p->attn_mode);
  if (st != cudaSuccess) {
    delete p;
    return dcuda(st, "decoder_create: device set-up");
  }
  p->sm_count = sms > 0 ? sms : 1;

  uocr_moe_desc md{};
  md.hidden = d.hidden;
  md.routed_experts = d.routed_experts;
  md.experts_per_token = d.experts_per_token;
  md.expert_ffn = d.expert_ffn;
  md.shared_ffn = d.shared_ffn;
  md.layers = d.layers;
  md.max_rows = std::max<int64_t>(d.max_prefill, 1);
  md.weight_format = d.weight_format;
  md.renormalize = d.renormalize;
  md.device = d.device;
  md.flags = UOCR_PLAN_PRE_NORM | UOCR_PLAN_NO_GRAPHS;
  md.rms_norm_eps = d.rms_norm_eps;
  int rc = uocr_moe_plan_create(&md, &p->moe);
  if (rc != UOCR_OK) {
    delete p;
    return rc;
  }

  const int64_t H = d.hidden, A = d.heads * kDecHeadDim, R = d.max_prefill;
  p->layers.resize(static_cast<size_t>(d.layers));
  const size_t layer_bytes = up256(static_cast<size_t>(H) * 4) * 1 + matrix_bytes(p->qkv_rows, H, p->int8) +
                             matrix_bytes(H, A, p->int8);
  for (auto& L : p->layers) {
    st = cudaMalloc(&L.block, layer_bytes);
    if (st != cudaSuccess) {
      uocr_decoder_destroy(p);
      return dcuda(st, "decoder_create: layer allocation");
    }
    char* c = static_cast<char*>(L.block);
    L.input_norm = reinterpret_cast<float*>(c);
    c += up256(static_cast<size_t>(H) * 4);
    L.wqkv = c;
    c += up256(static_cast<size_t>(p->qkv_rows * H) * (p->int8 ? 1 : 2));
    if (p->int8) {
      L.wqkv_s = reinterpret_cast<float*>(c);
      c += up256(static_cast<size_t>(p->qkv_rows) * 4);
    }
    L.wo = c;
    c += up256(static_cast<size_t>(H * A) * (p->int8 ? 1 : 2));
    if (p->int8) L.wo_s = reinterpret_cast<float*>(c);
    p->weight_bytes += layer_bytes;
  }
  const size_t head_bytes = up256(static_cast<size_t>(d.vocab * H) * 2) + up256(static_cast<size_t>(H) * 4) +
                            matrix_bytes(d.vocab, H, p->int8);
  st = cudaMalloc(&p->head_block, head_bytes);
  if (st != cudaSuccess) {
    uocr_decoder_destroy(p);
    return dcuda(st, "decoder_create: head allocation");
  }
  {
    char* c = static_cast<char*>(p->head_block);
    p->embed = reinterpret_cast<__nv_bfloat16*>(c);
    c += up256(static_cast<size_t>(d.vocab * H) * 2);
    p->final_norm = reinterpret_cast<float*>(c);
    c += up256(static_cast<size_t>(H) * 4);
    p->lm_head = c;
    c += up256(static_cast<size_t>(d.vocab * H) * (p->int8 ? 1 : 2));
    if (p->int8) p->lm_head_s = reinterpret_cast<float*>(c);
    p->weight_bytes += head_bytes;
  }
  const int64_t cache = d.layers * d.kv_heads * d.max_positions * kDecHeadDim;
  const size_t sizes[] = {
      static_cast<size_t>(R * H) * 4,                                     // x
      static_cast<size_t>(A) * 4,                                         // q
      static_cast<size_t>(A) * 4,                                         // merged
      static_cast<size_t>(4),                                             // counters
      static_cast<size_t>(p->sm_count) * 8,                               // lm_part
      static_cast<size_t>(d.vocab) * 4,                                   // logits
      sizeof(DecState),                                                   // state
      static_cast<size_t>(d.max_positions) * 4,                           // tokens
      static_cast<size_t>(kDecHeadDim / 2) * 4,                           // inv_freq
      static_cast<size_t>(cache) * 2,                                     // kcache
      static_cast<size_t>(cache) * 2,                                     // vcache
      static_cast<size_t>(R * H) * 2,                                     // xn
      static_cast<size_t>(R * p->qkv_rows) * 4,                           // qkv
      static_cast<size_t>(R * A) * 2,                                     // qb
      static_cast<size_t>(R * A) * 2,                                     // attn
      p->int8 ? static_cast<size_t>(std::max(p->qkv_rows * H, H * A)) * 2 : 0,  // wexp
      sizeof(ErrorWord)};
  size_t total = 0;
  for (size_t v : sizes) total += up256(v);
  st = cudaMalloc(&p->arena, total);
  if (st == cudaSuccess) st = cudaMemset(p->arena, 0, total);
  if (st != cudaSuccess) {
    uocr_decoder_destroy(p);
    return dcuda(st, "decoder_create: scratch allocation");
  }
  p->arena_bytes = total;
  {
    char* c = static_cast<char*>(p->arena);
    size_t i = 0;
    auto take = [&](void** dst) {
      *dst = c;
      c += up256(sizes[i++]);
    };
    take(reinterpret_cast<void**>(&p->x));
    take(reinterpret_cast<void**>(&p->q));
    take(reinterpret_cast<void**>(&p->merged));
    take(reinterpret_cast<void**>(&p->counters));
    take(reinterpret_cast<void**>(&p->lm_part));
    take(reinterpret_cast<void**>(&p->logits));
    take(reinterpret_cast<void**>(&p->state));
    take(reinterpret_cast<void**>(&p->tokens));
    take(reinterpret_cast<void**>(&p->inv_freq));
    take(reinterpret_cast<void**>(&p->kcache));
    take(reinterpret_cast<void**>(&p->vcache));
    take(reinterpret_cast<void**>(&p->xn));
    take(reinterpret_cast<void**>(&p->qkv));
    take(reinterpret_cast<void**>(&p->qb));
    take(reinterpret_cast<void**>(&p->attn));
    take(reinterpret_cast<void**>(&p->wexp));
    take(reinterpret_cast<void**>(&p->err));
  }
  // RoPE frequencies: float(1 / theta^(i / 64)) in double, as PageRope
  // builds its table (src/model/page_rope.cpp:18-20), over all 64 pairs.
  std::vector<float> inv(kDecHeadDim / 2);
  for (int i = 0; i < kDecHeadDim / 2; ++i)
    inv[static_cast<size_t>(i)] =
        static_cast<float>(1.0 / std::pow(static_cast<double>(d.rope_theta), static_cast<double>(i) / (kDecHeadDim / 2)));
  st = cudaMemcpy(p->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice);
  if (st != cudaSuccess) {
    uocr_decoder_destroy(p);
    return dcuda(st, "decoder_create: rope table");
  }
  *out = p;
  return UOCR_OK;
}

int uocr_decoder_destroy(uocr_decoder* p) {
  if (p == nullptr) return UOCR_OK;
  Guard guard(p->d.device);
  if (p->graph != nullptr) cudaGraphExecDestroy(p->graph);
  for (auto& L : p->layers)
    if (L.block != nullptr) cudaFree(L.block);
  if (p->head_block != nullptr) cudaFree(p->head_block);
  if (p->arena != nullptr) cudaFree(p->arena);
  if (p->moe != nullptr) uocr_moe_plan_destroy(p->moe);
  delete p;
  return UOCR_OK;
}

int uocr_decoder_bytes(const uocr_decoder* p, int64_t* weight_bytes, int64_t* other_bytes) {
  if (p == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_bytes: null decoder");
  int64_t mw = 0, ma = 0;
  DEC_RC(uocr_moe_plan_bytes(p->moe, &mw, &ma));
  if (weight_bytes != nullptr) *weight_bytes = static_cast<int64_t>(p->weight_bytes) + mw;
  if (other_bytes != nullptr) *other_bytes = static_cast<int64_t>(p->arena_bytes) + ma;
  return UOCR_OK;
}

int uocr_decoder_set_layer(uocr_decoder* p, int64_t layer, const uocr_decoder_layer_src* src, void* stream_v) {
  if (p == nullptr || src == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_set_layer: null argument");
  if (layer < 0 || layer >= p->d.layers) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_set_layer: layer out of range");
  if (src->memory != UOCR_MEMORY_HOST && src->memory != UOCR_MEMORY_DEVICE)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_set_layer: memory must be host or device");
  Guard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  DecLayer& L = p->layers[static_cast<size_t>(layer)];
  const int64_t H = p->d.hidden, A = p->d.heads * kDecHeadDim, KV = p->d.kv_heads * kDecHeadDim;
  const size_t eb = p->int8 ? 1 : 2;
  DEC_RC(copy_gain(src->memory, src->input_norm, L.input_norm, H, stream, "input_norm"));
  char* wqkv = static_cast<char*>(L.wqkv);
  DEC_RC(convert_matrix(src->memory, src->dtype, src->wq, A, H, p->int8, wqkv, L.wqkv_s, stream, "wq"));
  DEC_RC(convert_matrix(src->memory, src->dtype, src->wk, KV, H, p->int8, wqkv + static_cast<size_t>(A * H) * eb,
                        L.wqkv_s != nullptr ? L.wqkv_s + A : nullptr, stream, "wk"));
  DEC_RC(convert_matrix(src->memory, src->dtype, src->wv, KV, H, p->int8,
                        wqkv + static_cast<size_t>((A + KV) * H) * eb,
                        L.wqkv_s != nullptr ? L.wqkv_s + A + KV : nullptr, stream, "wv"));
  DEC_RC(convert_matrix(src->memory, src->dtype, src->wo, H, A, p->int8, L.wo, L.wo_s, stream, "wo"));
  if (src->post_norm == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder: missing post_norm");
  uocr_moe_layer_src m{};
  m.memory = src->memory;
  m.dtype = src->dtype;
  m.router = src->router;
  m.gate = src->gate;
  m.up = src->up;
  m.down = src->down;
  m.shared_gate = src->shared_gate;
  m.shared_up = src->shared_up;
  m.shared_down = src->shared_down;
  m.norm = src->post_norm;
  DEC_RC(uocr_moe_set_layer(p->moe, layer, &m, stream_v));
  L.loaded = true;
  return UOCR_OK;
}

int uocr_decoder_set_head(uocr_decoder* p, int32_t memory, int32_t dtype, const void* embed, const float* final_norm,
                          const void* lm_head, void* stream_v) {
  if (p == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_set_head: null decoder");
  if (memory != UOCR_MEMORY_HOST && memory != UOCR_MEMORY_DEVICE)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_set_head: memory must be host or device");
  Guard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  const int64_t H = p->d.hidden, V = p->d.vocab;
  DEC_RC(convert_matrix(memory, dtype, embed, V, H, false, p->embed, nullptr, stream, "embed"));
  DEC_RC(copy_gain(memory, final_norm, p->final_norm, H, stream, "final_norm"));
  DEC_RC(convert_matrix(memory, dtype, lm_head, V, H, p->int8, p->lm_head, p->lm_head_s, stream, "lm_head"));
  p->head_loaded = true;
  return UOCR_OK;
}

int uocr_decoder_prefill(uocr_decoder* p, const float* embeds, int64_t rows, float* logits, int32_t* token,
                         void* stream_v) {
  if (p == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: null decoder");
  if (rows <= 0 || rows > p->d.max_prefill)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: rows outside [1, max_prefill]");
  if (embeds == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: null embeddings");
  if ((reinterpret_cast<uintptr_t>(embeds) & 15) != 0)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: embeddings must be 16-byte aligned");
  for (const auto& L : p->layers)
    if (!L.loaded) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: a layer's weights are not set");
  if (!p->head_loaded) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_prefill: head weights not set");
  Guard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  const DecShape& s = p->shape;
  const int64_t H = p->d.hidden, A = p->d.heads * kDecHeadDim;
  DEC_TRY(cudaMemcpyAsync(p->x, embeds, static_cast<size_t>(rows * H) * 4, cudaMemcpyDeviceToDevice, stream),
          "decoder_prefill: input copy");
  for (int64_t l = 0; l < p->d.layers; ++l) {
    const DecLayer& L = p->layers[static_cast<size_t>(l)];
    DEC_TRY(launch_norm_rows_bf16(p->x, rows, static_cast<int>(H), L.input_norm, p->d.rms_norm_eps, p->xn, stream),
            "decoder_prefill: norm");
    cudaError_t st = cudaSuccess;
    const __nv_bfloat16* wqkv = gemm_operand(p, L.wqkv, L.wqkv_s, p->qkv_rows, H, stream, &st);
    DEC_TRY(st, "decoder_prefill: int8 expansion");
    DEC_TRY(gemm(p, p->xn, rows, H, wqkv, p->qkv_rows, p->qkv, false, stream), "decoder_prefill: q/k/v GEMM");
    DEC_TRY(launch_rope_rows(s, p->qkv, rows, p->inv_freq, p->qb, kc_of(p, l), vc_of(p, l), stream),
            "decoder_prefill: rope");
    DEC_TRY(launch_prefill_attn(s, p->qb, rows, kc_of(p, l), vc_of(p, l), p->attn, stream),
            "decoder_prefill: attention");
    const __nv_bfloat16* wo = gemm_operand(p, L.wo, L.wo_s, H, A, stream, &st);
    DEC_TRY(st, "decoder_prefill: int8 expansion");
    DEC_TRY(gemm(p, p->attn, rows, A, wo, H, p->x, true, stream), "decoder_prefill: output GEMM");
    DEC_RC(moe_layer_inplace(p->moe, l, p->x, rows, stream));
  }
  DEC_TRY(launch_dec_lmhead(s, p->int8, p->x + (rows - 1) * H, p->final_norm, DecMatrix{p->lm_head, p->lm_head_s},
                            p->logits, p->state, p->lm_part, p->counters, p->tokens, 0,
                            static_cast<int>(rows), p->sm_count, stream, false),
          "decoder_prefill: lm_head");
  if (logits != nullptr)
    DEC_TRY(cudaMemcpyAsync(logits, p->logits, static_cast<size_t>(p->d.vocab) * 4, cudaMemcpyDeviceToDevice, stream),
            "decoder_prefill: logits copy");
  if (token != nullptr)
    DEC_TRY(cudaMemcpyAsync(token, p->tokens, 4, cudaMemcpyDeviceToDevice, stream), "decoder_prefill: token copy");
  p->length = rows;
  p->generated = 1;
  p->started = true;
  return UOCR_OK;
}

int uocr_decoder_decode(uocr_decoder* p, int64_t steps, int32_t* tokens, float* logits, void* stream_v) {
  if (p == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_decode: null decoder");
  if (!p->started) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_decode: no prefill started a sequence");
  if (steps < 0 || p->length + steps > p->d.max_positions)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_decode: the sequence would pass max_positions");
  if (steps == 0) return UOCR_OK;
  Guard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  DEC_TRY(cudaStreamIsCapturing(stream, &cap), "decoder_decode: capture status");
  const bool graphs = cap == cudaStreamCaptureStatusNone && stream != nullptr && stream != cudaStreamLegacy;
  if (graphs && (p->graph == nullptr || p->graph_stream != stream)) {
    if (p->graph != nullptr) {
      cudaGraphExecDestroy(p->graph);
      p->graph = nullptr;
    }
    DEC_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "decoder_decode: begin capture");
    const int rc = decode_step(p, stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t end = cudaStreamEndCapture(stream, &graph);
    if (rc != UOCR_OK) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      return rc;
    }
    if (end != cudaSuccess) return dcuda(end, "decoder_decode: end capture");
    const cudaError_t inst = cudaGraphInstantiate(&p->graph, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) return dcuda(inst, "decoder_decode: instantiate");
    p->graph_stream = stream;
  }
  for (int64_t i = 0; i < steps; ++i) {
    if (graphs)
      DEC_TRY(cudaGraphLaunch(p->graph, stream), "decoder_decode: graph launch");
    else
      DEC_RC(decode_step(p, stream));
    if (logits != nullptr)
      DEC_TRY(cudaMemcpyAsync(logits + i * p->d.vocab, p->logits, static_cast<size_t>(p->d.vocab) * 4,
                              cudaMemcpyDeviceToDevice, stream),
              "decoder_decode: logits copy");
  }
  if (tokens != nullptr)
    DEC_TRY(cudaMemcpyAsync(tokens, p->tokens + p->generated, static_cast<size_t>(steps) * 4,
                            cudaMemcpyDeviceToDevice, stream),
            "decoder_decode: token copy");
  p->length += steps;
  p->generated += steps;
  return UOCR_OK;
}

int uocr_decoder_profile_decode(uocr_decoder* p, int64_t steps, float* ms, void* stream_v) {
  if (p == nullptr || ms == nullptr || steps <= 0)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_profile_decode: bad argument");
  if (!p->started) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_profile_decode: no prefill started a sequence");
  if (p->length + steps > p->d.max_positions)
    return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_profile_decode: the sequence would pass max_positions");
  Guard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  const size_t nev = static_cast<size_t>(p->d.layers * (kProfilePhases + 1) + 1);
  std::vector<cudaEvent_t> ev(nev, nullptr);
  int rc = UOCR_OK;
  for (auto& e : ev)
    if (cudaEventCreate(&e) != cudaSuccess) rc = dfail(UOCR_ERR_CUDA, "decoder_profile_decode: event");
  double acc[kProfilePhases + 1] = {};
  for (int64_t i = 0; i < steps && rc == UOCR_OK; ++i) {
    rc = decode_step(p, stream, ev.data());
    if (rc != UOCR_OK) break;
    if (cudaEventSynchronize(ev[nev - 1]) != cudaSuccess) {
      rc = dfail(UOCR_ERR_CUDA, "decoder_profile_decode: synchronise");
      break;
    }
    for (int64_t l = 0; l < p->d.layers; ++l)
      for (int k = 0; k < kProfilePhases; ++k) {
        float t = 0.0f;
        cudaEventElapsedTime(&t, ev[l * (kProfilePhases + 1) + k], ev[l * (kProfilePhases + 1) + k + 1]);
        acc[k] += t;
      }
    float t = 0.0f;
    cudaEventElapsedTime(&t, ev[(p->d.layers - 1) * (kProfilePhases + 1) + kProfilePhases], ev[nev - 1]);
    acc[kProfilePhases] += t;
  }
  for (auto& e : ev)
    if (e != nullptr) cudaEventDestroy(e);
  if (rc != UOCR_OK) return rc;
  for (int k = 0; k <= kProfilePhases; ++k) ms[k] = static_cast<float>(acc[k] / static_cast<double>(steps));
  p->length += steps;
  p->generated += steps;
  return UOCR_OK;
}

int uocr_decoder_check(uocr_decoder* p, void* stream_v) {
  if (p == nullptr) return dfail(UOCR_ERR_INVALID_ARGUMENT, "decoder_check: null decoder");
  Guard guard(p->d.device);
  DEC_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream_v)), "decoder_check: stream");
  ErrorWord e{};
  DEC_TRY(cudaMemcpy(&e, p->err, sizeof(e), cudaMemcpyDeviceToHost), "decoder_check: error word");
  if (e.code != kDevOk) {
    DEC_TRY(cudaMemset(p->err, 0, sizeof(e)), "decoder_check: clear");
    return dfail(e.code == kDevWaitTimeout ? UOCR_ERR_TIMEOUT : UOCR_ERR_DEVICE,
                 "decoder: device error " + std::to_string(e.code) + " at site " + std::to_string(e.where));
  }
  return uocr_moe_check(p->moe, stream_v);
}

}  // extern "C"
