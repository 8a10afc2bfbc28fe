// uocr_moe.hpp — header-only C++ layer over the C ABI in uocr_moe.h.
//
// Two things for a C++ caller such as the reference's CudaDecoder:
//   * free functions with the call shapes of the reference's CUDA backend ops
//     (src/backend/cuda/ops.h:14-17, 80-82, 87-90; gemv_ops.h:33-35), the
//     Context replaced by the stream it carries, so a call site changes only
//     its namespace and first argument;
//   * RAII owners of a plan and of a checkpoint.
// Status codes come back as the exceptions the reference's callers expect:
// argument and shape misuse as std::invalid_argument (ops.cu:653-655,
// gemv_ops.cu:193-195), CUDA and device failures as std::runtime_error
// (context.cu:24-34); checkpoint problems as std::runtime_error and a missing
// tensor as std::out_of_range (src/weights/safetensors.h:28-34,
// sharded_weights.h:16-27).
#ifndef UOCR_MOE_HPP
#define UOCR_MOE_HPP

#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>

#include "uocr_moe.h"

namespace uocr_b200 {

// Throws for a failed status: std::invalid_argument for argument and shape
// misuse, std::runtime_error otherwise. The message is uocr_last_error().
inline void check(int status) {
  if (status == UOCR_OK) return;
  const std::string what = std::string("uocr: ") + uocr_last_error();
  if (status == UOCR_ERR_INVALID_ARGUMENT || status == UOCR_ERR_UNSUPPORTED) throw std::invalid_argument(what);
  throw std::runtime_error(what);
}

// GRPC_UOCR_WEIGHT_FORMAT as the engine reads it for the cuda backend
// (src/service/config.cpp:28-39, 53-55; default bf16, config.h:20): unset or
// empty is bf16, "bf16" and "int8" select, anything else throws
// std::invalid_argument naming the variable and its choices.
inline uocr_weight_format weight_format_from_env() {
  const char* raw = std::getenv("GRPC_UOCR_WEIGHT_FORMAT");
  if (raw == nullptr || *raw == '\0') return UOCR_WEIGHT_BF16;
  const std::string value(raw);
  if (value == "bf16") return UOCR_WEIGHT_BF16;
  if (value == "int8") return UOCR_WEIGHT_INT8;
  throw std::invalid_argument("GRPC_UOCR_WEIGHT_FORMAT must be one of bf16, int8");
}

// ---- the reference's op shapes (stream first instead of the Context) --------

// Softmax + top-k (lower id on a tie), raw softmax weights as the reference
// returns them; renormalize = true divides them by their sum.
inline void expert_topk(void* stream, const float* logits, std::int64_t rows, std::int64_t experts, std::int64_t k,
                        std::int64_t* ids, float* weights, bool renormalize = false) {
  check(uocr_expert_topk(logits, rows, experts, k, renormalize ? 1 : 0, ids, weights, stream));
}

inline void expert_ffn_one(void* stream, const float* x, std::int64_t hidden, std::int64_t ffn,
                           const std::uint16_t* gate, const std::uint16_t* up, const std::uint16_t* down,
                           const std::int64_t* ids, const float* weights, std::int64_t k, float* out) {
  check(uocr_expert_ffn_one(x, hidden, ffn, gate, up, down, ids, weights, k, out, stream));
}

// Throws std::runtime_error when an op above recorded a bad expert id on the
// current device since the last call (synchronises the stream).
inline void ops_check(void* stream) { check(uocr_ops_check(stream)); }

// int8 stacks with one fp32 scale per weight row (the reference's Q8Weights
// holds one per 32 inputs; uocr_quantize_q8 with group = cols makes these).
struct Q8Weights {
  const std::int8_t* q;  // [rows, cols]
  const float* scales;   // [rows]
};

inline void expert_ffn_one_q8(void* stream, const float* x, std::int64_t hidden, std::int64_t ffn, Q8Weights gate,
                              Q8Weights up, Q8Weights down, const std::int64_t* ids, const float* weights,
                              std::int64_t k, float* out) {
  check(uocr_expert_ffn_one_q8(x, hidden, ffn, gate.q, gate.scales, up.q, up.scales, down.q, down.scales, ids,
                               weights, k, out, stream));
}

inline void linear(void* stream, const float* x, std::int64_t m, std::int64_t k, const std::uint16_t* w_bf16,
                   std::int64_t n, const float* bias, float* y) {
  check(uocr_linear(x, m, k, w_bf16, n, bias, y, stream));
}

// ---- owners ------------------------------------------------------------------

class Checkpoint;

// One MoE stack on one device (uocr_moe_plan); see uocr_moe.h for the calls.
class MoePlan {
 public:
  explicit MoePlan(const uocr_moe_desc& desc) { check(uocr_moe_plan_create(&desc, &plan_)); }
  ~MoePlan() {
    if (plan_ != nullptr) uocr_moe_plan_destroy(plan_);
  }
  MoePlan(const MoePlan&) = delete;
  MoePlan& operator=(const MoePlan&) = delete;
  MoePlan(MoePlan&& o) noexcept : plan_(std::exchange(o.plan_, nullptr)) {}
  MoePlan& operator=(MoePlan&& o) noexcept {
    if (this != &o) {
      if (plan_ != nullptr) uocr_moe_plan_destroy(plan_);
      plan_ = std::exchange(o.plan_, nullptr);
    }
    return *this;
  }

  uocr_moe_plan* get() const { return plan_; }

  void set_layer(std::int64_t layer, const uocr_moe_layer_src& src, void* stream) {
    check(uocr_moe_set_layer(plan_, layer, &src, stream));
  }
  void set_layer(std::int64_t layer, const uocr_moe_layer_parts& parts, void* stream) {
    check(uocr_moe_set_layer_parts(plan_, layer, &parts, stream));
  }
  inline void load_layer(const Checkpoint& ckpt, std::int64_t layer, std::int64_t plan_layer, void* stream);
  void forward(std::int64_t layer, const float* x, std::int64_t rows, float* y, void* stream,
               std::int32_t* ids = nullptr, float* weights = nullptr) {
    check(uocr_moe_forward(plan_, layer, x, rows, y, ids, weights, stream));
  }
  // The layer's router gate: logits [rows, E] in the CPU reference's dot order.
  void router_logits(std::int64_t layer, const float* x, std::int64_t rows, float* logits, void* stream) {
    check(uocr_moe_router_logits(plan_, layer, x, rows, logits, stream));
  }
  void forward_stack(float* h, std::int64_t rows, void* stream) {
    check(uocr_moe_forward_stack(plan_, h, rows, stream));
  }
  // Synchronises the stream and throws if a kernel recorded an error.
  void check_device(void* stream) { check(uocr_moe_check(plan_, stream)); }

 private:
  uocr_moe_plan* plan_ = nullptr;
};

// A checkpoint mapped read-only (uocr_checkpoint_open: a shard index or one
// .safetensors file).
class Checkpoint {
 public:
  explicit Checkpoint(const std::string& path) {
    const int rc = uocr_checkpoint_open(path.c_str(), &ckpt_);
    if (rc != UOCR_OK) throw std::runtime_error(std::string("uocr: ") + uocr_last_error());
  }
  ~Checkpoint() {
    if (ckpt_ != nullptr) uocr_checkpoint_close(ckpt_);
  }
  Checkpoint(const Checkpoint&) = delete;
  Checkpoint& operator=(const Checkpoint&) = delete;
  Checkpoint(Checkpoint&& o) noexcept : ckpt_(std::exchange(o.ckpt_, nullptr)) {}
  Checkpoint& operator=(Checkpoint&& o) noexcept {
    if (this != &o) {
      if (ckpt_ != nullptr) uocr_checkpoint_close(ckpt_);
      ckpt_ = std::exchange(o.ckpt_, nullptr);
    }
    return *this;
  }

  const uocr_checkpoint* get() const { return ckpt_; }

  std::int64_t size() const {
    std::int64_t n = 0;
    check(uocr_checkpoint_count(ckpt_, &n));
    return n;
  }
  // Nothing copied: the view points into the mapping while this object lives.
  uocr_tensor_view at(const std::string& name) const {
    uocr_tensor_view v{};
    if (uocr_checkpoint_tensor(ckpt_, name.c_str(), &v) != UOCR_OK)
      throw std::out_of_range(std::string("uocr: ") + uocr_last_error());
    return v;
  }

 private:
  uocr_checkpoint* ckpt_ = nullptr;
};

inline void MoePlan::load_layer(const Checkpoint& ckpt, std::int64_t layer, std::int64_t plan_layer, void* stream) {
  check(uocr_moe_load_layer(plan_, ckpt.get(), layer, plan_layer, stream));
}

}  // namespace uocr_b200

#endif  // UOCR_MOE_HPP
