// TEST INFRASTRUCTURE ONLY (never linked into the product library).
//
// A C-ABI shim over the reference's own fp32 mixture-of-experts, compiled
// together with the reference sources where they lie (see oracle/Makefile):
//   src/model/feed_forward.cpp   MixtureOfExperts::forward (:36-78), GatedMlp (:18-24)
//   src/backend/reference/ops.cpp linear/dot (:25-38, :91-109), softmax_rows (:169-187), silu (:163-167),
//                                 rms_norm (:129-141, the decoder's pre-feed-forward norm)
//   src/model/weight_source.cpp   TableWeights (:77-83)
//   src/model/page_rope.cpp       PageRope (:8-56, the decoder's rotate-half rotation)
//   src/tensor/dtype.cpp
// The shim only packs caller arrays into a TableWeights under the tensor names
// the reference reads (src/weights/architecture.cpp:113-117) and calls
// MixtureOfExperts::forward unchanged. The reference has no renormalisation
// switch and no router bias (feed_forward.cpp:40, architecture.cpp:113), so
// this entry point is the renorm-off, bias-free semantics only.

#include <cstdint>
#include <cstring>
#include <exception>
#include <format>
#include <memory>
#include <string>
#include <vector>

#include "backend/reference/ops.h"
#include "backend/reference/parallel.h"
#include "model/feed_forward.h"
#include "model/page_rope.h"
#include "model/weight_source.h"
#include "weights/architecture.h"
#include "weights/sharded_weights.h"

namespace uocr {
// weight_source.cpp's CheckpointWeights::get references these two symbols; the
// safetensors reader that defines them needs nlohmann_json, which is absent.
// The shim never reads a checkpoint, so both only throw.
const TensorInfo& ShardedWeights::at(const std::string& name) const {
  throw std::out_of_range("ref_shim: no checkpoint reader (" + name + ")");
}
std::int64_t TensorInfo::element_count() const { throw std::logic_error("ref_shim: no checkpoint reader"); }
}  // namespace uocr

namespace {

thread_local std::string g_error;

uocr::Tensor copy_tensor(std::vector<std::int64_t> shape, const float* src) {
  uocr::Tensor t(std::move(shape));
  std::memcpy(t.data(), src, static_cast<std::size_t>(t.numel()) * sizeof(float));
  return t;
}

struct RefMoe {
  std::unique_ptr<uocr::MixtureOfExperts> moe;
  std::int64_t hidden = 0;
};

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

void ref_set_threads(int threads) { uocr::reference::set_thread_count(static_cast<unsigned>(threads)); }

unsigned ref_get_threads() { return uocr::reference::thread_count(); }

// Builds one MoE layer from stacked arrays: router [E,H]; gate/up [E*F,H];
// down [E*H,F]; shared gate/up [S,H], shared down [H,S]. Returns null on error.
void* ref_moe_create(std::int64_t hidden, std::int64_t experts, std::int64_t top_k, std::int64_t ffn,
                     std::int64_t shared_ffn, const float* router, const float* gate, const float* up,
                     const float* down, const float* shared_gate, const float* shared_up, const float* shared_down) {
  try {
    uocr::TableWeights table;
    const std::string p = "model.layers.1.mlp";
    table.put(p + ".gate.weight", copy_tensor({experts, hidden}, router));
    for (std::int64_t e = 0; e < experts; ++e) {
      const std::string ep = std::format("{}.experts.{}", p, e);
      table.put(ep + ".gate_proj.weight", copy_tensor({ffn, hidden}, gate + e * ffn * hidden));
      table.put(ep + ".up_proj.weight", copy_tensor({ffn, hidden}, up + e * ffn * hidden));
      table.put(ep + ".down_proj.weight", copy_tensor({hidden, ffn}, down + e * hidden * ffn));
    }
    table.put(p + ".shared_experts.gate_proj.weight", copy_tensor({shared_ffn, hidden}, shared_gate));
    table.put(p + ".shared_experts.up_proj.weight", copy_tensor({shared_ffn, hidden}, shared_up));
    table.put(p + ".shared_experts.down_proj.weight", copy_tensor({hidden, shared_ffn}, shared_down));
    uocr::DecoderDims dims;
    dims.hidden = hidden;
    dims.routed_experts = experts;
    dims.experts_per_token = top_k;
    dims.expert_ffn = ffn;
    auto* h = new RefMoe;
    h->moe = std::make_unique<uocr::MixtureOfExperts>(table, p, dims);
    h->hidden = hidden;
    return h;
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

// y [tokens, H] = MixtureOfExperts::forward(x [tokens, H]). 0 on success.
int ref_moe_run(void* handle, const float* x, std::int64_t tokens, float* y) {
  try {
    auto* h = static_cast<RefMoe*>(handle);
    const uocr::Tensor out = h->moe->forward(copy_tensor({tokens, h->hidden}, x));
    std::memcpy(y, out.data(), static_cast<std::size_t>(out.numel()) * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

void ref_moe_destroy(void* handle) { delete static_cast<RefMoe*>(handle); }

// x [rows, cols] <- rms_norm(x, weight [cols], eps), in place. 0 on success.
int ref_rms_norm(float* x, std::int64_t rows, std::int64_t cols, const float* weight, float eps) {
  try {
    uocr::Tensor t = copy_tensor({rows, cols}, x);
    uocr::reference::rms_norm(t, copy_tensor({cols}, weight), eps);
    std::memcpy(x, t.data(), static_cast<std::size_t>(t.numel()) * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// out [lq, dv] = attention_head(q [lq, d], k [lk, d], v [lk, dv], bias [lq, lk]
// or null, scale): ops.cpp:219-251 unchanged. 0 on success.
int ref_attention_head(const float* q, std::int64_t lq, const float* k, std::int64_t lk, std::int64_t d,
                       const float* v, std::int64_t dv, const float* bias, float scale, float* out) {
  try {
    const uocr::Tensor tq = copy_tensor({lq, d}, q), tk = copy_tensor({lk, d}, k), tv = copy_tensor({lk, dv}, v);
    uocr::Tensor tb;
    if (bias != nullptr) tb = copy_tensor({lq, lk}, bias);
    const uocr::Tensor o = uocr::reference::attention_head(tq, tk, tv, bias != nullptr ? &tb : nullptr, scale);
    std::memcpy(out, o.data(), static_cast<std::size_t>(o.numel()) * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// x [rows, width] rotated in place by PageRope(dim, tok_theta, page_theta,
// page_pairs, page_mod) at coordinates (tok[r], page[r]); also returns the
// rope's frequency tables (inv_tok then inv_page) in inv. 0 on success.
int ref_page_rope(float* x, std::int64_t rows, std::int64_t width, std::int64_t dim, double tok_theta,
                  double page_theta, std::int64_t page_pairs, std::int64_t page_mod, const std::int64_t* tok,
                  const std::int64_t* page, float* inv) {
  try {
    const uocr::PageRope rope(dim, tok_theta, page_theta, page_pairs, page_mod);
    uocr::Tensor t = copy_tensor({rows, width}, x);
    std::vector<uocr::RopeCoord> coords(static_cast<std::size_t>(rows));
    for (std::int64_t r = 0; r < rows; ++r) coords[static_cast<std::size_t>(r)] = {tok[r], page[r]};
    rope.apply(t, coords);
    std::memcpy(x, t.data(), static_cast<std::size_t>(t.numel()) * sizeof(float));
    float* o = inv;
    for (float f : rope.inv_tok()) *o++ = f;
    for (float f : rope.inv_page()) *o++ = f;
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

}  // extern "C"
