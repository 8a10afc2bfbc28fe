// TEST INFRASTRUCTURE ONLY: the op-level drop-in of the integration notes,
// built into the reference's own CUDA decoder test (oracle/Makefile,
// target cuda_decoder_test). These two definitions replace the reference's
// uocr::cuda::expert_topk (src/backend/cuda/ops.cu:650-660) and
// uocr::cuda::expert_ffn_one (src/backend/cuda/gemv_ops.cu:221-227), whose
// own definitions the Makefile turns into weak symbols, so CudaDecoder::moe
// (src/model/cuda/cuda_decoder.cpp:137-192) runs this library's kernels on
// its decode steps. The int8 decoder keeps the reference's expert_ffn_one_q8:
// its weights carry one scale per 32 inputs, the library's int8 path one per
// row. At exit the binding reports how often it was called, so the test can
// tell that the library's kernels ran.
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "../include/uocr_moe.h"
#include "backend/cuda/context.h"
#include "backend/cuda/context_impl.h"
#include "backend/cuda/ops.h"
#include "weights/sharded_weights.h"

namespace uocr {
// architecture.cpp's checkpoint check references these two; their source
// (sharded_weights.cpp) needs nlohmann_json, which is absent. The test reads
// no checkpoint, so both only throw.
const TensorInfo* ShardedWeights::find(const std::string& name) const {
  throw std::logic_error("ref_cuda_bind: no checkpoint reader (" + name + ")");
}
std::vector<std::string> ShardedWeights::names() const {
  throw std::logic_error("ref_cuda_bind: no checkpoint reader");
}
}  // namespace uocr

namespace {

struct Calls {
  long topk = 0, ffn = 0;
  ~Calls() { std::printf("uocr binding: expert_topk %ld, expert_ffn_one %ld\n", topk, ffn); }
} g_calls;

void require_ok(int rc) {
  if (rc == UOCR_OK) return;
  const std::string what = std::string("uocr: ") + uocr_last_error();
  if (rc == UOCR_ERR_INVALID_ARGUMENT || rc == UOCR_ERR_UNSUPPORTED) throw std::invalid_argument(what);
  throw std::runtime_error(what);
}

}  // namespace

namespace uocr::cuda {

void expert_topk(const Context& ctx, const float* logits, std::int64_t rows, std::int64_t experts, std::int64_t k,
                 std::int64_t* ids, float* weights) {
  ++g_calls.topk;
  require_ok(uocr_expert_topk(logits, rows, experts, k, 0, ids, weights, ctx.impl().stream));
}

void expert_ffn_one(const Context& ctx, const float* x, std::int64_t hidden, std::int64_t ffn,
                    const std::uint16_t* gate, const std::uint16_t* up, const std::uint16_t* down,
                    const std::int64_t* ids, const float* weights, std::int64_t k, float* out) {
  ++g_calls.ffn;
  require_ok(uocr_expert_ffn_one(x, hidden, ffn, gate, up, down, ids, weights, k, out, ctx.impl().stream));
}

}  // namespace uocr::cuda
