// uocr_expert_ffn_one_noalloc: expert_ffn_one for callers that cannot
// allocate device memory on the call path.
//
// Who needs it: a serving loop whose device memory is reserved up front by
// another allocator (a caching allocator that already holds the pool, so a
// cudaMalloc there fails or fragments it), a latency-critical decode step
// that must not take cudaMalloc's device-wide synchronisation or a memory
// pool's bookkeeping, and host runtimes whose policy forbids device
// allocations after start-up. uocr_expert_ffn_one takes its scratch from
// cudaMallocAsync, as the reference's expert_ffn does; this variant takes it
// from one static device array instead and allocates nothing.
//
// The scratch (routing table and the [k, ffn] bf16 activation rows) lives in
// g_noalloc_scratch below: about 146 KiB that every GPU which loads this
// library holds until the process exits. Every call shares it and it keeps
// the last call's contents; each call fully rewrites the routing table and
// the activation rows it reads, so nothing in it has to start at zero. Calls
// that overlap on the GPU (different streams, or different host threads, on
// the same device) race on the array and must be serialised by the caller.
// A bad expert id goes to the device's op-level error word (also static
// device memory), which uocr_ops_check reads and clears.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/uocr_moe.h"
#include "moe_kernels.h"

using namespace uocr_b200;

namespace {

constexpr int64_t kNoAllocMaxK = kMaxTopK;  // 8 routed experts per call
constexpr int64_t kNoAllocMaxFfn = 8192;    // expert width
constexpr size_t kRouteOffset = 0;
constexpr size_t kActOffset = (sizeof(DecodeRoute) + 255) / 256 * 256;
constexpr size_t kScratchBytes = kActOffset + static_cast<size_t>(kNoAllocMaxK * kNoAllocMaxFfn) * 2;

// The only storage this entry point uses. In host code this name is a
// host-side stand-in, not a device address: kernels get the address from
// cudaGetSymbolAddress (scratch_address below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

int noalloc_fail(int code, const std::string& what) { return set_last_error(code, what); }

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (the first call on a device does this; make that first call
// before any stream capture), and the current device's ordinal.
int scratch_address(unsigned char** out, int* device) {
  static std::mutex mu;
  static unsigned char* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return noalloc_fail(UOCR_ERR_CUDA, std::string("no current device: ") + cudaGetErrorString(st));
  if (dev >= kMaxDevices) return noalloc_fail(UOCR_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess)
      return noalloc_fail(UOCR_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(st));
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
  *device = dev;
  return UOCR_OK;
}

}  // namespace

extern "C" int uocr_expert_ffn_one_noalloc(const float* x, int64_t hidden, int64_t ffn, const uint16_t* gate,
                                           const uint16_t* up, const uint16_t* down, const int64_t* ids,
                                           const float* weights, int64_t k, float* out, void* stream_v) {
  if (hidden <= 0 || hidden % 16 != 0 || ffn <= 0 || ffn % 16 != 0)
    return noalloc_fail(UOCR_ERR_INVALID_ARGUMENT,
                        "expert_ffn_one_noalloc: hidden and ffn must be positive multiples of 16");
  if (k <= 0 || k > kNoAllocMaxK)
    return noalloc_fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one_noalloc: k must be in [1, 8]");
  if (ffn > kNoAllocMaxFfn)
    return noalloc_fail(UOCR_ERR_INVALID_ARGUMENT,
                        "expert_ffn_one_noalloc: ffn above 8192, the static scratch holds 8 x 8192 bf16 activations");
  if (x == nullptr || gate == nullptr || up == nullptr || down == nullptr || ids == nullptr || weights == nullptr ||
      out == nullptr)
    return noalloc_fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one_noalloc: null pointer");
  unsigned char* base = nullptr;
  int dev = 0;
  const int rc = scratch_address(&base, &dev);
  if (rc != UOCR_OK) return rc;
  ErrorWord* err = nullptr;
  cudaError_t st = ops_error_word(&err);
  if (st != cudaSuccess)
    return noalloc_fail(UOCR_ERR_CUDA, std::string("expert_ffn_one_noalloc: error word: ") + cudaGetErrorString(st));
  int sms = 0;
  st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (st != cudaSuccess)
    return noalloc_fail(UOCR_ERR_CUDA, std::string("expert_ffn_one_noalloc: SM count: ") + cudaGetErrorString(st));
  auto stream = static_cast<cudaStream_t>(stream_v);
  auto* route = reinterpret_cast<DecodeRoute*>(base + kRouteOffset);
  auto* act = reinterpret_cast<__nv_bfloat16*>(base + kActOffset);
  auto b = [](const uint16_t* v) { return reinterpret_cast<const __nv_bfloat16*>(v); };
  st = launch_route_from_ids(ids, weights, static_cast<int>(k), kMaxExperts, route, err, stream);
  const DecodeRouting routing{nullptr, route, kMaxExperts, static_cast<int>(k), 0, nullptr, nullptr};
  if (st == cudaSuccess)
    st = launch_decode_experts_bf16(x, 1, static_cast<int>(hidden), static_cast<int>(ffn), 0, b(gate), b(up),
                                    b(down), nullptr, nullptr, nullptr, routing, act, nullptr, nullptr, out, err,
                                    sms > 0 ? sms : 1, stream);
  if (st != cudaSuccess)
    return noalloc_fail(UOCR_ERR_CUDA, std::string("expert_ffn_one_noalloc: ") + cudaGetErrorString(st));
  return UOCR_OK;
}
