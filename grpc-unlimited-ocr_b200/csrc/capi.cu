// The C ABI (include/uocr_moe.h): plan lifetime, weight upload, the MoE
// forward dispatch, and the op-level mirrors of the reference's uocr::cuda
// MoE ops. Host code only; kernels live in router.cu, decode.cu, weights.cu.
//
// The dispatch replaces CudaDecoder::moe (src/model/cuda/cuda_decoder.cpp:
// 137-192): it routes on the device for every row count (the reference
// downloads the logits and routes on the host when rows > 1, :159-175) and
// keeps all scratch in one arena allocated with the plan (the reference
// cudaMallocAsync's per op, gemv_ops.cu:176, ops.cu:275).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "../../include/uocr_moe.h"
#include "checkpoint.h"
#include "ep.h"
#include "moe_kernels.h"
#include "plan_internal.h"
#include "prefill.h"

using namespace uocr_b200;

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& what) {
  g_error = what;
  return code;
}

int cuda_fail(cudaError_t st, const char* what) {
  return fail(st == cudaErrorMemoryAllocation ? UOCR_ERR_OUT_OF_MEMORY : UOCR_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(st));
}

#define UOCR_TRY(expr, what)                     \
  do {                                           \
    cudaError_t st_ = (expr);                    \
    if (st_ != cudaSuccess) return cuda_fail(st_, what); \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device-side view of one layer's weights.
struct LayerDev {
  void* block = nullptr;
  size_t bytes = 0;
  bool loaded = false;
  float* router = nullptr;
  float* bias = nullptr;
  float* norm = nullptr;  // [H] RMSNorm gain (pre-norm plans)
  void* gate = nullptr;
  void* up = nullptr;
  void* down = nullptr;
  void* sgate = nullptr;
  void* sup = nullptr;
  void* sdown = nullptr;
  float* gate_s = nullptr;
  float* up_s = nullptr;
  float* down_s = nullptr;
  float* sgate_s = nullptr;
  float* sup_s = nullptr;
  float* sdown_s = nullptr;
};

// Bump allocator over one device block.
struct Carver {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = align_up(off, 256);
    T* p = base == nullptr ? nullptr : reinterpret_cast<T*>(base + off);
    off += count * sizeof(T);
    return p;
  }
};

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (prev_ != device) cudaSetDevice(device);
  }
  ~DeviceGuard() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

}  // namespace

int uocr_b200::set_last_error(int code, const std::string& what) { return fail(code, what); }

struct uocr_moe_plan {
  uocr_moe_desc d{};
  int sm_count = 0;
  int decode_rows = 0;  // largest row count the decode kernels take
  std::vector<LayerDev> layers;
  char* arena = nullptr;
  size_t arena_bytes = 0;
  size_t weight_bytes = 0;
  float* logits = nullptr;
  int* ids = nullptr;
  float* weights = nullptr;
  DecodeRoute* route = nullptr;
  __nv_bfloat16* act = nullptr;
  __nv_bfloat16* act_s = nullptr;
  unsigned* counter = nullptr;  // the decode router's last-block ticket
  ErrorWord* err = nullptr;
  bool pre_norm = false;
  float* xnorm = nullptr;  // [max_rows, H] normalised rows for the prefill path (pre-norm plans)
  // int8 plans on the prefill path: the layer's experts and shared expert
  // expanded to bf16 (gate, up, down, shared gate, up, down) before the GEMMs.
  __nv_bfloat16* wexp = nullptr;
  // Prefill (rows above decode_rows): tcgen05 grouped GEMM path (bf16; int8
  // layers are expanded to bf16 first, as the reference does for m > 1).
  bool prefill = false;
  PrefillDims pdims{};
  PrefillScratch pscratch{};
  // Expert parallelism (ep_world > 1): this rank's exchange region, the peers'
  // (IPC mappings, closed on destroy) and the EP scratch in the arena.
  bool ep = false;
  EpTables etab;  // host copy of the placement tables
  EpMap emap{};
  EpLayout elay{};
  EpScratch escr{};
  EpPeers epeers{};
  char* exchange = nullptr;
  std::vector<char*> opened;
  bool ep_connected = false;
  bool ep_local_group = false;
  uint64_t ep_wait_ns = 20ull * 1000 * 1000 * 1000;  // UOCR_EP_WAIT_MS at creation, default 20 s
  // The shared expert's stream under expert parallelism (overlaps the pull).
  cudaStream_t ep_side = nullptr;
  cudaEvent_t ep_fork = nullptr, ep_join = nullptr;

  // Captured forward_stack graphs, keyed by (h, rows, stream); least recently used evicted.
  struct GraphEntry {
    const float* h;
    int64_t rows;
    cudaStream_t stream;
    cudaGraphExec_t exec;
    uint64_t last_use;
  };
  std::vector<GraphEntry> graphs;
  uint64_t tick = 0;
  static constexpr size_t kMaxGraphs = 8;

  size_t elem_bytes() const { return d.weight_format == UOCR_WEIGHT_INT8 ? 1 : 2; }

  // Routed experts whose weights this plan holds (its own under expert parallelism).
  int64_t held_experts() const { return ep ? emap.local : d.routed_experts; }
  // Global id of held expert i (slot i under expert parallelism).
  int64_t held_expert(int64_t i) const {
    return ep ? etab.slot_expert[static_cast<size_t>(emap.rank) * etab.max_local + static_cast<size_t>(i)] : i;
  }

  void carve_layer(Carver& c, LayerDev& L) const {
    const size_t H = d.hidden, F = d.expert_ffn, S = d.shared_ffn, eb = elem_bytes();
    const size_t E = static_cast<size_t>(held_experts());
    L.router = c.take<float>(static_cast<size_t>(d.routed_experts) * H);
    L.bias = d.router_bias ? c.take<float>(static_cast<size_t>(d.routed_experts)) : nullptr;
    L.norm = pre_norm ? c.take<float>(H) : nullptr;
    L.gate = c.take<char>(E * F * H * eb);
    L.up = c.take<char>(E * F * H * eb);
    L.down = c.take<char>(E * H * F * eb);
    L.sgate = c.take<char>(S * H * eb);
    L.sup = c.take<char>(S * H * eb);
    L.sdown = c.take<char>(H * S * eb);
    if (d.weight_format == UOCR_WEIGHT_INT8) {
      L.gate_s = c.take<float>(E * F);
      L.up_s = c.take<float>(E * F);
      L.down_s = c.take<float>(E * H);
      L.sgate_s = c.take<float>(S);
      L.sup_s = c.take<float>(S);
      L.sdown_s = c.take<float>(H);
    }
  }

  void carve_arena(Carver& c) {
    const size_t rows = d.max_rows, E = d.routed_experts, K = d.experts_per_token, F = d.expert_ffn,
                 S = d.shared_ffn, dr = decode_rows;
    logits = c.take<float>(rows * E);
    ids = c.take<int>(rows * K);
    weights = c.take<float>(rows * K);
    route = c.take<DecodeRoute>(1);
    act = c.take<__nv_bfloat16>(dr * K * F);
    act_s = c.take<__nv_bfloat16>(dr * (S > 0 ? S : 1));
    counter = c.take<unsigned>(1);
    err = c.take<ErrorWord>(1);
    if (pre_norm && (prefill || ep)) xnorm = c.take<float>(rows * static_cast<size_t>(d.hidden));
    if (prefill && d.weight_format == UOCR_WEIGHT_INT8)
      wexp = c.take<__nv_bfloat16>(3 * static_cast<size_t>(d.routed_experts) * F * d.hidden +
                                   3 * S * static_cast<size_t>(d.hidden));
    if (prefill) {
      char* base = c.take<char>(prefill_scratch_bytes(pdims, !ep));
      carve_prefill_scratch(pdims, base, &pscratch, !ep);
    }
    if (ep) {
      char* base = c.take<char>(ep_scratch_bytes(pdims, elay, emap));
      carve_ep_scratch(pdims, elay, emap, base, &escr);
      emap.owner = c.take<int>(etab.owner.size());
      emap.slot = c.take<int>(etab.slot.size());
      emap.slot_expert = c.take<int>(etab.slot_expert.size());
    }
  }
};

namespace {

// Shared body of the expert_ffn_one mirrors: scratch from cudaMallocAsync on
// the stream, as the reference's expert_ffn does (gemv_ops.cu:176,182). A bad
// expert id is recorded in the device's op-level error word, which
// uocr_ops_check reads.
template <typename Launch>
int ffn_one(const float* x, int64_t hidden, int64_t ffn, const int64_t* ids, const float* weights, int64_t k,
            float* out, int64_t experts_hint, cudaStream_t stream, Launch&& launch) {
  if (hidden <= 0 || hidden % 16 != 0 || ffn <= 0 || ffn % 16 != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one: hidden and ffn must be positive multiples of 16");
  if (k <= 0 || k > kMaxTopK) return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one: k must be in [1, 8]");
  if (x == nullptr || ids == nullptr || weights == nullptr || out == nullptr)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one: null pointer");
  const size_t route_off = 0, act_off = align_up(sizeof(DecodeRoute), 256),
               total = act_off + static_cast<size_t>(k * ffn) * 2;
  ErrorWord* err = nullptr;
  UOCR_TRY(ops_error_word(&err), "expert_ffn_one: error word");
  char* scratch = nullptr;
  UOCR_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), total, stream), "expert_ffn_one: scratch");
  auto* route = reinterpret_cast<DecodeRoute*>(scratch + route_off);
  auto* act = reinterpret_cast<__nv_bfloat16*>(scratch + act_off);
  cudaError_t st =
      launch_route_from_ids(ids, weights, static_cast<int>(k), static_cast<int>(experts_hint), route, err, stream);
  if (st == cudaSuccess) st = launch(route, act, err);
  cudaFreeAsync(scratch, stream);
  if (st != cudaSuccess) return cuda_fail(st, "expert_ffn_one");
  return UOCR_OK;
}

int device_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 1;
}

}  // namespace

extern "C" {

const char* uocr_last_error(void) { return g_error.c_str(); }
int uocr_abi_version(void) { return UOCR_MOE_ABI_VERSION; }

int uocr_moe_plan_create(const uocr_moe_desc* desc, uocr_moe_plan** out) {
  if (desc == nullptr || out == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: null argument");
  *out = nullptr;
  const uocr_moe_desc& d = *desc;
  if (d.hidden <= 0 || d.hidden % 16 != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: hidden must be a positive multiple of 16");
  if (d.routed_experts <= 0 || d.routed_experts > kMaxExperts)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: routed_experts must be in [1, 128]");
  if (d.experts_per_token <= 0 || d.experts_per_token > kMaxTopK || d.experts_per_token > d.routed_experts)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: experts_per_token must be in [1, min(8, experts)]");
  if (d.expert_ffn <= 0 || d.expert_ffn % 16 != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: expert_ffn must be a positive multiple of 16");
  if (d.shared_ffn < 0 || d.shared_ffn % 16 != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: shared_ffn must be a non-negative multiple of 16");
  if (d.layers <= 0 || d.max_rows <= 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: layers and max_rows must be positive");
  if (d.weight_format != UOCR_WEIGHT_BF16 && d.weight_format != UOCR_WEIGHT_INT8)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: weight_format must be bf16 (0) or int8 (1)");
  const bool pre_norm = (d.flags & UOCR_PLAN_PRE_NORM) != 0;
  if (pre_norm && !(d.rms_norm_eps >= 0.0f && d.rms_norm_eps < 1.0e30f))
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: rms_norm_eps must be a finite value >= 0");
  const bool ep = d.ep_world > 1;
  if (d.ep_world < 0 || d.ep_world > kMaxEpRanks)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: ep_world must be in [0, 8]");
  if (ep) {
    if (d.ep_rank < 0 || d.ep_rank >= d.ep_world)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: ep_rank must be in [0, ep_world)");
    if (d.weight_format != UOCR_WEIGHT_BF16 ||
        !prefill_shapes_ok(static_cast<int>(d.hidden), static_cast<int>(d.expert_ffn), static_cast<int>(d.shared_ffn)))
      return fail(UOCR_ERR_UNSUPPORTED,
                  "plan_create: expert parallelism runs the prefill path: bf16 weights, hidden % 256 == 0, "
                  "expert_ffn and shared_ffn % 128 == 0");
  }
  EpTables tabs;
  if (ep) {
    std::string why;
    if (!build_ep_tables(static_cast<int>(d.routed_experts), d.ep_world, d.ep_owner,
                         (d.flags & UOCR_PLAN_EP_STRIDED) != 0, &tabs, &why))
      return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: expert placement: " + why);
  }
  int ndev = 0;
  UOCR_TRY(cudaGetDeviceCount(&ndev), "plan_create: cudaGetDeviceCount");
  if (d.device < 0 || d.device >= ndev) return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_create: no such device");
  DeviceGuard guard(d.device);

  auto* p = new uocr_moe_plan;
  p->d = d;
  p->pre_norm = pre_norm;
  UOCR_TRY(cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, d.device), "plan_create: SM count");
  int smem_optin = 0;
  UOCR_TRY(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d.device),
           "plan_create: shared memory limit");
  // The decode kernels stage the batch's rows in shared memory (the router
  // also holds ~5 KB of static shared memory of its own).
  // (An expert-parallel plan runs every row count through the prefill path.)
  int dr = ep ? 0 : static_cast<int>(d.max_rows < kDecodeMaxRows ? d.max_rows : kDecodeMaxRows);
  while (dr > 0 && router_decode_smem(dr, static_cast<int>(d.hidden), static_cast<int>(d.routed_experts),
                                      pre_norm) + 8192 > static_cast<size_t>(smem_optin))
    --dr;
  p->decode_rows = dr;
  if (dr > 0) {
    cudaError_t pst = prepare_router_decode();
    if (pst == cudaSuccess) pst = prepare_decode_experts(dr, static_cast<int>(d.hidden));
    if (pst != cudaSuccess) {
      delete p;
      return cuda_fail(pst, "plan_create: kernel set-up");
    }
  }
  // Rows above the decode limit run the prefill path: the tile multiples of
  // the tensor-core grouped GEMM (int8 weights are expanded to bf16 per layer).
  p->prefill = d.max_rows > dr && prefill_shapes_ok(static_cast<int>(d.hidden), static_cast<int>(d.expert_ffn),
                                                    static_cast<int>(d.shared_ffn));
  p->pdims = PrefillDims{static_cast<int>(d.max_rows), static_cast<int>(d.hidden), static_cast<int>(d.routed_experts),
                         static_cast<int>(d.experts_per_token), static_cast<int>(d.expert_ffn),
                         static_cast<int>(d.shared_ffn), d.renormalize};
  if (ep) {
    p->ep = true;
    const int W = d.ep_world;
    p->etab = std::move(tabs);
    p->emap = EpMap{W, d.ep_rank, static_cast<int>(d.routed_experts),
                    p->etab.slot_count[static_cast<size_t>(d.ep_rank)], p->etab.max_local, nullptr, nullptr, nullptr};
    p->elay = ep_layout(p->pdims, p->emap);
    if (const char* v = std::getenv("UOCR_EP_WAIT_MS")) {
      const long long ms = std::atoll(v);
      if (ms > 0) p->ep_wait_ns = static_cast<uint64_t>(ms) * 1000000ull;
    }
  }

  Carver probe{nullptr};
  LayerDev tmp;
  p->carve_layer(probe, tmp);
  const size_t layer_bytes = align_up(probe.off, 256);
  p->layers.resize(static_cast<size_t>(d.layers));
  for (auto& L : p->layers) {
    cudaError_t st = cudaMalloc(&L.block, layer_bytes);
    if (st != cudaSuccess) {
      uocr_moe_plan_destroy(p);
      return cuda_fail(st, "plan_create: weight allocation");
    }
    L.bytes = layer_bytes;
    Carver c{static_cast<char*>(L.block)};
    p->carve_layer(c, L);
    p->weight_bytes += layer_bytes;
  }
  Carver ap{nullptr};
  p->carve_arena(ap);
  p->arena_bytes = align_up(ap.off, 256);
  cudaError_t st = cudaMalloc(&p->arena, p->arena_bytes);
  if (st != cudaSuccess) {
    uocr_moe_plan_destroy(p);
    return cuda_fail(st, "plan_create: arena allocation");
  }
  Carver ac{p->arena};
  p->carve_arena(ac);
  st = cudaMemset(p->arena, 0, p->arena_bytes);
  if (st == cudaSuccess && p->ep) {
    const EpTables& t = p->etab;
    st = cudaMemcpy(const_cast<int*>(p->emap.owner), t.owner.data(), t.owner.size() * 4, cudaMemcpyHostToDevice);
    if (st == cudaSuccess)
      st = cudaMemcpy(const_cast<int*>(p->emap.slot), t.slot.data(), t.slot.size() * 4, cudaMemcpyHostToDevice);
    if (st == cudaSuccess)
      st = cudaMemcpy(const_cast<int*>(p->emap.slot_expert), t.slot_expert.data(), t.slot_expert.size() * 4,
                      cudaMemcpyHostToDevice);
  }
  if (st != cudaSuccess) {
    uocr_moe_plan_destroy(p);
    return cuda_fail(st, "plan_create: arena clear");
  }
  if (p->ep) {
    // A block of its own: CUDA IPC exports whole cudaMalloc allocations.
    st = cudaMalloc(&p->exchange, p->elay.bytes);
    if (st == cudaSuccess) st = cudaMemset(p->exchange, 0, p->elay.bytes);
    if (st == cudaSuccess) st = cudaStreamCreateWithFlags(&p->ep_side, cudaStreamNonBlocking);
    if (st == cudaSuccess) st = cudaEventCreateWithFlags(&p->ep_fork, cudaEventDisableTiming);
    if (st == cudaSuccess) st = cudaEventCreateWithFlags(&p->ep_join, cudaEventDisableTiming);
    if (st != cudaSuccess) {
      uocr_moe_plan_destroy(p);
      return cuda_fail(st, "plan_create: exchange region");
    }
    p->arena_bytes += p->elay.bytes;
    p->pscratch.seg_count = reinterpret_cast<int*>(p->exchange + p->elay.seg_count);
    p->pscratch.seg_start = reinterpret_cast<int*>(p->exchange + p->elay.seg_start);
    p->pscratch.xperm = nullptr;  // the owners pull rows straight from x^
    p->pscratch.xhat = reinterpret_cast<__nv_bfloat16*>(p->exchange + p->elay.xhat);
    p->pscratch.yperm = reinterpret_cast<__nv_bfloat16*>(p->exchange + p->elay.yback);
    p->epeers.base[p->emap.rank] = p->exchange;
  }
  *out = p;
  return UOCR_OK;
}

int uocr_moe_plan_destroy(uocr_moe_plan* p) {
  if (p == nullptr) return UOCR_OK;
  DeviceGuard guard(p->d.device);
  for (auto& g : p->graphs) cudaGraphExecDestroy(g.exec);
  for (auto& L : p->layers)
    if (L.block != nullptr) cudaFree(L.block);
  if (p->arena != nullptr) cudaFree(p->arena);
  for (char* q : p->opened) cudaIpcCloseMemHandle(q);
  if (p->exchange != nullptr) cudaFree(p->exchange);
  if (p->ep_fork != nullptr) cudaEventDestroy(p->ep_fork);
  if (p->ep_join != nullptr) cudaEventDestroy(p->ep_join);
  if (p->ep_side != nullptr) cudaStreamDestroy(p->ep_side);
  delete p;
  return UOCR_OK;
}

int uocr_moe_plan_bytes(const uocr_moe_plan* p, int64_t* weight_bytes, int64_t* arena_bytes) {
  if (p == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "plan_bytes: null plan");
  if (weight_bytes) *weight_bytes = static_cast<int64_t>(p->weight_bytes);
  if (arena_bytes) *arena_bytes = static_cast<int64_t>(p->arena_bytes);
  return UOCR_OK;
}

namespace {

// Brings one matrix [rows, cols] into the plan's format at `dst` (+ scales).
int upload_matrix(const uocr_moe_plan* p, const uocr_moe_layer_src& src, const void* from, int64_t rows,
                  int64_t cols, void* dst, float* scales, cudaStream_t stream, const char* name) {
  if (rows * cols == 0) return UOCR_OK;
  if (from == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, std::string("set_layer: missing ") + name);
  const size_t sb = src.dtype == UOCR_DTYPE_BF16 ? 2 : 4;
  const size_t n = static_cast<size_t>(rows * cols);
  const void* dev_src = from;
  void* staging = nullptr;
  if (src.memory == UOCR_MEMORY_HOST) {
    UOCR_TRY(cudaMallocAsync(&staging, n * sb, stream), "set_layer: staging allocation");
    const cudaError_t up = cudaMemcpyAsync(staging, from, n * sb, cudaMemcpyHostToDevice, stream);
    if (up != cudaSuccess) {
      cudaFreeAsync(staging, stream);
      return cuda_fail(up, "set_layer: upload");
    }
    dev_src = staging;
  }
  cudaError_t st = cudaSuccess;
  if (p->d.weight_format == UOCR_WEIGHT_INT8) {
    st = launch_quantize_rows(dev_src, src.dtype == UOCR_DTYPE_BF16, rows, cols, cols, static_cast<int8_t*>(dst),
                              scales, stream);
  } else if (src.dtype == UOCR_DTYPE_BF16) {
    st = cudaMemcpyAsync(dst, dev_src, n * 2, cudaMemcpyDeviceToDevice, stream);
  } else {
    st = launch_f32_to_bf16(static_cast<const float*>(dev_src), static_cast<__nv_bfloat16*>(dst),
                            static_cast<int64_t>(n), stream);
  }
  if (staging != nullptr) cudaFreeAsync(staging, stream);
  if (st != cudaSuccess) return cuda_fail(st, "set_layer: conversion");
  if (src.memory == UOCR_MEMORY_HOST) UOCR_TRY(cudaStreamSynchronize(stream), "set_layer: upload wait");
  return UOCR_OK;
}

int copy_f32(const uocr_moe_layer_src& src, const float* from, float* dst, size_t n, cudaStream_t stream,
             const char* name) {
  if (from == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, std::string("set_layer: missing ") + name);
  UOCR_TRY(cudaMemcpyAsync(dst, from, n * 4,
                           src.memory == UOCR_MEMORY_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                           stream),
           "set_layer: fp32 copy");
  return UOCR_OK;
}

}  // namespace

int uocr_moe_set_layer(uocr_moe_plan* p, int64_t layer, const uocr_moe_layer_src* src, void* stream_v) {
  if (p == nullptr || src == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer: null argument");
  if (layer < 0 || layer >= p->d.layers) return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer: layer out of range");
  if (src->memory != UOCR_MEMORY_HOST && src->memory != UOCR_MEMORY_DEVICE)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer: memory must be host (0) or device (1)");
  if (src->dtype != UOCR_DTYPE_F32 && src->dtype != UOCR_DTYPE_BF16)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer: dtype must be f32 (0) or bf16 (1)");
  if (p->d.router_bias && src->router_bias == nullptr)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer: the plan expects a router bias");
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  LayerDev& L = p->layers[static_cast<size_t>(layer)];
  const int64_t H = p->d.hidden, E = p->d.routed_experts, F = p->d.expert_ffn, S = p->d.shared_ffn;
  int rc = copy_f32(*src, src->router, L.router, static_cast<size_t>(E * H), stream, "router");
  if (rc == UOCR_OK && p->d.router_bias) rc = copy_f32(*src, src->router_bias, L.bias, E, stream, "router_bias");
  if (rc == UOCR_OK && p->pre_norm) {
    if (src->norm != nullptr)
      rc = copy_f32(*src, src->norm, L.norm, static_cast<size_t>(H), stream, "norm");
    else
      UOCR_TRY(launch_fill_f32(L.norm, 1.0f, H, stream), "set_layer: unit norm gain");
  }
  if (!p->ep) {
    if (rc == UOCR_OK) rc = upload_matrix(p, *src, src->gate, E * F, H, L.gate, L.gate_s, stream, "gate");
    if (rc == UOCR_OK) rc = upload_matrix(p, *src, src->up, E * F, H, L.up, L.up_s, stream, "up");
    if (rc == UOCR_OK) rc = upload_matrix(p, *src, src->down, E * H, F, L.down, L.down_s, stream, "down");
  } else {
    // Expert parallelism: only this rank's experts, from the full stacks.
    const size_t sb = src->dtype == UOCR_DTYPE_BF16 ? 2 : 4, eb = p->elem_bytes();
    auto at = [](const void* base, size_t bytes) {
      return base == nullptr ? nullptr : static_cast<const char*>(base) + bytes;
    };
    for (int i = 0; i < p->emap.local && rc == UOCR_OK; ++i) {
      const int64_t e = p->held_expert(i);
      char* g = static_cast<char*>(L.gate) + static_cast<size_t>(i * F * H) * eb;
      char* u = static_cast<char*>(L.up) + static_cast<size_t>(i * F * H) * eb;
      char* dn = static_cast<char*>(L.down) + static_cast<size_t>(i * H * F) * eb;
      rc = upload_matrix(p, *src, at(src->gate, static_cast<size_t>(e * F * H) * sb), F, H, g, nullptr, stream, "gate");
      if (rc == UOCR_OK)
        rc = upload_matrix(p, *src, at(src->up, static_cast<size_t>(e * F * H) * sb), F, H, u, nullptr, stream, "up");
      if (rc == UOCR_OK)
        rc = upload_matrix(p, *src, at(src->down, static_cast<size_t>(e * H * F) * sb), H, F, dn, nullptr, stream,
                           "down");
    }
  }
  if (rc == UOCR_OK && S > 0) {
    rc = upload_matrix(p, *src, src->shared_gate, S, H, L.sgate, L.sgate_s, stream, "shared_gate");
    if (rc == UOCR_OK) rc = upload_matrix(p, *src, src->shared_up, S, H, L.sup, L.sup_s, stream, "shared_up");
    if (rc == UOCR_OK) rc = upload_matrix(p, *src, src->shared_down, H, S, L.sdown, L.sdown_s, stream, "shared_down");
  }
  if (rc == UOCR_OK && src->memory == UOCR_MEMORY_HOST)
    UOCR_TRY(cudaStreamSynchronize(stream), "set_layer: host copies");
  if (rc == UOCR_OK) L.loaded = true;
  return rc;
}

namespace {

// fp32 [n] from an fp32 or bf16 source on the host or the device; bf16 is
// widened exactly on the device.
int copy_widen(int32_t memory, int32_t dtype, const void* from, float* dst, size_t n, cudaStream_t stream,
               const char* name) {
  if (from == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, std::string("set_layer_parts: missing ") + name);
  const cudaMemcpyKind kind = memory == UOCR_MEMORY_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  if (dtype == UOCR_DTYPE_F32) {
    UOCR_TRY(cudaMemcpyAsync(dst, from, n * 4, kind, stream), "set_layer_parts: fp32 copy");
    return UOCR_OK;
  }
  const void* dev = from;
  void* staging = nullptr;
  if (memory == UOCR_MEMORY_HOST) {
    UOCR_TRY(cudaMallocAsync(&staging, n * 2, stream), "set_layer_parts: staging allocation");
    const cudaError_t st = cudaMemcpyAsync(staging, from, n * 2, kind, stream);
    if (st != cudaSuccess) {
      cudaFreeAsync(staging, stream);
      return cuda_fail(st, "set_layer_parts: upload");
    }
    dev = staging;
  }
  const cudaError_t st = launch_bf16_to_f32(static_cast<const __nv_bfloat16*>(dev), dst, static_cast<int64_t>(n), stream);
  if (staging != nullptr) cudaFreeAsync(staging, stream);
  if (st != cudaSuccess) return cuda_fail(st, "set_layer_parts: widening");
  return UOCR_OK;
}

}  // namespace

int uocr_moe_set_layer_parts(uocr_moe_plan* p, int64_t layer, const uocr_moe_layer_parts* src, void* stream_v) {
  if (p == nullptr || src == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: null argument");
  if (layer < 0 || layer >= p->d.layers)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: layer out of range");
  if (src->memory != UOCR_MEMORY_HOST && src->memory != UOCR_MEMORY_DEVICE)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: memory must be host (0) or device (1)");
  if (src->dtype != UOCR_DTYPE_F32 && src->dtype != UOCR_DTYPE_BF16)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: dtype must be f32 (0) or bf16 (1)");
  if (p->d.router_bias && src->router_bias == nullptr)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: the plan expects a router bias");
  const int64_t H = p->d.hidden, E = p->d.routed_experts, F = p->d.expert_ffn, S = p->d.shared_ffn;
  if (E > 0 && (src->gate == nullptr || src->up == nullptr || src->down == nullptr))
    return fail(UOCR_ERR_INVALID_ARGUMENT, "set_layer_parts: gate, up and down must each list the experts");
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  LayerDev& L = p->layers[static_cast<size_t>(layer)];
  uocr_moe_layer_src ms{};  // the memory and dtype upload_matrix reads
  ms.memory = src->memory;
  ms.dtype = src->dtype;
  int rc = copy_widen(src->memory, src->dtype, src->router, L.router, static_cast<size_t>(E * H), stream, "router");
  if (rc == UOCR_OK && p->d.router_bias)
    rc = copy_widen(src->memory, src->dtype, src->router_bias, L.bias, static_cast<size_t>(E), stream, "router_bias");
  if (rc == UOCR_OK && p->pre_norm) {
    if (src->norm != nullptr)
      rc = copy_widen(src->memory, src->dtype, src->norm, L.norm, static_cast<size_t>(H), stream, "norm");
    else
      UOCR_TRY(launch_fill_f32(L.norm, 1.0f, H, stream), "set_layer_parts: unit norm gain");
  }
  // Held expert i is expert e of the checkpoint (i == e without expert
  // parallelism); its rows go to row block i of the stacks.
  const size_t eb = p->elem_bytes();
  for (int64_t i = 0; i < p->held_experts() && rc == UOCR_OK; ++i) {
    const int64_t e = p->held_expert(i);
    char* g = static_cast<char*>(L.gate) + static_cast<size_t>(i * F * H) * eb;
    char* u = static_cast<char*>(L.up) + static_cast<size_t>(i * F * H) * eb;
    char* dn = static_cast<char*>(L.down) + static_cast<size_t>(i * H * F) * eb;
    float* gs = L.gate_s != nullptr ? L.gate_s + i * F : nullptr;
    float* us = L.up_s != nullptr ? L.up_s + i * F : nullptr;
    float* ds = L.down_s != nullptr ? L.down_s + i * H : nullptr;
    rc = upload_matrix(p, ms, src->gate[e], F, H, g, gs, stream, "gate");
    if (rc == UOCR_OK) rc = upload_matrix(p, ms, src->up[e], F, H, u, us, stream, "up");
    if (rc == UOCR_OK) rc = upload_matrix(p, ms, src->down[e], H, F, dn, ds, stream, "down");
  }
  if (rc == UOCR_OK && S > 0) {
    rc = upload_matrix(p, ms, src->shared_gate, S, H, L.sgate, L.sgate_s, stream, "shared_gate");
    if (rc == UOCR_OK) rc = upload_matrix(p, ms, src->shared_up, S, H, L.sup, L.sup_s, stream, "shared_up");
    if (rc == UOCR_OK) rc = upload_matrix(p, ms, src->shared_down, H, S, L.sdown, L.sdown_s, stream, "shared_down");
  }
  if (rc == UOCR_OK && src->memory == UOCR_MEMORY_HOST)
    UOCR_TRY(cudaStreamSynchronize(stream), "set_layer_parts: host copies");
  if (rc == UOCR_OK) L.loaded = true;
  return rc;
}

int uocr_moe_load_layer(uocr_moe_plan* p, const uocr_checkpoint* ckpt, int64_t layer, int64_t plan_layer,
                        void* stream) {
  if (p == nullptr || ckpt == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "load_layer: null argument");
  if (layer < 0) return fail(UOCR_ERR_INVALID_ARGUMENT, "load_layer: layer out of range");
  if (p->d.router_bias)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "load_layer: the plan expects a router bias, which the checkpoint does not hold");
  const int64_t H = p->d.hidden, E = p->d.routed_experts, F = p->d.expert_ffn, S = p->d.shared_ffn;
  const std::string pre = "model.layers." + std::to_string(layer) + ".";
  int dtype = -1;
  // The tensor's data if it is present with this shape and the layer's one dtype.
  auto get = [&](const std::string& name, std::vector<int64_t> shape, const void** out) -> int {
    const CkTensor* t = checkpoint_find(ckpt, name);
    if (t == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "load_layer: missing " + name);
    if (t->dtype != UOCR_DTYPE_BF16 && t->dtype != UOCR_DTYPE_F32)
      return fail(UOCR_ERR_INVALID_ARGUMENT,
                  "load_layer: " + name + ": dtype " + dtype_name(t->dtype) + ", expected BF16 or F32");
    if (dtype >= 0 && t->dtype != dtype)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "load_layer: layer " + std::to_string(layer) + ": mixed dtypes");
    dtype = t->dtype;
    if (t->shape != shape) {
      auto text = [](const std::vector<int64_t>& v) {
        std::string s = "[";
        for (size_t k = 0; k < v.size(); ++k) s += (k ? ", " : "") + std::to_string(v[k]);
        return s + "]";
      };
      return fail(UOCR_ERR_INVALID_ARGUMENT,
                  "load_layer: " + name + ": shape " + text(t->shape) + ", expected " + text(shape));
    }
    *out = t->data;
    return UOCR_OK;
  };
  uocr_moe_layer_parts parts{};
  parts.memory = UOCR_MEMORY_HOST;
  std::vector<const void*> g(static_cast<size_t>(E)), u(static_cast<size_t>(E)), dn(static_cast<size_t>(E));
  int rc = get(pre + "mlp.gate.weight", {E, H}, &parts.router);
  if (rc == UOCR_OK) rc = get(pre + "post_attention_layernorm.weight", {H}, &parts.norm);
  for (int64_t e = 0; e < E && rc == UOCR_OK; ++e) {
    const std::string q = pre + "mlp.experts." + std::to_string(e) + ".";
    rc = get(q + "gate_proj.weight", {F, H}, &g[static_cast<size_t>(e)]);
    if (rc == UOCR_OK) rc = get(q + "up_proj.weight", {F, H}, &u[static_cast<size_t>(e)]);
    if (rc == UOCR_OK) rc = get(q + "down_proj.weight", {H, F}, &dn[static_cast<size_t>(e)]);
  }
  if (rc == UOCR_OK && S > 0) {
    const std::string q = pre + "mlp.shared_experts.";
    rc = get(q + "gate_proj.weight", {S, H}, &parts.shared_gate);
    if (rc == UOCR_OK) rc = get(q + "up_proj.weight", {S, H}, &parts.shared_up);
    if (rc == UOCR_OK) rc = get(q + "down_proj.weight", {H, S}, &parts.shared_down);
  }
  if (rc != UOCR_OK) return rc;
  parts.dtype = dtype;
  parts.gate = g.data();
  parts.up = u.data();
  parts.down = dn.data();
  return uocr_moe_set_layer_parts(p, plan_layer, &parts, stream);
}

namespace {

constexpr int kMaxProfileKernels = 6;

const __nv_bfloat16* as_bf16(void* v) { return static_cast<const __nv_bfloat16*>(v); }

PrefillCall prefill_call(const uocr_moe_plan* p, const LayerDev& L, const float* x, int64_t rows, const float* resid,
                         float* y) {
  PrefillCall c{};
  c.dims = p->pdims;
  c.scratch = p->pscratch;
  c.rows = static_cast<int>(rows);
  c.x = x;
  c.router = L.router;
  c.bias = L.bias;
  c.gate = as_bf16(L.gate);
  c.up = as_bf16(L.up);
  c.down = as_bf16(L.down);
  c.sgate = as_bf16(L.sgate);
  c.sup = as_bf16(L.sup);
  c.sdown = as_bf16(L.sdown);
  c.logits = p->logits;
  c.ids = p->ids;
  c.weights = p->weights;
  c.resid = resid;
  c.y = y;
  c.err = p->err;
  c.sm_count = p->sm_count;
  c.events = nullptr;
  return c;
}

EpCall ep_call(const uocr_moe_plan* p, const LayerDev& L, const float* x, int64_t rows, const float* resid, float* y) {
  EpCall c{};
  c.pc = prefill_call(p, L, x, rows, resid, y);
  c.map = p->emap;
  c.peers = p->epeers;
  c.lay = p->elay;
  c.es = p->escr;
  c.gate_local = as_bf16(L.gate);
  c.up_local = as_bf16(L.up);
  c.down_local = as_bf16(L.down);
  c.wait_ns = p->ep_wait_ns;
  c.side = p->ep_side;
  c.fork = p->ep_fork;
  c.join = p->ep_join;
  return c;
}

// One layer on `rows` rows: route, then experts. resid != null adds the
// layer input back (the stack's residual); y may then alias resid. For
// measurement, ev (kMaxProfileKernels events) receives one event after each
// kernel of the path taken and *nev their count.
int run_layer(uocr_moe_plan* p, const LayerDev& L, const float* x, int64_t rows, const float* resid, float* y,
              cudaStream_t stream, cudaEvent_t* ev = nullptr, int* nev = nullptr) {
  const uocr_moe_desc& d = p->d;
  const int T = static_cast<int>(rows), H = static_cast<int>(d.hidden), E = static_cast<int>(d.routed_experts),
            K = static_cast<int>(d.experts_per_token), F = static_cast<int>(d.expert_ffn),
            S = static_cast<int>(d.shared_ffn);
  const RowNorm norm{L.norm, d.rms_norm_eps, p->pre_norm ? 1 : 0};
  // The prefill and expert-parallel paths read normalised rows from a copy.
  if (p->pre_norm && (p->ep || rows > p->decode_rows) && rows > 0) {
    UOCR_TRY(launch_rms_norm_rows(x, rows, H, norm, p->xnorm, stream), "forward: pre-norm");
    x = p->xnorm;
  }
  if (p->ep) {
    EpCall c = ep_call(p, L, x, rows, resid, y);
    UOCR_TRY(ep_forward(c, stream, ev), "forward: expert-parallel prefill");
    if (nev != nullptr) *nev = 6;
    return UOCR_OK;
  }
  if (rows > p->decode_rows) {
    if (!p->prefill)
      return fail(UOCR_ERR_UNSUPPORTED,
                  "forward: more than 16 rows needs the prefill path: hidden % 256 == 0, "
                  "expert_ffn and shared_ffn % 128 == 0");
    PrefillCall c = prefill_call(p, L, x, rows, resid, y);
    if (d.weight_format == UOCR_WEIGHT_INT8) {
      // The reference's m > 1 int8 path: expand to bf16, then the bf16 GEMMs.
      const int64_t EF = static_cast<int64_t>(E) * F, EH = static_cast<int64_t>(E) * H;
      __nv_bfloat16* g = p->wexp;
      __nv_bfloat16* u = g + EF * H;
      __nv_bfloat16* dn = u + EF * H;
      __nv_bfloat16* sg = dn + EH * F;
      __nv_bfloat16* su = sg + static_cast<int64_t>(S) * H;
      __nv_bfloat16* sd = su + static_cast<int64_t>(S) * H;
      auto q8 = [](void* v) { return static_cast<const int8_t*>(v); };
      UOCR_TRY(launch_dequant_rows(q8(L.gate), L.gate_s, EF, H, g, stream), "forward: int8 expansion");
      UOCR_TRY(launch_dequant_rows(q8(L.up), L.up_s, EF, H, u, stream), "forward: int8 expansion");
      UOCR_TRY(launch_dequant_rows(q8(L.down), L.down_s, EH, F, dn, stream), "forward: int8 expansion");
      if (S > 0) {
        UOCR_TRY(launch_dequant_rows(q8(L.sgate), L.sgate_s, S, H, sg, stream), "forward: int8 expansion");
        UOCR_TRY(launch_dequant_rows(q8(L.sup), L.sup_s, S, H, su, stream), "forward: int8 expansion");
        UOCR_TRY(launch_dequant_rows(q8(L.sdown), L.sdown_s, H, S, sd, stream), "forward: int8 expansion");
      }
      c.gate = g;
      c.up = u;
      c.down = dn;
      c.sgate = sg;
      c.sup = su;
      c.sdown = sd;
    }
    c.events = ev;
    UOCR_TRY(launch_prefill(c, stream), "forward: prefill");
    if (nev != nullptr) *nev = 6;
    return UOCR_OK;
  }
  // Programmatic dependent launch chains router -> gate/up -> down (and the
  // next layer's router); the profiling path records events between them instead.
  const bool pdl = ev == nullptr;
  // The router builds the routing table once; the expert kernels copy it.
  const RouteOut ro{p->route, K, d.renormalize, p->ids, p->weights, p->counter, p->err};
  UOCR_TRY(launch_router_logits(x, T, H, L.router, L.bias, E, p->logits, stream, pdl, &ro, norm), "forward: router");
  if (ev != nullptr) UOCR_TRY(cudaEventRecord(ev[0], stream), "forward: event");
  cudaEvent_t between = ev != nullptr ? ev[1] : nullptr;
  const DecodeRouting routing{nullptr, p->route, E, K, d.renormalize, nullptr, nullptr};
  if (d.weight_format == UOCR_WEIGHT_BF16) {
    auto b = [](void* v) { return static_cast<const __nv_bfloat16*>(v); };
    UOCR_TRY(launch_decode_experts_bf16(x, T, H, F, S, b(L.gate), b(L.up), b(L.down), b(L.sgate), b(L.sup),
                                        b(L.sdown), routing, p->act, p->act_s, resid, y, p->err, p->sm_count,
                                        stream, between, pdl, norm),
             "forward: experts");
  } else {
    auto q = [](void* v, float* s, int64_t cols) { return Q8Rows{static_cast<const int8_t*>(v), s, cols}; };
    UOCR_TRY(launch_decode_experts_q8(x, T, H, F, S, q(L.gate, L.gate_s, H), q(L.up, L.up_s, H),
                                      q(L.down, L.down_s, F), q(L.sgate, L.sgate_s, H), q(L.sup, L.sup_s, H),
                                      q(L.sdown, L.sdown_s, S), routing, p->act, p->act_s, resid, y, p->err,
                                      p->sm_count, stream, between, pdl, norm),
             "forward: experts");
  }
  if (ev != nullptr) UOCR_TRY(cudaEventRecord(ev[2], stream), "forward: event");
  if (nev != nullptr) *nev = 3;
  return UOCR_OK;
}

}  // namespace

namespace {

// An expert-parallel plan forwards only once connected, and virtual ranks of
// a local group only through uocr_moe_ep_forward_local.
int ep_ready(const uocr_moe_plan* p, const char* what) {
  if (!p->ep) return UOCR_OK;
  if (!p->ep_connected)
    return fail(UOCR_ERR_INVALID_ARGUMENT, std::string(what) + ": expert-parallel plan not connected");
  if (p->ep_local_group)
    return fail(UOCR_ERR_INVALID_ARGUMENT, std::string(what) + ": local-group ranks run through ep_forward_local");
  return UOCR_OK;
}

}  // namespace

int uocr_moe_forward(uocr_moe_plan* p, int64_t layer, const float* x, int64_t rows, float* y, int32_t* ids,
                     float* weights, void* stream_v) {
  if (p == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: null plan");
  if (layer < 0 || layer >= p->d.layers) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: layer out of range");
  if (rows < 0 || rows > p->d.max_rows) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: rows outside [0, max_rows]");
  if (int rc = ep_ready(p, "forward"); rc != UOCR_OK) return rc;
  if (rows == 0 && !p->ep) return UOCR_OK;  // an expert-parallel rank takes part with no rows
  if (rows > 0 && (x == nullptr || y == nullptr)) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: null x or y");
  if (rows > 0 && x == y) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: x and y must not overlap");
  if (rows > 0 && (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: x must be 16-byte aligned");
  const LayerDev& L = p->layers[static_cast<size_t>(layer)];
  if (!L.loaded) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward: layer weights not set");
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  int rc = run_layer(p, L, x, rows, nullptr, y, stream);
  if (rc != UOCR_OK) return rc;
  const size_t nk = static_cast<size_t>(rows * p->d.experts_per_token);
  if (ids != nullptr)
    UOCR_TRY(cudaMemcpyAsync(ids, p->ids, nk * 4, cudaMemcpyDeviceToDevice, stream), "forward: ids copy");
  if (weights != nullptr)
    UOCR_TRY(cudaMemcpyAsync(weights, p->weights, nk * 4, cudaMemcpyDeviceToDevice, stream), "forward: weights copy");
  return UOCR_OK;
}

int uocr_moe_router_logits(uocr_moe_plan* p, int64_t layer, const float* x, int64_t rows, float* logits,
                           void* stream_v) {
  if (p == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: null plan");
  if (layer < 0 || layer >= p->d.layers) return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: layer out of range");
  if (rows < 0 || rows > p->d.max_rows)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: rows outside [0, max_rows]");
  if (rows == 0) return UOCR_OK;
  if (x == nullptr || logits == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: null x or logits");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: x must be 16-byte aligned");
  const LayerDev& L = p->layers[static_cast<size_t>(layer)];
  if (!L.loaded) return fail(UOCR_ERR_INVALID_ARGUMENT, "router_logits: layer weights not set");
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  const uocr_moe_desc& d = p->d;
  const int T = static_cast<int>(rows), H = static_cast<int>(d.hidden), E = static_cast<int>(d.routed_experts);
  const RowNorm norm{L.norm, d.rms_norm_eps, p->pre_norm ? 1 : 0};
  if (rows > p->decode_rows || p->ep) {
    if (p->pre_norm) {
      UOCR_TRY(launch_rms_norm_rows(x, rows, H, norm, p->xnorm, stream), "router_logits: pre-norm");
      x = p->xnorm;
    }
    UOCR_TRY(launch_router_logits_rows(x, T, H, L.router, L.bias, E, logits, stream), "router_logits");
    return UOCR_OK;
  }
  const RouteOut ro{p->route, static_cast<int>(d.experts_per_token), d.renormalize, p->ids, p->weights, p->counter,
                    p->err};
  UOCR_TRY(launch_router_logits(x, T, H, L.router, L.bias, E, logits, stream, false, &ro, norm), "router_logits");
  return UOCR_OK;
}

int uocr_moe_forward_stack(uocr_moe_plan* p, float* h, int64_t rows, void* stream_v) {
  if (p == nullptr || (h == nullptr && rows > 0))
    return fail(UOCR_ERR_INVALID_ARGUMENT, "forward_stack: null argument");
  if (rows < 0 || rows > p->d.max_rows)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "forward_stack: rows outside [0, max_rows]");
  if (rows > 0 && (reinterpret_cast<uintptr_t>(h) & 15) != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "forward_stack: h must be 16-byte aligned");
  if (int rc = ep_ready(p, "forward_stack"); rc != UOCR_OK) return rc;
  if (rows == 0 && !p->ep) return UOCR_OK;
  for (const auto& L : p->layers)
    if (!L.loaded) return fail(UOCR_ERR_INVALID_ARGUMENT, "forward_stack: a layer's weights are not set");
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  auto run_all = [&]() {
    for (const auto& L : p->layers) {
      int rc = run_layer(p, L, h, rows, h, h, stream);
      if (rc != UOCR_OK) return rc;
    }
    return static_cast<int>(UOCR_OK);
  };
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  UOCR_TRY(cudaStreamIsCapturing(stream, &cap), "forward_stack: capture status");
  if ((p->d.flags & UOCR_PLAN_NO_GRAPHS) != 0 || cap != cudaStreamCaptureStatusNone || stream == nullptr ||
      stream == cudaStreamLegacy)
    return run_all();
  for (auto& g : p->graphs)
    if (g.h == h && g.rows == rows && g.stream == stream) {
      g.last_use = ++p->tick;
      UOCR_TRY(cudaGraphLaunch(g.exec, stream), "forward_stack: graph launch");
      return UOCR_OK;
    }
  // First call for this (h, rows, stream): capture the stack once.
  UOCR_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "forward_stack: begin capture");
  const int rc = run_all();
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(stream, &graph);
  if (rc != UOCR_OK) {
    if (graph != nullptr) cudaGraphDestroy(graph);
    return rc;
  }
  if (end != cudaSuccess) return cuda_fail(end, "forward_stack: end capture");
  cudaGraphExec_t exec = nullptr;
  const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (inst != cudaSuccess) return cuda_fail(inst, "forward_stack: instantiate");
  if (p->graphs.size() >= uocr_moe_plan::kMaxGraphs) {
    size_t oldest = 0;
    for (size_t i = 1; i < p->graphs.size(); ++i)
      if (p->graphs[i].last_use < p->graphs[oldest].last_use) oldest = i;
    cudaGraphExecDestroy(p->graphs[oldest].exec);
    p->graphs.erase(p->graphs.begin() + static_cast<std::ptrdiff_t>(oldest));
  }
  p->graphs.push_back({h, rows, stream, exec, ++p->tick});
  UOCR_TRY(cudaGraphLaunch(exec, stream), "forward_stack: graph launch");
  return UOCR_OK;
}

int uocr_moe_profile_stack(uocr_moe_plan* p, float* h, int64_t rows, int32_t iters, float* ms, void* stream_v) {
  if (p == nullptr || h == nullptr || ms == nullptr || iters <= 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "profile_stack: bad argument");
  if (rows <= 0 || rows > p->d.max_rows)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "profile_stack: rows outside [1, max_rows]");
  for (const auto& L : p->layers)
    if (!L.loaded) return fail(UOCR_ERR_INVALID_ARGUMENT, "profile_stack: a layer's weights are not set");
  if (int rc = ep_ready(p, "profile_stack"); rc != UOCR_OK) return rc;
  DeviceGuard guard(p->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  const size_t nl = p->layers.size();
  // Per layer pass: a start event, then one event after each kernel.
  constexpr size_t kSlot = kMaxProfileKernels + 1;
  const size_t passes = static_cast<size_t>(iters) * nl;
  std::vector<cudaEvent_t> ev(passes * kSlot);
  for (auto& e : ev) UOCR_TRY(cudaEventCreate(&e), "profile_stack: event");
  int rc = UOCR_OK;
  int nk = 0;
  if (p->ep) {
    // The ranks start the timed passes together: a device barrier first, so
    // that the skew of their host launches is not counted in the first wait.
    EpCall c = ep_call(p, p->layers[0], h, rows, h, h);
    UOCR_TRY(ep_arrive(c, stream), "profile_stack: barrier");
    UOCR_TRY(ep_wait(c, 63, stream), "profile_stack: barrier");
  }
  for (size_t j = 0; j < passes && rc == UOCR_OK; ++j) {
    rc = cudaEventRecord(ev[j * kSlot], stream) == cudaSuccess ? UOCR_OK : fail(UOCR_ERR_CUDA, "profile_stack: event");
    if (rc == UOCR_OK) rc = run_layer(p, p->layers[j % nl], h, rows, h, h, stream, &ev[j * kSlot + 1], &nk);
  }
  double sum[kMaxProfileKernels] = {};
  float total = 0;
  if (rc == UOCR_OK && cudaEventSynchronize(ev[(passes - 1) * kSlot + nk]) == cudaSuccess) {
    for (size_t j = 0; j < passes; ++j)
      for (int i = 0; i < nk; ++i) {
        float t = 0;
        cudaEventElapsedTime(&t, ev[j * kSlot + i], ev[j * kSlot + i + 1]);
        sum[i] += t;
      }
    cudaEventElapsedTime(&total, ev[0], ev[(passes - 1) * kSlot + nk]);
  } else if (rc == UOCR_OK) {
    rc = fail(UOCR_ERR_CUDA, "profile_stack: synchronise");
  }
  for (auto& e : ev) cudaEventDestroy(e);
  if (rc != UOCR_OK) return rc;
  for (int i = 0; i < 8; ++i) ms[i] = 0.0f;
  for (int i = 0; i < nk; ++i) ms[i] = static_cast<float>(sum[i] / static_cast<double>(passes));
  ms[6] = static_cast<float>(nk);
  ms[7] = total / static_cast<float>(iters);
  return UOCR_OK;
}

int uocr_moe_check(uocr_moe_plan* p, void* stream_v) {
  if (p == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "check: null plan");
  DeviceGuard guard(p->d.device);
  UOCR_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream_v)), "check: stream");
  ErrorWord e{};
  UOCR_TRY(cudaMemcpy(&e, p->err, sizeof(e), cudaMemcpyDeviceToHost), "check: error word");
  if (e.code == kDevOk) return UOCR_OK;
  UOCR_TRY(cudaMemset(p->err, 0, sizeof(ErrorWord)), "check: clear");
  char buf[160];
  std::snprintf(buf, sizeof(buf), "device error %d at site %d (%d, %d)", e.code, e.where, e.a, e.b);
  return fail(e.code == kDevWaitTimeout ? UOCR_ERR_TIMEOUT : UOCR_ERR_DEVICE, buf);
}

// ---- expert parallelism ----------------------------------------------------

namespace {

constexpr uint32_t kEpMagic = 0x31504555u;  // "UEP1"

// What a rank's handle carries besides its IPC handle: enough to refuse
// plans that do not fit together.
struct EpFingerprint {
  uint32_t magic;
  int32_t world, rank, strided;
  unsigned char uuid[16];
  int64_t hidden, experts, top_k, ffn, shared_ffn, max_rows, layers;
  uint64_t region_bytes;
  uint64_t map_hash;  // the expert placement: every rank must use the same
};
static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(EpFingerprint) <= sizeof(uocr_ep_handle), "handle size");

EpFingerprint fingerprint(const uocr_moe_plan* p) {
  EpFingerprint f{};
  f.magic = kEpMagic;
  f.world = p->emap.world;
  f.rank = p->emap.rank;
  f.strided = (p->d.flags & UOCR_PLAN_EP_STRIDED) != 0 ? 1 : 0;
  f.map_hash = p->etab.hash;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, p->d.device) == cudaSuccess) std::memcpy(f.uuid, &prop.uuid, 16);
  f.hidden = p->d.hidden;
  f.experts = p->d.routed_experts;
  f.top_k = p->d.experts_per_token;
  f.ffn = p->d.expert_ffn;
  f.shared_ffn = p->d.shared_ffn;
  f.max_rows = p->d.max_rows;
  f.layers = p->d.layers;
  f.region_bytes = p->elay.bytes;
  return f;
}

bool same_shape(const EpFingerprint& a, const EpFingerprint& b) {
  return a.magic == b.magic && a.world == b.world && a.strided == b.strided && a.hidden == b.hidden &&
         a.experts == b.experts && a.top_k == b.top_k && a.ffn == b.ffn && a.shared_ffn == b.shared_ffn &&
         a.max_rows == b.max_rows && a.layers == b.layers && a.region_bytes == b.region_bytes &&
         a.map_hash == b.map_hash;
}

}  // namespace

int uocr_moe_ep_handle(uocr_moe_plan* p, uocr_ep_handle* out) {
  if (p == nullptr || out == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_handle: null argument");
  if (!p->ep) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_handle: the plan has ep_world <= 1");
  DeviceGuard guard(p->d.device);
  std::memset(out, 0, sizeof(*out));
  cudaIpcMemHandle_t h{};
  UOCR_TRY(cudaIpcGetMemHandle(&h, p->exchange), "ep_handle: cudaIpcGetMemHandle");
  const EpFingerprint f = fingerprint(p);
  std::memcpy(out->bytes, &h, sizeof(h));
  std::memcpy(out->bytes + sizeof(h), &f, sizeof(f));
  return UOCR_OK;
}

int uocr_moe_ep_connect(uocr_moe_plan* p, const uocr_ep_handle* handles) {
  if (p == nullptr || handles == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect: null argument");
  if (!p->ep) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect: the plan has ep_world <= 1");
  if (p->ep_connected) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect: already connected");
  DeviceGuard guard(p->d.device);
  const EpFingerprint mine = fingerprint(p);
  const int W = p->emap.world;
  for (int s = 0; s < W; ++s) {
    EpFingerprint f{};
    std::memcpy(&f, handles[s].bytes + sizeof(cudaIpcMemHandle_t), sizeof(f));
    if (!same_shape(f, mine) || f.rank != s)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect: handle " + std::to_string(s) +
                                                 " is not rank " + std::to_string(s) + " of a plan of the same shape");
    if (s != p->emap.rank && std::memcmp(f.uuid, mine.uuid, 16) == 0)
      return fail(UOCR_ERR_UNSUPPORTED, "ep_connect: ranks " + std::to_string(s) + " and " +
                                            std::to_string(p->emap.rank) +
                                            " share a GPU; use uocr_moe_ep_connect_local for virtual ranks");
  }
  EpPeers peers = p->epeers;
  std::vector<char*> opened;
  for (int s = 0; s < W; ++s) {
    if (s == p->emap.rank) continue;
    cudaIpcMemHandle_t h{};
    std::memcpy(&h, handles[s].bytes, sizeof(h));
    void* q = nullptr;
    const cudaError_t st = cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess);
    if (st != cudaSuccess) {
      for (char* o : opened) cudaIpcCloseMemHandle(o);
      return fail(UOCR_ERR_COMM, std::string("ep_connect: opening rank ") + std::to_string(s) +
                                     "'s memory: " + cudaGetErrorString(st));
    }
    opened.push_back(static_cast<char*>(q));
    peers.base[s] = static_cast<char*>(q);
  }
  p->opened = std::move(opened);
  p->epeers = peers;
  p->ep_connected = true;
  return UOCR_OK;
}

int uocr_moe_ep_connect_local(uocr_moe_plan* const* plans, int32_t n) {
  if (plans == nullptr || n < 2 || n > kMaxEpRanks)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect_local: need 2..8 plans");
  for (int i = 0; i < n; ++i) {
    const uocr_moe_plan* q = plans[i];
    if (q == nullptr || !q->ep || q->emap.world != n || q->emap.rank != i || q->ep_connected)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect_local: plan " + std::to_string(i) +
                                                 " is not an unconnected rank " + std::to_string(i) + " of " +
                                                 std::to_string(n));
    if (q->d.device != plans[0]->d.device || !same_shape(fingerprint(q), fingerprint(plans[0])))
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_connect_local: plans differ in device or shape");
  }
  EpPeers peers{};
  for (int i = 0; i < n; ++i) peers.base[i] = plans[i]->exchange;
  for (int i = 0; i < n; ++i) {
    plans[i]->epeers = peers;
    plans[i]->ep_connected = true;
    plans[i]->ep_local_group = true;
  }
  return UOCR_OK;
}

int uocr_moe_ep_forward_local(uocr_moe_plan* const* plans, int32_t n, int64_t layer, const float* const* x,
                              const int64_t* rows, float* const* y, void* stream_v) {
  if (plans == nullptr || x == nullptr || rows == nullptr || y == nullptr || n < 2 || n > kMaxEpRanks)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: bad argument");
  std::vector<EpCall> calls;
  for (int i = 0; i < n; ++i) {
    uocr_moe_plan* q = plans[i];
    if (q == nullptr || !q->ep_local_group || q->emap.rank != i || q->emap.world != n)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: plans are not one local group in rank order");
    if (layer < 0 || layer >= q->d.layers) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: bad layer");
    if (rows[i] < 0 || rows[i] > q->d.max_rows)
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: rows outside [0, max_rows]");
    if (rows[i] > 0 && (x[i] == nullptr || y[i] == nullptr || x[i] == y[i]))
      return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: null or overlapping x, y");
    const LayerDev& L = q->layers[static_cast<size_t>(layer)];
    if (!L.loaded) return fail(UOCR_ERR_INVALID_ARGUMENT, "ep_forward_local: layer weights not set");
    calls.push_back(ep_call(q, L, q->pre_norm && rows[i] > 0 ? q->xnorm : x[i], rows[i], nullptr, y[i]));
  }
  DeviceGuard guard(plans[0]->d.device);
  auto stream = static_cast<cudaStream_t>(stream_v);
  for (int i = 0; i < n; ++i) {
    const uocr_moe_plan* q = plans[i];
    const LayerDev& L = q->layers[static_cast<size_t>(layer)];
    if (q->pre_norm && rows[i] > 0)
      UOCR_TRY(launch_rms_norm_rows(x[i], rows[i], static_cast<int>(q->d.hidden),
                                    RowNorm{L.norm, q->d.rms_norm_eps, 1}, q->xnorm, stream),
               "ep_forward_local: pre-norm");
  }
  // Each phase for every rank before the next phase: stream order stands in
  // for the barriers.
  for (auto& c : calls) UOCR_TRY(ep_route(c, stream), "ep_forward_local: route");
  for (auto& c : calls) UOCR_TRY(ep_experts(c, stream), "ep_forward_local: experts");
  for (auto& c : calls) UOCR_TRY(ep_shared(c, stream), "ep_forward_local: shared");
  for (auto& c : calls) UOCR_TRY(ep_combine(c, stream), "ep_forward_local: combine");
  return UOCR_OK;
}

// ---- op-level mirrors ----------------------------------------------------

int uocr_ops_check(void* stream) {
  UOCR_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "ops_check: stream");
  ErrorWord* word = nullptr;
  UOCR_TRY(ops_error_word(&word), "ops_check: error word");
  ErrorWord e{};
  UOCR_TRY(cudaMemcpy(&e, word, sizeof(e), cudaMemcpyDeviceToHost), "ops_check: read");
  if (e.code == kDevOk) return UOCR_OK;
  UOCR_TRY(cudaMemset(word, 0, sizeof(ErrorWord)), "ops_check: clear");
  char buf[160];
  if (e.code == kDevBadIndex && e.where == 2)
    std::snprintf(buf, sizeof(buf), "expert_ffn_one: expert id %d at position %d is outside [0, %d)", e.b, e.a,
                  kMaxExperts);
  else
    std::snprintf(buf, sizeof(buf), "device error %d at site %d (%d, %d)", e.code, e.where, e.a, e.b);
  return fail(e.code == kDevWaitTimeout ? UOCR_ERR_TIMEOUT : UOCR_ERR_DEVICE, buf);
}

int uocr_expert_topk(const float* logits, int64_t rows, int64_t experts, int64_t k, int32_t renormalize,
                     int64_t* ids, float* weights, void* stream) {
  if (experts > kMaxExperts) return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_topk: more than 128 experts");
  if (experts <= 0 || k <= 0 || k > experts || k > kMaxTopK || rows < 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_topk: bad shape");
  if (rows > 0 && (logits == nullptr || ids == nullptr || weights == nullptr))
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_topk: null pointer");
  UOCR_TRY(launch_topk_rows(logits, rows, static_cast<int>(experts), static_cast<int>(k), renormalize, ids, weights,
                            static_cast<cudaStream_t>(stream)),
           "expert_topk");
  return UOCR_OK;
}


int uocr_expert_ffn_one(const float* x, int64_t hidden, int64_t ffn, const uint16_t* gate, const uint16_t* up,
                        const uint16_t* down, const int64_t* ids, const float* weights, int64_t k, float* out,
                        void* stream_v) {
  if (gate == nullptr || up == nullptr || down == nullptr)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one: null weights");
  auto stream = static_cast<cudaStream_t>(stream_v);
  const int sms = device_sms();
  auto b = [](const uint16_t* v) { return reinterpret_cast<const __nv_bfloat16*>(v); };
  // Expert ids are not bounded by a plan here; the stacks' extent is the
  // caller's contract, as in the reference (ops.h:82-89).
  return ffn_one(x, hidden, ffn, ids, weights, k, out, kMaxExperts, stream,
                 [&](DecodeRoute* route, __nv_bfloat16* act, ErrorWord* err) {
                   const DecodeRouting routing{nullptr, route, kMaxExperts, static_cast<int>(k), 0, nullptr,
                                               nullptr};
                   return launch_decode_experts_bf16(x, 1, static_cast<int>(hidden), static_cast<int>(ffn), 0,
                                                     b(gate), b(up), b(down), nullptr, nullptr, nullptr, routing, act,
                                                     nullptr, nullptr, out, err, sms, stream);
                 });
}

int uocr_expert_ffn_one_q8(const float* x, int64_t hidden, int64_t ffn, const int8_t* gate_q, const float* gate_s,
                           const int8_t* up_q, const float* up_s, const int8_t* down_q, const float* down_s,
                           const int64_t* ids, const float* weights, int64_t k, float* out, void* stream_v) {
  if (gate_q == nullptr || up_q == nullptr || down_q == nullptr || gate_s == nullptr || up_s == nullptr ||
      down_s == nullptr)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "expert_ffn_one_q8: null weights");
  auto stream = static_cast<cudaStream_t>(stream_v);
  const int sms = device_sms();
  const int H = static_cast<int>(hidden), F = static_cast<int>(ffn);
  return ffn_one(x, hidden, ffn, ids, weights, k, out, kMaxExperts, stream,
                 [&](DecodeRoute* route, __nv_bfloat16* act, ErrorWord* err) {
                   const Q8Rows none{nullptr, nullptr, 0};
                   const DecodeRouting routing{nullptr, route, kMaxExperts, static_cast<int>(k), 0, nullptr,
                                               nullptr};
                   return launch_decode_experts_q8(x, 1, H, F, 0, Q8Rows{gate_q, gate_s, H}, Q8Rows{up_q, up_s, H},
                                                   Q8Rows{down_q, down_s, F}, none, none, none, routing, act,
                                                   nullptr, nullptr, out, err, sms, stream);
                 });
}

int uocr_linear(const float* x, int64_t m, int64_t k, const uint16_t* w_bf16, int64_t n, const float* bias, float* y,
                void* stream_v) {
  if (m < 0 || k <= 0 || n <= 0) return fail(UOCR_ERR_INVALID_ARGUMENT, "linear: bad shape");
  if (k % 64 != 0 || n % 256 != 0)
    return fail(UOCR_ERR_UNSUPPORTED, "linear: this build needs k % 64 == 0 and n % 256 == 0");
  if (m == 0) return UOCR_OK;
  if (x == nullptr || w_bf16 == nullptr || y == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "linear: null pointer");
  auto stream = static_cast<cudaStream_t>(stream_v);
  const size_t xb_bytes = align_up(static_cast<size_t>(m * k) * 2, 256);
  char* scratch = nullptr;
  UOCR_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), xb_bytes + sizeof(ErrorWord), stream),
           "linear: scratch");
  auto* xb = reinterpret_cast<__nv_bfloat16*>(scratch);
  auto* err = reinterpret_cast<ErrorWord*>(scratch + xb_bytes);
  cudaError_t st = cudaMemsetAsync(err, 0, sizeof(ErrorWord), stream);
  if (st == cudaSuccess) st = launch_f32_to_bf16(x, xb, m * k, stream);
  if (st == cudaSuccess) {
    GroupedGemm g{};
    g.mode = 1;
    g.experts = 0;
    g.k_routed = 64;
    g.n_cols_routed = 256;
    g.shared_rows = static_cast<int>(m);
    g.a_shared = xb;
    g.k_shared = static_cast<int>(k);
    g.b0_shared = reinterpret_cast<const __nv_bfloat16*>(w_bf16);
    g.b1_shared = g.b0_shared;
    g.b_shared_rows = n;
    g.n_cols_shared = static_cast<int>(n);
    g.out_shared = y;
    g.ld_out_shared = n;
    g.shared_out_f32 = true;
    g.err = err;
    g.blocks = device_sms();
    st = launch_grouped_gemm(g, stream);
  }
  if (st == cudaSuccess && bias != nullptr) st = launch_add_bias(y, bias, m, n, stream);
  cudaFreeAsync(scratch, stream);
  if (st != cudaSuccess) return cuda_fail(st, "linear");
  return UOCR_OK;
}

int uocr_quantize_q8(const void* w, int32_t dtype, int64_t rows, int64_t cols, int64_t group, int8_t* q,
                     float* scales, void* stream) {
  if (rows < 0 || cols <= 0 || group <= 0 || cols % group != 0)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "quantize_q8: the group must divide the row width");
  if (dtype != UOCR_DTYPE_F32 && dtype != UOCR_DTYPE_BF16)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "quantize_q8: dtype must be f32 or bf16");
  if (rows > 0 && (w == nullptr || q == nullptr || scales == nullptr))
    return fail(UOCR_ERR_INVALID_ARGUMENT, "quantize_q8: null pointer");
  UOCR_TRY(launch_quantize_rows(w, dtype == UOCR_DTYPE_BF16, rows, cols, group, q, scales,
                                static_cast<cudaStream_t>(stream)),
           "quantize_q8");
  return UOCR_OK;
}

uint64_t uocr_synth_stream(uint64_t layer, uint64_t kind, uint64_t index) {
  return (layer << 40) | (kind << 32) | index;
}

int uocr_synth_fill(uint64_t seed, uint64_t stream_id, float sigma, int64_t offset, int64_t n, int32_t dtype,
                    void* out, void* stream) {
  if (n < 0 || offset < 0) return fail(UOCR_ERR_INVALID_ARGUMENT, "synth_fill: negative size");
  if (dtype != UOCR_DTYPE_F32 && dtype != UOCR_DTYPE_BF16)
    return fail(UOCR_ERR_INVALID_ARGUMENT, "synth_fill: dtype must be f32 or bf16");
  if (n > 0 && out == nullptr) return fail(UOCR_ERR_INVALID_ARGUMENT, "synth_fill: null output");
  UOCR_TRY(launch_synth(seed, stream_id, sigma, offset, n, dtype == UOCR_DTYPE_BF16, out,
                        static_cast<cudaStream_t>(stream)),
           "synth_fill");
  return UOCR_OK;
}

}  // extern "C"

int uocr_b200::moe_layer_inplace(uocr_moe_plan* p, int64_t layer, float* h, int64_t rows, cudaStream_t stream) {
  if (rows == 0) return UOCR_OK;
  return run_layer(p, p->layers[static_cast<size_t>(layer)], h, rows, h, h, stream);
}
