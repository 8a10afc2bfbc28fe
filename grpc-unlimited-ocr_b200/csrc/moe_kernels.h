// Kernel launchers of the MoE path (host-callable, stream-ordered, no
// allocation, no synchronisation). Each returns the launch status.
#pragma once

#include <string>

#include "moe_common.cuh"

namespace uocr_b200 {

// Records `what` as uocr_last_error() for this thread and returns `code`.
int set_last_error(int code, const std::string& what);

// One-time per-device set-up (shared-memory opt-in) so that later launches,
// including those inside a stream capture, only launch.
cudaError_t prepare_router_decode();
cudaError_t prepare_decode_experts(int max_rows, int hidden);

// cudaLaunchKernelExC, optionally with programmatic stream serialisation
// (the kernel may start before the previous grid in the stream finishes and
// must call griddepcontrol.wait before reading that grid's output).
cudaError_t launch_maybe_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args,
                             bool pdl);

// ---- router (router.cu) ----
// logits [T, E] = x [T, H] . router [E, H]^T (+ bias), the reference's fp32 dot order.
// Optional routing output of the decode router: the last block builds the
// batch's routing table (and the rank-order ids / weights) once.
struct RouteOut {
  DecodeRoute* table;
  int top_k, renorm;
  int* ids_out;
  float* w_out;
  unsigned* ticket;  // zero between launches; the last block resets it
  ErrorWord* err;    // bounded waits that gave up (null: not reported)
};
// With norm.on the router normalises the x rows it stages (rms_norm.cuh).
cudaError_t launch_router_logits(const float* x, int T, int H, const float* router, const float* bias, int E,
                                 float* logits, cudaStream_t stream, bool pdl = false,
                                 const RouteOut* route = nullptr, RowNorm norm = RowNorm{nullptr, 0.0f, 0});
// Shared memory the decode routers take next to the x rows (plan sizing).
size_t router_decode_smem(int T, int H, int E, bool norm);
cudaError_t launch_topk_rows(const float* logits, int64_t rows, int E, int K, int renorm, int64_t* ids,
                             float* weights, cudaStream_t stream);
cudaError_t launch_route_from_ids(const int64_t* ids, const float* weights, int K, int E, DecodeRoute* route,
                                  ErrorWord* err, cudaStream_t stream);
// Device address of the current device's op-level error word (looked up once
// per device): the expert_ffn_one mirrors record bad ids there, and
// uocr_ops_check reads and clears it.
cudaError_t ops_error_word(ErrorWord** out);

// ---- decode experts (decode.cu) ----
// Where the decode expert kernels take their routing from: the router's
// logits (each block runs softmax/top-k itself), or, when logits is null, a
// prepared table. ids_out / weights_out (optional) receive the rank-order
// selection [T, k].
struct DecodeRouting {
  const float* logits;
  const DecodeRoute* table;
  int experts;
  int top_k;
  int renormalize;
  int* ids_out;
  float* weights_out;
};

// Launches gate/up then down+combine; `between` (optional) is recorded
// between the two, for per-kernel timing. With norm.on the gate/up kernel
// normalises the x rows it stages (the residual stays the raw rows).
cudaError_t launch_decode_experts_bf16(const float* x, int T, int H, int F, int S, const __nv_bfloat16* gate,
                                       const __nv_bfloat16* up, const __nv_bfloat16* down,
                                       const __nv_bfloat16* sgate, const __nv_bfloat16* sup,
                                       const __nv_bfloat16* sdown, const DecodeRouting& routing,
                                       __nv_bfloat16* act, __nv_bfloat16* act_s, const float* resid, float* y,
                                       ErrorWord* err, int sm_count, cudaStream_t stream,
                                       cudaEvent_t between = nullptr, bool pdl = false,
                                       RowNorm norm = RowNorm{nullptr, 0.0f, 0});
cudaError_t launch_decode_experts_q8(const float* x, int T, int H, int F, int S, Q8Rows gate, Q8Rows up,
                                     Q8Rows down, Q8Rows sgate, Q8Rows sup, Q8Rows sdown,
                                     const DecodeRouting& routing, __nv_bfloat16* act, __nv_bfloat16* act_s,
                                     const float* resid, float* y, ErrorWord* err, int sm_count, cudaStream_t stream,
                                     cudaEvent_t between = nullptr, bool pdl = false,
                                     RowNorm norm = RowNorm{nullptr, 0.0f, 0});

// ---- weights and synthetic inputs (weights.cu) ----
cudaError_t launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t stream);
cudaError_t launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n, cudaStream_t stream);
// y[r, c] += bias[c]
cudaError_t launch_add_bias(float* y, const float* bias, int64_t rows, int64_t cols, cudaStream_t stream);
cudaError_t launch_quantize_rows(const void* w, bool bf16, int64_t rows, int64_t cols, int64_t group, int8_t* q,
                                 float* scales, cudaStream_t stream);
cudaError_t launch_synth(uint64_t seed, uint64_t stream_id, float sigma, int64_t offset, int64_t n, bool bf16,
                         void* out, cudaStream_t stream);
cudaError_t launch_fill_f32(float* dst, float value, int64_t n, cudaStream_t stream);
// out [rows, cols] = bf16(float(q) * scale[row]) — the reference's expansion of
// int8 weights before a bf16 GEMM (src/backend/cuda/gemv_ops.cu:185-190, 214-218),
// here with one scale per row. cols % 16 == 0.
cudaError_t launch_dequant_rows(const int8_t* q, const float* scale, int64_t rows, int64_t cols, __nv_bfloat16* out,
                                cudaStream_t stream);
// out [rows, H] = RMSNorm(x) with norm.gain / norm.eps (one warp per row).
cudaError_t launch_rms_norm_rows(const float* x, int64_t rows, int H, RowNorm norm, float* out, cudaStream_t stream);

}  // namespace uocr_b200
