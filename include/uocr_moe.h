/* uocr_moe.h — C ABI of the B200 (sm_100a) decoder mixture-of-experts path.
 *
 * Drop-in for the MoE part of grpc-unlimited-ocr's CUDA backend: the router
 * gate, softmax/top-k, the routed SwiGLU experts, the shared expert and the
 * combine. Every entry point takes plain pointers, sizes and a cudaStream_t
 * passed as void*, enqueues work on that stream and never synchronises it
 * (uocr_moe_check is the one exception, and says so). Status codes replace the
 * reference's exceptions (src/backend/cuda/context.cu:24-34, ops.cu:653-655);
 * the message of the last failure on the calling thread is uocr_last_error().
 *
 * Layouts follow the reference (src/backend/cuda/ops.h:3-6): activations are
 * fp32 row-major [rows, hidden]; expert matrices are stacked by expert —
 * gate/up [E*F, H], down [E*H, F] (src/model/cuda/cuda_decoder.h:42-47);
 * the shared expert is one gated MLP of width S: gate/up [S, H], down [H, S]
 * (src/weights/architecture.cpp:117). The router is fp32 [E, H]
 * (src/model/cuda/cuda_decoder.cpp:64-67).
 */
#ifndef UOCR_MOE_H
#define UOCR_MOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UOCR_MOE_ABI_VERSION 5

typedef enum uocr_status {
  UOCR_OK = 0,
  UOCR_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
  UOCR_ERR_UNSUPPORTED = 2,      /* a shape or mode this build does not implement */
  UOCR_ERR_CUDA = 3,             /* reference: std::runtime_error from check() */
  UOCR_ERR_OUT_OF_MEMORY = 4,
  UOCR_ERR_DEVICE = 5,           /* a kernel recorded an error word (bad index, capacity) */
  UOCR_ERR_TIMEOUT = 6,          /* a bounded device-side wait gave up */
  UOCR_ERR_COMM = 7              /* expert-parallel exchange failure */
} uocr_status;

/* GRPC_UOCR_WEIGHT_FORMAT (src/service/config.cpp:54-56). INT8 here is
 * symmetric per-output-channel (one fp32 scale per weight row). */
typedef enum uocr_weight_format { UOCR_WEIGHT_BF16 = 0, UOCR_WEIGHT_INT8 = 1 } uocr_weight_format;
typedef enum uocr_memory { UOCR_MEMORY_HOST = 0, UOCR_MEMORY_DEVICE = 1 } uocr_memory;
typedef enum uocr_dtype {
  UOCR_DTYPE_F32 = 0,
  UOCR_DTYPE_BF16 = 1,
  /* further dtypes a checkpoint may hold (src/tensor/dtype.cpp:15-22) */
  UOCR_DTYPE_F16 = 2,
  UOCR_DTYPE_I64 = 3,
  UOCR_DTYPE_I32 = 4,
  UOCR_DTYPE_U8 = 5
} uocr_dtype;

/* Message of the last failed call on this thread ("" when none). */
const char* uocr_last_error(void);
int uocr_abi_version(void);

/* ---- Plan: one MoE stack with its weights and a preallocated arena -------
 * Replaces the per-layer state of CudaDecoder (src/model/cuda/cuda_decoder.h:
 * 25-104: moe_gate_f32, experts, shared) and DecoderDims' MoE fields
 * (src/weights/architecture.h:26-30). All scratch is carved from an arena
 * sized at creation for max_rows, so forward never allocates. */
typedef struct uocr_moe_plan uocr_moe_plan;

typedef struct uocr_moe_desc {
  int64_t hidden;            /* H */
  int64_t routed_experts;    /* E, at most 128 (ops.cu:653) */
  int64_t experts_per_token; /* k */
  int64_t expert_ffn;        /* F */
  int64_t shared_ffn;        /* S = shared_experts * expert_ffn; 0 = no shared expert */
  int64_t layers;
  int64_t max_rows;          /* largest row count forward accepts */
  int32_t weight_format;     /* uocr_weight_format */
  int32_t renormalize;       /* 1: top-k weights divided by their sum; 0: raw softmax (feed_forward.cpp:40) */
  int32_t router_bias;       /* 1: each layer carries an fp32 [E] bias added to the logits */
  int32_t device;            /* CUDA device ordinal the plan lives on */
  int32_t flags;             /* UOCR_PLAN_* bits */
  int32_t ep_world;          /* expert parallelism: ranks (GPUs) sharing the experts; 0 or 1 = none */
  int32_t ep_rank;           /* this plan's rank in [0, ep_world) */
  float rms_norm_eps;        /* with UOCR_PLAN_PRE_NORM: the norm's epsilon (DecoderDims::rms_norm_eps) */
  int32_t reserved;          /* 0 */
  /* Expert placement under expert parallelism, or NULL: [routed_experts *
   * ep_world] int32, entry e * ep_world + s = the rank that computes the rows
   * of expert e that rank s routed. An expert may appear for several ranks (a
   * hot expert replicated, its rows split by source rank); a rank holds the
   * weights of every expert it appears for, and each rank must hold at least
   * one. Every rank passes the same table (connect checks it). NULL: the
   * contiguous ranges, or UOCR_PLAN_EP_STRIDED's e % ep_world, with
   * routed_experts a multiple of ep_world. Read at creation only. */
  const int32_t* ep_owner;
} uocr_moe_desc;

/* forward_stack replays a CUDA graph it captured on the first call for the
 * same (h, rows, stream-capturable) — one launch per step instead of three per
 * layer. This flag turns the cache off. A stream that is already capturing,
 * or the legacy default stream, always gets plain launches. */
#define UOCR_PLAN_NO_GRAPHS 1
/* (Flag bit 2 is unused.) */
/* Expert parallelism: expert e lives on rank e % ep_world instead of the
 * default contiguous ranges (rank e / (routed_experts / ep_world)). */
#define UOCR_PLAN_EP_STRIDED 4
/* Each layer's input passes the decoder's pre-feed-forward RMSNorm first
 * (src/model/decoder.cpp:180-181, 200-201; ref::rms_norm,
 * src/backend/reference/ops.cpp:129-141): forward computes
 * y = MoE(RMSNorm(x)) and forward_stack h <- h + MoE(RMSNorm(h)) — the
 * decoder's whole feed-forward block. The gain is each layer's src.norm.
 * Decode batches normalise inside the router and gate/up kernels; the
 * tensor-core decode flag is then ignored. */
#define UOCR_PLAN_PRE_NORM 8

int uocr_moe_plan_create(const uocr_moe_desc* desc, uocr_moe_plan** plan);
int uocr_moe_plan_destroy(uocr_moe_plan* plan);
/* Bytes of device memory the plan holds (weights + arena). */
int uocr_moe_plan_bytes(const uocr_moe_plan* plan, int64_t* weight_bytes, int64_t* arena_bytes);

/* One layer's weights as the reference's WeightSource hands them over (fp32,
 * src/model/weight_source.h:16-21), or bf16. They are converted on the device
 * to the plan's format: bf16, or int8 quantised per output channel
 * (scale = rowmax|w| / 127, src/model/cuda/device_weight.cpp:11-26 with one
 * group per row). Replaces stacked_weight / device_weight
 * (src/model/cuda/device_weight.cpp:57-72). Synchronises nothing, but host
 * sources are copied before the call returns. */
typedef struct uocr_moe_layer_src {
  int32_t memory;            /* uocr_memory of every pointer below */
  int32_t dtype;             /* uocr_dtype of gate/up/down/shared_* (router and bias are always fp32) */
  const float* router;       /* [E, H] */
  const float* router_bias;  /* [E], required iff desc.router_bias */
  const void* gate;          /* [E*F, H] */
  const void* up;            /* [E*F, H] */
  const void* down;          /* [E*H, F] */
  const void* shared_gate;   /* [S, H] (ignored when S == 0) */
  const void* shared_up;     /* [S, H] */
  const void* shared_down;   /* [H, S] */
  const float* norm;         /* [H] RMSNorm gain with UOCR_PLAN_PRE_NORM (NULL: all ones); ignored otherwise */
} uocr_moe_layer_src;

int uocr_moe_set_layer(uocr_moe_plan* plan, int64_t layer, const uocr_moe_layer_src* src, void* stream);

/* The same layer as a checkpoint holds it: one tensor per routed expert and
 * projection, each behind its own pointer (a view into a memory-mapped
 * safetensors shard, say), all in `dtype` — bf16 in the published checkpoint,
 * whose names are model.layers.{l}.mlp.experts.{e}.{gate,up,down}_proj.weight,
 * mlp.shared_experts.*, mlp.gate.weight (the router) and
 * post_attention_layernorm.weight (the pre-norm gain),
 * src/weights/architecture.cpp:108-117. Expert e's rows land at rows e*F
 * (gate/up) and e*H (down) of the plan's stacks; the router, bias and gain are
 * widened to fp32 exactly, as CheckpointWeights does
 * (src/model/weight_source.cpp:21), and the matrices are converted as
 * uocr_moe_set_layer converts them. Replaces CudaDecoder's stack_experts and
 * expert() (src/model/cuda/cuda_decoder.cpp:44-46, 67-69, 75-84) over
 * stacked_weight (src/model/cuda/device_weight.cpp:63-72), without first
 * stacking the experts on the host. In an expert-parallel plan only this
 * rank's experts are read (the others may be NULL). */
typedef struct uocr_moe_layer_parts {
  int32_t memory;                 /* uocr_memory of every pointer below */
  int32_t dtype;                  /* uocr_dtype of every tensor below */
  const void* router;             /* [E, H] */
  const void* router_bias;        /* [E], required iff desc.router_bias */
  const void* const* gate;        /* E pointers, each [F, H] */
  const void* const* up;          /* E pointers, each [F, H] */
  const void* const* down;        /* E pointers, each [H, F] */
  const void* shared_gate;        /* [S, H] (ignored when S == 0) */
  const void* shared_up;          /* [S, H] */
  const void* shared_down;        /* [H, S] */
  const void* norm;               /* [H] gain with UOCR_PLAN_PRE_NORM (NULL: all ones); ignored otherwise */
} uocr_moe_layer_parts;

int uocr_moe_set_layer_parts(uocr_moe_plan* plan, int64_t layer, const uocr_moe_layer_parts* parts, void* stream);

/* ---- Checkpoints: safetensors shards, memory-mapped read-only ------------
 * uocr_checkpoint_open takes a shard index (model.safetensors.index.json) or
 * one .safetensors file and checks what the reference's readers check:
 * SafetensorsFile (src/weights/safetensors.cpp:69-163: header length, JSON
 * object, dtype, dims, offsets, sizes, extents tiling the data section
 * exactly) and ShardedWeights::open (src/weights/sharded_weights.cpp:12-61:
 * plain shard file names, every indexed tensor in the shard the index names,
 * no unlisted tensor). Failures return UOCR_ERR_INVALID_ARGUMENT with the
 * file and the first problem in uocr_last_error(). Host only: no GPU needed. */
typedef struct uocr_checkpoint uocr_checkpoint;

#define UOCR_MAX_TENSOR_RANK 8
typedef struct uocr_tensor_view {
  int32_t dtype;                         /* uocr_dtype */
  int32_t rank;
  int64_t shape[UOCR_MAX_TENSOR_RANK];
  const void* data;                      /* into the mapping; valid until uocr_checkpoint_close */
  int64_t bytes;
} uocr_tensor_view;

int uocr_checkpoint_open(const char* path, uocr_checkpoint** out);
int uocr_checkpoint_close(uocr_checkpoint* ckpt);
int uocr_checkpoint_count(const uocr_checkpoint* ckpt, int64_t* tensors);
/* UOCR_ERR_INVALID_ARGUMENT ("no tensor named ...") when absent. */
int uocr_checkpoint_tensor(const uocr_checkpoint* ckpt, const char* name, uocr_tensor_view* out);

/* Checkpoint layer `layer`'s MoE tensors (the names above; all BF16 or all
 * F32) into plan layer `plan_layer` through uocr_moe_set_layer_parts. A
 * missing tensor, a shape other than the plan's or mixed dtypes fail with
 * UOCR_ERR_INVALID_ARGUMENT naming the tensor, before anything is copied. */
int uocr_moe_load_layer(uocr_moe_plan* plan, const uocr_checkpoint* ckpt, int64_t layer, int64_t plan_layer,
                        void* stream);

/* y [rows, H] = MoE_layer(x [rows, H]) — the work of CudaDecoder::moe
 * (src/model/cuda/cuda_decoder.cpp:137-192) and MixtureOfExperts::forward
 * (src/model/feed_forward.cpp:36-78): fp32 router, softmax, top-k (lower id on
 * a tie), optional renormalisation, routed SwiGLU experts on bf16-rounded
 * inputs, shared expert, and the combine in expert-id order. Rows <= 16 stream
 * the selected experts' weights (bf16 or int8); more rows run the tensor-core
 * grouped GEMMs (hidden % 256, expert_ffn and shared_ffn % 128 == 0), with an
 * int8 layer first expanded to bf16(q * scale) as the reference's linear_q8
 * does for m > 1 (src/backend/cuda/gemv_ops.cu:214-218). ids [rows, k]
 * (int32, rank order) and weights [rows, k] are optional outputs (NULL to
 * skip). x, y, ids and weights are device pointers; x and y must not overlap;
 * x is 16-byte aligned (as every cudaMalloc block is). */
int uocr_moe_forward(uocr_moe_plan* plan, int64_t layer, const float* x, int64_t rows, float* y, int32_t* ids,
                     float* weights, void* stream);

/* logits [rows, E] = the layer's router gate on x [rows, H] (+ its bias; the
 * plan's pre-norm first when it has one): the gemm_nt of CudaDecoder::moe
 * (src/model/cuda/cuda_decoder.cpp:139-140) and ref::linear of
 * MixtureOfExperts::forward (src/model/feed_forward.cpp:38), in the CPU
 * reference's dot order (src/backend/reference/ops.cpp:25-38, :91-109), with
 * the kernel forward uses at that row count. Device pointers; x is 16-byte
 * aligned. */
int uocr_moe_router_logits(uocr_moe_plan* plan, int64_t layer, const float* x, int64_t rows, float* logits,
                           void* stream);

/* h <- h + MoE_l(h) for l = 0 .. layers-1, in place on device memory h
 * [rows, H]: the decoder's residual around its feed-forward block
 * (src/model/decoder.cpp:181,201) with nothing between the layers. h is
 * 16-byte aligned. */
int uocr_moe_forward_stack(uocr_moe_plan* plan, float* h, int64_t rows, void* stream);

/* Synchronises `stream`, then reports and clears any error word a kernel of
 * this plan recorded (bounded waits that gave up, bad indices). */
int uocr_moe_check(uocr_moe_plan* plan, void* stream);

/* Instrumented forward_stack for measurement: runs `iters` stack passes with
 * CUDA events between the kernels, synchronises, and writes ms_per_kernel[8]:
 * [0..5] the mean device time per launch of each kernel in launch order —
 * decode rows (<= 16): router, gate/up, down+combine; prefill rows: router,
 * top-k, permutation, gate/up GEMM, down GEMM, combine — [6] how many of those
 * entries are used, [7] the mean time of one whole stack pass (events between
 * kernels: no overlap between them). No reference counterpart. */
int uocr_moe_profile_stack(uocr_moe_plan* plan, float* h, int64_t rows, int32_t iters, float* ms_per_kernel,
                           void* stream);

/* ---- Expert parallelism across the GPUs of one node ----------------------
 * No reference counterpart (the reference has no multi-GPU path). A plan with
 * ep_world = G > 1 is one rank of G processes, one per GPU: it holds its
 * share of the experts (routed_experts / G of them, or the ones desc.ep_owner
 * assigns it; set_layer still takes the full stacks and keeps its own) and
 * forwards its own rows. Every forward call on
 * such a plan is collective: all G ranks make the same calls in the same
 * order, any row count including 0. Layers run the prefill path (bf16,
 * hidden % 256 == 0, expert_ffn and shared_ffn % 128 == 0) whatever the row
 * count. Between the phases the ranks pull rows and expert outputs from each
 * other's memory over NVLink (CUDA IPC mappings) and meet at device-side
 * barriers; a rank that does not arrive within 20 s (UOCR_EP_WAIT_MS in the
 * environment at plan creation overrides it) makes uocr_moe_check report
 * UOCR_ERR_TIMEOUT, after which the ranks' plans must be recreated.
 * The result equals, bit for bit, a single-GPU plan's on the same rows.
 *
 * Setup: each rank gets its handle, the ranks exchange them (any transport:
 * torch.distributed all_gather, a file, a socket), each calls
 * uocr_moe_ep_connect with all G handles in rank order, and the ranks meet
 * (a host barrier) before the first forward. Destroy after a host barrier,
 * when no rank is inside a forward. */
typedef struct uocr_ep_handle {
  unsigned char bytes[256]; /* IPC handle of the rank's exchange memory + a fingerprint of its plan */
} uocr_ep_handle;
int uocr_moe_ep_handle(uocr_moe_plan* plan, uocr_ep_handle* out);
/* handles[ep_world] in rank order (this rank's own included). Fails with
 * UOCR_ERR_INVALID_ARGUMENT when the plans differ in shape or rank, and
 * UOCR_ERR_UNSUPPORTED when two ranks share a GPU (device-side waits between
 * processes on one GPU are not allowed: use the local group below). */
int uocr_moe_ep_connect(uocr_moe_plan* plan, const uocr_ep_handle* handles);
/* Test harness for one GPU: n plans on the same device, created with
 * ep_world = n and ep_rank = 0..n-1, become one group of virtual ranks.
 * Such plans run only through uocr_moe_ep_forward_local, which runs each
 * phase for every rank in turn on one stream (no barriers are needed). */
int uocr_moe_ep_connect_local(uocr_moe_plan* const* plans, int32_t n);
int uocr_moe_ep_forward_local(uocr_moe_plan* const* plans, int32_t n, int64_t layer, const float* const* x,
                              const int64_t* rows, float* const* y, void* stream);

/* ---- Op-level mirrors of the reference's uocr::cuda MoE ops -------------- */

/* Device errors of the op-level mirrors. The reference's kernels index the
 * stacks with whatever id they are given (gemv_ops.cu:145-169) and surface
 * only CUDA statuses through check() (src/backend/cuda/context.cu:24-34).
 * Here uocr_expert_ffn_one, _q8 and _noalloc record an expert id outside
 * [0, 128) in a per-device error word (that slot then reads expert 0 with
 * weight 0, so no memory outside the stacks is touched) and still return
 * UOCR_OK, as they only enqueue work. The word is sticky: the first such
 * error stays recorded until this call, which synchronises the stream, reads
 * the current device's word, clears it, and returns UOCR_ERR_DEVICE with the
 * offending id and position in uocr_last_error() (UOCR_OK when clean). */
int uocr_ops_check(void* stream);

/* src/backend/cuda/ops.h:80-81 expert_topk: softmax over each row of
 * logits [rows, experts <= 128], then the top k (lower index on a tie) as
 * int64 ids and their scores; renormalize = 1 divides the k scores by their
 * sum (the reference never does). Device pointers. */
int uocr_expert_topk(const float* logits, int64_t rows, int64_t experts, int64_t k, int32_t renormalize,
                     int64_t* ids, float* weights, void* stream);

/* src/backend/cuda/ops.h:87-89 expert_ffn_one: one decode row through its
 * k routed experts, bf16 stacks gate/up [E*F, H], down [E*H, F]:
 *   out[c] = sum_j weights[j] * down[ids[j]] (silu(gate[ids[j]] x) * up[ids[j]] x)
 * with x and the hidden activation rounded to bf16. Like the reference it
 * takes its [k, F] activation scratch from cudaMallocAsync on the stream. */
int uocr_expert_ffn_one(const float* x, int64_t hidden, int64_t ffn, const uint16_t* gate, const uint16_t* up,
                        const uint16_t* down, const int64_t* ids, const float* weights, int64_t k, float* out,
                        void* stream);

/* uocr_expert_ffn_one without any device allocation. No counterpart in the
 * reference. For callers that cannot allocate device memory on the call path:
 * a serving loop whose memory another allocator reserved up front, a decode
 * step that must not pay cudaMalloc's synchronisation or a pool's bookkeeping,
 * a runtime that forbids allocations after start-up. Same arguments and
 * result as uocr_expert_ffn_one; its scratch is one static device array of
 * about 146 KiB that every GPU loading this library holds until exit, so
 * k <= 8 and ffn <= 8192 (larger is UOCR_ERR_INVALID_ARGUMENT). The first call
 * on a device looks the array's address up; make it before any stream
 * capture. All calls share the array: calls that overlap on the GPU race. */
int uocr_expert_ffn_one_noalloc(const float* x, int64_t hidden, int64_t ffn, const uint16_t* gate,
                                const uint16_t* up, const uint16_t* down, const int64_t* ids, const float* weights,
                                int64_t k, float* out, void* stream);

/* src/backend/cuda/gemv_ops.h:33-35 expert_ffn_one_q8 with per-output-channel
 * int8 stacks: q [rows, cols] int8 and one fp32 scale per row. */
int uocr_expert_ffn_one_q8(const float* x, int64_t hidden, int64_t ffn, const int8_t* gate_q, const float* gate_s,
                           const int8_t* up_q, const float* up_s, const int8_t* down_q, const float* down_s,
                           const int64_t* ids, const float* weights, int64_t k, float* out, void* stream);

/* src/backend/cuda/ops.h:14-17 linear: y[m, n] = x[m, k] w[n, k]^T (+ bias[n]),
 * x rounded to bf16 for the product, fp32 accumulation — on the tcgen05
 * tensor cores (the reference calls cublasGemmEx). Like the reference it takes
 * its bf16 copy of x from cudaMallocAsync on the stream. This build needs
 * k % 64 == 0 and n % 256 == 0 (UOCR_ERR_UNSUPPORTED otherwise). */
int uocr_linear(const float* x, int64_t m, int64_t k, const uint16_t* w_bf16, int64_t n, const float* bias, float* y,
                void* stream);

/* src/model/cuda/device_weight.cpp:11-26 quantize_q8_rows on the device, with
 * the group free (group = cols is per output channel). w is fp32 or bf16
 * (dtype); q [rows, cols], scales [rows, cols/group]. Device pointers. */
int uocr_quantize_q8(const void* w, int32_t dtype, int64_t rows, int64_t cols, int64_t group, int8_t* q,
                     float* scales, void* stream);

/* Synthetic inputs (not part of the hot path): fills out[0..n) with the
 * counter-based N(0, sigma^2)-shaped stream `stream_id` of `seed`, starting
 * at element `offset`, as fp32 or as bf16 (round to nearest even). The same
 * values come out of the host generator the tests use. */
int uocr_synth_fill(uint64_t seed, uint64_t stream_id, float sigma, int64_t offset, int64_t n, int32_t dtype,
                    void* out, void* stream);
uint64_t uocr_synth_stream(uint64_t layer, uint64_t kind, uint64_t index);

#ifdef __cplusplus
}
#endif
#endif /* UOCR_MOE_H */
