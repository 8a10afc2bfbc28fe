// Grouped GEMM on the 5th-generation tensor cores, for the prefill experts.
//
// One persistent block per SM, warp-specialised:
//   warp 0  (one lane) TMA producer: A tile [128 rows x 64 K] and B tile
//           [256 rows x 64 K] per stage, bf16, 128-byte swizzle, 4 stages;
//   warp 1  allocates 512 TMEM columns; one lane issues tcgen05.mma
//           (M=128, N=256, K=16, fp32 accumulate) into one of two 256-column
//           accumulators, and commits stage releases and "tile done";
//   warps 2-5 epilogue: tcgen05.ld the accumulator (thread = tile row), fuse
//           SwiGLU (gate columns 0-127, up columns 128-255) or convert, and
//           store through a per-warp staging area as whole row segments.
// Groups are the routed experts (rows = the expert's segment of the permuted
// activations) plus, optionally, the shared expert over all rows. Tiles are
// (group, 128-row block, 256-column block), dealt to blocks round-robin.
//
// Reference counterpart: the per-expert cuBLAS GEMMs of the prefill MoE
// (src/model/cuda/cuda_decoder.cpp:127-135,176-190 via linear, ops.cu:268-287)
// and the shared expert's linear calls.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "moe_kernels.h"
#include "tc.cuh"
#include "tc_gemm.h"

namespace uocr_b200 {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStageTileBytes = 32 * 128;  // an epilogue warp's staging area: 32 rows x 128 bytes
constexpr int kTmemCols = 512;          // two 256-column fp32 accumulators
constexpr int kThreads = 192;
constexpr int kMaxGroups = kMaxExperts + 1;

struct KernelArgs {
  CUtensorMap a_routed, a_shared, b0_routed, b1_routed, b0_shared, b1_shared;
  const int* seg_count;
  const int* seg_start;
  int experts, shared_rows;
  int n_tiles_routed, n_tiles_shared;
  int k_blocks_routed, k_blocks_shared;
  int b_rows_per_expert, b1_offset, b_tile_rows;
  int mode;  // 0: SwiGLU to bf16 (128 columns per tile); 1: store (256 columns per tile)
  void* out_routed;
  int64_t ld_out_routed;
  void* out_shared;
  int64_t ld_out_shared;
  int shared_out_f32;
  int shared_accumulate;  // with shared_out_f32: out += A.B^T
  ErrorWord* err;
  RowScatter scatter;
};

struct __align__(8) Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
};

struct Tile {
  int g, m, n;
};

__device__ __forceinline__ Tile decode_tile(int t, const int* start, int groups, const KernelArgs& a) {
  int lo = 0, hi = groups - 1;  // last g with start[g] <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int nt = lo < a.experts ? a.n_tiles_routed : a.n_tiles_shared;
  const int local = t - start[lo];
  return Tile{lo, local / nt, local % nt};
}

__global__ void __launch_bounds__(kThreads, 1) tc_grouped_gemm_kernel(const __grid_constant__ KernelArgs args) {
  extern __shared__ unsigned char dyn_raw[];
  __shared__ Barriers bars;
  __shared__ int tile_start[kMaxGroups + 1];
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;
  // 1024-byte aligned stage buffers (the 128-byte swizzle pattern repeats every 1024 bytes).
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = args.experts + (args.shared_rows > 0 ? 1 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.tmem_full[i], 1);
      mbar_init(&bars.tmem_empty[i], 4 * 32);
    }
    mbar_init(&bars.drain, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    // Tile prefix over groups: rows -> 128-row blocks -> tiles.
    int carry = 0;
    for (int g0 = 0; g0 < groups; g0 += 32) {
      const int g = g0 + lane;
      int tiles = 0;
      if (g < groups) {
        const int rows = g < args.experts ? __ldcg(args.seg_count + g) : args.shared_rows;
        const int nt = g < args.experts ? args.n_tiles_routed : args.n_tiles_shared;
        tiles = ((rows + kBM - 1) / kBM) * nt;
      }
      int incl = tiles;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      if (g < groups) tile_start[g] = carry + incl - tiles;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) tile_start[groups] = carry;
  }
  if (warp == 1) tmem_alloc(&tmem_holder, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;
  const int total_tiles = tile_start[groups];

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      prefetch_tmap(&args.a_routed);
      prefetch_tmap(&args.b0_routed);
      prefetch_tmap(&args.b1_routed);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const Tile tl = decode_tile(t, tile_start, groups, args);
        const bool routed = tl.g < args.experts;
        const CUtensorMap* amap = routed ? &args.a_routed : &args.a_shared;
        const CUtensorMap* b0map = routed ? &args.b0_routed : &args.b0_shared;
        const CUtensorMap* b1map = routed ? &args.b1_routed : &args.b1_shared;
        const int a_row = (routed ? __ldcg(args.seg_start + tl.g) : 0) + tl.m * kBM;
        const int b_row = (routed ? tl.g * args.b_rows_per_expert : 0) + tl.n * args.b_tile_rows;
        const int kb_count = routed ? args.k_blocks_routed : args.k_blocks_shared;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars.empty[stage], phase ^ 1)) {
            raise_error(args.err, kDevWaitTimeout, 40, t, kb);
            abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars.full[stage], kStageBytes);
          unsigned char* sa = smem + stage * kStageBytes;
          tma_load_2d(sa, amap, kb * kBK, a_row, &bars.full[stage]);
          tma_load_2d(sa + kABytes, b0map, kb * kBK, b_row, &bars.full[stage]);
          tma_load_2d(sa + kABytes + kBBytes / 2, b1map, kb * kBK, b_row + args.b1_offset, &bars.full[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = bf16_idesc(kBM, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
        const Tile tl = decode_tile(t, tile_start, groups, args);
        const int kb_count = tl.g < args.experts ? args.k_blocks_routed : args.k_blocks_shared;
        const int acc = local & 1;
        if (!mbar_wait(&bars.tmem_empty[acc], ((local >> 1) & 1) ^ 1)) {
          raise_error(args.err, kDevWaitTimeout, 41, t, 0);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars.full[stage], phase)) {
            raise_error(args.err, kDevWaitTimeout, 42, t, kb);
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + stage * kStageBytes);
          const uint64_t adesc = sw128_kmajor_desc(sa);
          const uint64_t bdesc = sw128_kmajor_desc(sa + kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // +32 bytes along K per instruction: +2 in the address field
            umma_bf16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&bars.empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&bars.tmem_full[acc]);
      }
      // Every MMA this thread issued must be complete before TMEM is freed.
      umma_commit(&bars.drain);
      if (!mbar_wait(&bars.drain, 0)) raise_error(args.err, kDevWaitTimeout, 43, 0, 0);
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quarter = warp % 4 ----
    // A thread holds one row's 32 columns after each tcgen05.ld; 64 bf16 or
    // 32 fp32 columns pass through a 4 KB swizzled staging area of the warp so
    // that the stores leave as whole 128-byte row lines, four rows per
    // instruction, instead of 32 rows x 16 bytes.
    const int quarter = warp & 3;
    unsigned char* stg = smem + kStages * kStageBytes + (warp - 2) * kStageTileBytes;
    // 64 columns of this lane's row as bf16 (two tcgen05.ld chunks, v0 then
    // v1) into its 128-byte row of the staging area, then out as whole
    // 128-byte lines: lane j of pass i takes 16 bytes of row (32 i + j) / 8,
    // stored at rowp[i] (that row's first column; null: the row does not
    // exist) + col.
    auto put_bf16x64 = [&](const float (&v0)[32], const float (&v1)[32], __nv_bfloat16* const (&rowp)[8], int col) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint4 pk;
        uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = k < 4 ? v0[(k & 3) * 8 + 2 * i] : v1[(k & 3) * 8 + 2 * i];
          const float b = k < 4 ? v0[(k & 3) * 8 + 2 * i + 1] : v1[(k & 3) * 8 + 2 * i + 1];
          const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
          w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(stg + lane * 128 + ((k ^ (lane & 7)) << 4)) = pk;
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = it * 32 + lane, rr = idx >> 3, k = idx & 7;
        const uint4 val = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((k ^ (rr & 7)) << 4));
        if (rowp[it] != nullptr) *reinterpret_cast<uint4*>(rowp[it] + col + k * 8) = val;
      }
      __syncwarp();
    };
    // The rows of the passes for a plain output: row0 + (32 i + lane) / 8.
    auto plain_rows = [&](__nv_bfloat16* out, int64_t ld, int64_t row0, int nvalid, __nv_bfloat16* (&rowp)[8]) {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = (it * 32 + lane) >> 3;
        rowp[it] = rr < nvalid ? out + (row0 + rr) * ld : nullptr;
      }
    };
    // The same for fp32 (128 bytes a row); acc: out += v.
    auto put_f32 = [&](const float (&v)[32], float* out, int64_t ld, int64_t row0, int nvalid, bool acc) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<float4*>(stg + lane * 128 + ((k ^ (lane & 7)) << 4)) =
            make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = it * 32 + lane, rr = idx >> 3, k = idx & 7;
        const float4 val = *reinterpret_cast<const float4*>(stg + rr * 128 + ((k ^ (rr & 7)) << 4));
        if (rr < nvalid) {
          float4* d = reinterpret_cast<float4*>(out + (row0 + rr) * ld + k * 4);
          if (acc) {
            const float4 o = *d;
            *d = make_float4(o.x + val.x, o.y + val.y, o.z + val.z, o.w + val.w);
          } else {
            *d = val;
          }
        }
      }
      __syncwarp();
    };
    int local = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
      const Tile tl = decode_tile(t, tile_start, groups, args);
      const bool routed = tl.g < args.experts;
      const int acc = local & 1;
      if (!mbar_wait(&bars.tmem_full[acc], (local >> 1) & 1)) {
        raise_error(args.err, kDevWaitTimeout, 44, t, 0);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int rows = routed ? __ldcg(args.seg_count + tl.g) : args.shared_rows;
      // This warp's 32 rows: the first is row0 of the output, nvalid of them exist.
      const int r0 = tl.m * kBM + quarter * 32;
      const int nvalid = rows - r0 < 0 ? 0 : (rows - r0 > 32 ? 32 : rows - r0);
      const int64_t row0 = (routed ? __ldcg(args.seg_start + tl.g) : 0) + static_cast<int64_t>(r0);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
      if (args.mode == 0) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(routed ? args.out_routed : args.out_shared);
        const int64_t ld = routed ? args.ld_out_routed : args.ld_out_shared;
        __nv_bfloat16* rowp[8];
        plain_rows(out + tl.n * (kBN / 2), ld, row0, nvalid, rowp);
#pragma unroll 1
        for (int c = 0; c < kBN / 2; c += 64) {
          float g0[32], g1[32], u[32];
          tmem_ld32(taddr + c, g0);
          tmem_ld32(taddr + kBN / 2 + c, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) g0[i] = swiglu(g0[i], u[i]);
          tmem_ld32(taddr + c + 32, g1);
          tmem_ld32(taddr + kBN / 2 + c + 32, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) g1[i] = swiglu(g1[i], u[i]);
          put_bf16x64(g0, g1, rowp, c);
        }
      } else if (routed && args.scatter.world > 0) {
        // This lane's four rows of the passes: their segment and destination.
        const int W = args.scatter.world;
        const int my_dst = lane < W ? __ldcg(args.scatter.seg_dst + tl.g * W + lane) : 0;
        const int my_src = lane < W ? __ldcg(args.scatter.seg_src + tl.g * W + lane) : 0;
        __nv_bfloat16* rowp[8];
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int rr = (it * 32 + lane) >> 3;
          const int64_t R = row0 + rr;
          int s_sel = 0, d_sel = 0, src_sel = 0;
          for (int s2 = 0; s2 < W; ++s2) {
            const int d = __shfl_sync(0xffffffffu, my_dst, s2);
            const int sr = __shfl_sync(0xffffffffu, my_src, s2);
            if (d <= R) {
              s_sel = s2;
              d_sel = d;
              src_sel = sr;
            }
          }
          rowp[it] = rr < nvalid ? static_cast<__nv_bfloat16*>(args.scatter.base[s_sel]) +
                                       (static_cast<int64_t>(src_sel) + (R - d_sel)) * args.ld_out_routed +
                                       tl.n * kBN
                                 : nullptr;
        }
#pragma unroll 1
        for (int c = 0; c < kBN; c += 64) {
          float v0[32], v1[32];
          tmem_ld32(taddr + c, v0);
          tmem_ld32(taddr + c + 32, v1);
          put_bf16x64(v0, v1, rowp, c);
        }
      } else {
        const bool f32 = !routed && args.shared_out_f32;
        const int64_t ld = routed ? args.ld_out_routed : args.ld_out_shared;
        if (f32) {
#pragma unroll 1
          for (int c = 0; c < kBN; c += 32) {
            float v[32];
            tmem_ld32(taddr + c, v);
            put_f32(v, static_cast<float*>(args.out_shared) + tl.n * kBN + c, ld, row0, nvalid,
                    args.shared_accumulate != 0);
          }
        } else {
          __nv_bfloat16* rowp[8];
          plain_rows(static_cast<__nv_bfloat16*>(routed ? args.out_routed : args.out_shared) + tl.n * kBN, ld, row0,
                     nvalid, rowp);
#pragma unroll 1
          for (int c = 0; c < kBN; c += 64) {
            float v0[32], v1[32];
            tmem_ld32(taddr + c, v0);
            tmem_ld32(taddr + c + 32, v1);
            put_bf16x64(v0, v1, rowp, c);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars.tmem_empty[acc]);
    }
  }
  __syncwarp();  // the single-lane roles rejoin their warps before the block barrier
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// bf16 [rows, cols] row-major, box = 64 columns x box_rows rows, 128-byte swizzle.
bool make_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiled fn = encoder();
  if (fn == nullptr || base == nullptr || cols % 8 != 0) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows > 0 ? rows : 1)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t grouped_gemm_smem_bytes() {
  return static_cast<size_t>(kStages) * kStageBytes + 4 * kStageTileBytes + 1024;
}

cudaError_t launch_grouped_gemm(const GroupedGemm& g, cudaStream_t stream) {
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < kMaxDevices && !attr_done[dev]) {
    st = cudaFuncSetAttribute(tc_grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(grouped_gemm_smem_bytes()));
    if (st != cudaSuccess) return st;
    attr_done[dev] = true;
  }
  if (g.k_routed % kBK != 0 || g.k_shared % kBK != 0 || g.experts > kMaxExperts)
    return cudaErrorInvalidValue;
  if (g.mode == 0 ? (g.n_cols_routed % (kBN / 2) != 0 || g.n_cols_shared % (kBN / 2) != 0)
                  : (g.n_cols_routed % kBN != 0 || g.n_cols_shared % kBN != 0))
    return cudaErrorInvalidValue;
  KernelArgs a{};
  const int b_box = kBN / 2;
  bool ok = g.experts == 0 || (make_tmap(&a.a_routed, g.a_routed, g.a_routed_rows, g.k_routed, kBM) &&
                               make_tmap(&a.b0_routed, g.b0_routed, g.b_routed_rows, g.k_routed, b_box) &&
                               make_tmap(&a.b1_routed, g.b1_routed, g.b_routed_rows, g.k_routed, b_box));
  if (ok && g.shared_rows > 0)
    ok = make_tmap(&a.a_shared, g.a_shared, g.shared_rows, g.k_shared, kBM) &&
         make_tmap(&a.b0_shared, g.b0_shared, g.b_shared_rows, g.k_shared, b_box) &&
         make_tmap(&a.b1_shared, g.b1_shared, g.b_shared_rows, g.k_shared, b_box);
  if (!ok) return cudaErrorInvalidValue;
  a.seg_count = g.seg_count;
  a.seg_start = g.seg_start;
  a.experts = g.experts;
  a.shared_rows = g.shared_rows;
  const int cols_per_tile = g.mode == 0 ? kBN / 2 : kBN;
  a.n_tiles_routed = g.n_cols_routed / cols_per_tile;
  a.n_tiles_shared = g.n_cols_shared / cols_per_tile;
  a.k_blocks_routed = g.k_routed / kBK;
  a.k_blocks_shared = g.k_shared / kBK;
  a.b_rows_per_expert = g.b_rows_per_expert;
  // SwiGLU: gate and up are separate matrices, same rows; store: the two
  // 128-row halves of one 256-row block of the same matrix.
  a.b1_offset = g.mode == 0 ? 0 : b_box;
  a.b_tile_rows = g.mode == 0 ? b_box : kBN;
  a.mode = g.mode;
  a.out_routed = g.out_routed;
  a.ld_out_routed = g.ld_out_routed;
  a.out_shared = g.out_shared;
  a.ld_out_shared = g.ld_out_shared;
  a.shared_out_f32 = g.shared_out_f32 ? 1 : 0;
  a.shared_accumulate = g.shared_accumulate ? 1 : 0;
  a.err = g.err;
  if (g.scatter.world < 0 || g.scatter.world > kMaxScatterRanks || (g.scatter.world > 0 && g.mode != 1))
    return cudaErrorInvalidValue;
  a.scatter = g.scatter;
  tc_grouped_gemm_kernel<<<g.blocks, kThreads, grouped_gemm_smem_bytes(), stream>>>(a);
  return cudaGetLastError();
}

}  // namespace uocr_b200
