// Router logits for many rows (the prefill and expert-parallel routers) in
// the CPU reference's fp32 dot order.
//
// ptxas fuses a mul.rn.f32x2 that feeds an add.rn.f32x2 into one
// fma.rn.f32x2, even with -fmad=false (measured on B200: the packed pair gave
// fmaf's result, not __fadd_rn(__fmul_rn)'s), which rounds once where the
// reference rounds the product and the sum separately. The product is
// therefore fma.rn.f32x2(x, w, -0) with the -0 a kernel argument: one rounding
// of x * w, exactly mul.rn's result (x * w + -0 == x * w, signed zeros
// included), and nothing left for ptxas to fuse with the add.
#include "moe_kernels.h"
#include "prefill.h"

namespace uocr_b200 {
namespace {

constexpr int kRouterTokens = 32;   // rows per router block
constexpr int kRouterExperts = 32;  // experts per router block
constexpr int kRouterChunk = 64;    // K elements staged per step
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Packed fp32 pairs (sm_100 f32x2): two independent chains advance per
// instruction, each element rounded as by __fmul_rn / __fadd_rn.
// mul2_rn(a, b, nz): nz holds -0.0f in both halves, unknown to the compiler.
__device__ __forceinline__ uint64_t mul2_rn(uint64_t a, uint64_t b, uint64_t nz) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(nz));
  return d;
}
__device__ __forceinline__ uint64_t add2_rn(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
  return f;
}
__device__ __forceinline__ void cp_async8(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(valid ? 8 : 0) : "memory");
}

// logits[t, e] in the reference's dot order (eight lane partial sums over
// i = 8j + lane, fixed tree, tail, bias: src/backend/reference/ops.cpp:25-38,
// :91-109), every product and sum separately rounded.
//
// A block covers 32 rows x 32 experts. The chains of lanes 2p and 2p+1 of one
// (row, expert) travel as one packed pair, so a thread owns lane pair p of
// 4 rows x 4 experts (16 packed accumulators) and one packed multiply and
// one packed add advance two chains. K is staged in chunks of 64 by 8-byte
// asynchronous copies (lanes 2p, 2p+1 of one j are adjacent in memory; rows
// 8-byte aligned) into
// [row][lane pair][j][2] tiles, rows padded to 20 floats, two buffers deep; a
// 16-byte shared read then holds the pairs of two consecutive j. Rows of a
// thread are rg + 8r and experts eg + 8i, so the addresses of one warp-wide
// read spread over all banks. Blocks with the same rows are adjacent in the
// grid: the second expert block finds the rows in L2.
constexpr int kRouterPer = kRouterChunk / 8;            // chain elements per lane per chunk
constexpr int kRouterPad = 2 * kRouterPer + 4;          // floats per (row, lane pair)
constexpr int kRouterTile = kRouterTokens * 4 * kRouterPad;  // floats per operand tile
static_assert(kRouterTokens == 32 && kRouterExperts == 32, "8 row groups x 8 expert groups x 4 lane pairs");
size_t router_rows_smem_bytes() { return static_cast<size_t>(4) * kRouterTile * sizeof(float); }

__global__ void __launch_bounds__(256, 3) router_logits_rows_kernel(const float* __restrict__ x, int T, int H,
                                                                    const float* __restrict__ router,
                                                                    const float* __restrict__ bias, int E,
                                                                    float* __restrict__ logits, float neg_zero) {
  extern __shared__ __align__(16) float rsm[];  // [2 buffers][x tile, w tile]
  const int tid = threadIdx.x;
  const int lp = tid & 3;                                     // lane pair: lanes 2lp, 2lp+1
  const int eg = ((tid >> 2) & 3) + 4 * ((tid >> 5) & 1);     // expert group 0..7
  const int rg = ((tid >> 4) & 1) + 2 * (tid >> 6);           // row group 0..7
  const int eblocks = (E + kRouterExperts - 1) / kRouterExperts;
  const int rblock = blockIdx.x / eblocks;
  const int e0 = (blockIdx.x - rblock * eblocks) * kRouterExperts;
  const int t0 = rblock * kRouterTokens;
  const int ne = min(kRouterExperts, E - e0);
  const int full = H & ~7;
  const int nchunks = (full + kRouterChunk - 1) / kRouterChunk;

  // Staging: element pairs (c, c+1), c even, of rows sr + 8u (u = 0..3).
  const int sc = 2 * (tid & 31), sr = tid >> 5;
  const int soff = (sr * 4 + ((sc & 7) >> 1)) * kRouterPad + 2 * (sc >> 3);
  unsigned xmask = 0, wmask = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    xmask |= (t0 + sr + 8 * u < T ? 1u : 0u) << u;
    wmask |= (sr + 8 * u < ne ? 1u : 0u) << u;
  }
  const float* xsrc = x + static_cast<int64_t>(min(t0 + sr, T - 1)) * H + sc;
  const float* wsrc = router + static_cast<int64_t>(e0 + min(sr, ne - 1)) * H + sc;
  const int64_t rstep = static_cast<int64_t>(8) * H;
  auto stage = [&](int chunk) {
    float* xs = rsm + (chunk & 1) * 2 * kRouterTile + soff;
    float* ws = xs + kRouterTile;
    const int k0 = chunk * kRouterChunk;
    const bool cok = sc < full - k0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bool okx = cok && ((xmask >> u) & 1u), okw = cok && ((wmask >> u) & 1u);
      const float* gx = okx ? xsrc + u * rstep + k0 : x;
      const float* gw = okw ? wsrc + u * rstep + k0 : router;
      float* dx = xs + u * 8 * 4 * kRouterPad;
      float* dw = ws + u * 8 * 4 * kRouterPad;
      cp_async8(dx, gx, okx);
      cp_async8(dw, gw, okw);
    }
    cp_async_commit();
  };

  uint64_t nz;
  asm("mov.b64 %0, {%1, %1};" : "=l"(nz) : "f"(neg_zero));
  uint64_t acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[r][i] = 0;  // +0.0f in both halves
  if (nchunks > 0) stage(0);
  for (int ch = 0; ch < nchunks; ++ch) {
    if (ch + 1 < nchunks) {
      stage(ch + 1);
      cp_async_wait_one();
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const float* xs = rsm + (ch & 1) * 2 * kRouterTile + (rg * 4 + lp) * kRouterPad;
    const float* ws = rsm + (ch & 1) * 2 * kRouterTile + kRouterTile + (eg * 4 + lp) * kRouterPad;
    const int per = min(kRouterChunk, full - ch * kRouterChunk) >> 3;
    if (per == kRouterPer) {
#pragma unroll
      for (int m = 0; m < 2 * kRouterPer; m += 4) {  // two j per 16-byte read
        ulonglong2 xv[4], wv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) xv[r] = *reinterpret_cast<const ulonglong2*>(xs + r * 8 * 4 * kRouterPad + m);
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const ulonglong2*>(ws + i * 8 * 4 * kRouterPad + m);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint64_t a = add2_rn(acc[r][i], mul2_rn(xv[r].x, wv[i].x, nz));
            acc[r][i] = add2_rn(a, mul2_rn(xv[r].y, wv[i].y, nz));
          }
      }
    } else {
      for (int j = 0; j < per; ++j) {
        uint64_t xv[4], wv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) xv[r] = *reinterpret_cast<const uint64_t*>(xs + r * 8 * 4 * kRouterPad + 2 * j);
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const uint64_t*>(ws + i * 8 * 4 * kRouterPad + 2 * j);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[r][i] = add2_rn(acc[r][i], mul2_rn(xv[r], wv[i], nz));
      }
    }
    __syncthreads();  // this buffer is refilled two chunks on
  }
  // The eight lanes of each (row, expert) sit in four consecutive threads,
  // two per thread. Thread lp keeps expert eg + 8 lp of its four rows.
  const int base = (tid & 31) & ~3;
  float sum[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    sum[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack2(__shfl_sync(0xffffffffu, acc[r][i], base + q));
        a[2 * q] = f.x;
        a[2 * q + 1] = f.y;
      }
      const float lo = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
      const float hi = __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7]));
      if (lp == i) sum[r] = __fadd_rn(lo, hi);
    }
  }
  const int el = eg + 8 * lp;
  if (el >= ne) return;
  const int e = e0 + el;
  const float* wr = router + static_cast<int64_t>(e) * H;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = t0 + rg + 8 * r;
    if (t >= T) break;
    const float* xrow = x + static_cast<int64_t>(t) * H;
    float tail = 0.0f;
    for (int c = full; c < H; ++c) tail = __fadd_rn(tail, __fmul_rn(__ldg(xrow + c), __ldg(wr + c)));
    float v = __fadd_rn(sum[r], tail);
    if (bias != nullptr) v = __fadd_rn(v, bias[e]);
    logits[static_cast<int64_t>(t) * E + e] = v;
  }
}

}  // namespace

cudaError_t launch_router_logits_rows(const float* x, int T, int H, const float* router, const float* bias, int E,
                                      float* logits, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < kMaxDevices && !attr_done[dev]) {
    st = cudaFuncSetAttribute(router_logits_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(router_rows_smem_bytes()));
    if (st != cudaSuccess) return st;
    attr_done[dev] = true;
  }
  const int64_t blocks = static_cast<int64_t>((T + kRouterTokens - 1) / kRouterTokens) *
                         ((E + kRouterExperts - 1) / kRouterExperts);
  // The 8-byte copies need 8-byte aligned rows: x and the router are 16-byte
  // aligned (checked at the C ABI; plan allocations) and H is a multiple of 16.
  router_logits_rows_kernel<<<static_cast<unsigned>(blocks), 256, router_rows_smem_bytes(), stream>>>(
      x, T, H, router, bias, E, logits, -0.0f);
  return cudaGetLastError();
}

}  // namespace uocr_b200
