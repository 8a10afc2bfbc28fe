// Decode-path experts on the 5th-generation tensor cores (bf16 weights).
//
// A decode batch has at most 16 rows, so each expert matrix product is a
// weight-streaming GEMV. Here the weights are the MMA's A operand (128 weight
// rows x 64 K per TMA tile, 128-byte swizzle) and the batch rows are B
// (N = 16, zero-padded), so D = W . X^T lands in TMEM as [128 rows x 16 batch
// rows] and the CUDA cores only touch the results. Work items are
// (expert or shared, 128-row block, K split); blocks take items round-robin.
// A K split writes its partial sums to global scratch and the last split to
// finish (an atomic ticket, no waiting) adds the splits in K order:
//   gate/up: act[u][t][f] = bf16(silu(sum_ks G) * sum_ks U)   (all 16 batch rows)
//   down:    y[t][c] = shared + sum over the row's experts, ascending id, of w * sum_ks D
// so results do not depend on timing. Roles per block: warp 0 TMA producer,
// warp 1 TMEM owner and MMA issuer, warps 2-5 epilogue.
//
// Reference counterpart: expert_gate_up_kernel / expert_down_kernel and the
// shared expert's gemv_kernel (src/backend/cuda/gemv_ops.cu:133-183).
#include <cuda.h>

#include <mutex>

#include "decode_tc.h"
#include "moe_kernels.h"
#include "route.cuh"
#include "tc.cuh"

namespace uocr_b200 {
namespace {

constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kBarEpi = 3;  // named barrier over the four epilogue warps
constexpr int kRowsB = 16;  // N of the MMA: batch rows, zero padded
constexpr uint32_t kIdesc = bf16_idesc(128, kRowsB);
constexpr int kTmemCols = 64;

struct __align__(8) DBars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t route_ready;
  uint64_t b_ready;
  uint64_t drain;
};

// Item split of one kernel: "units" (part, 128-row block) x ksplit K ranges.
struct Split {
  int ksplit;
  int kb_per_unit;
};

__device__ __forceinline__ Split choose_split(int units, int kblocks, int sm_count, int max_items) {
  int ks = (4 * sm_count + units - 1) / (units > 0 ? units : 1);  // about four items per block
  if (ks < 1) ks = 1;
  if (ks > kblocks) ks = kblocks;
  while (ks > 1 && units * ks > max_items) --ks;
  return Split{ks, kblocks};
}

__device__ __forceinline__ void kb_range(int kblocks, int ksplit, int ks, int& kb0, int& kb1) {
  kb0 = kblocks * ks / ksplit;
  kb1 = kblocks * (ks + 1) / ksplit;
}

__device__ __forceinline__ void init_bars(DBars& b, int stages) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&b.full[s], 1);
    mbar_init(&b.empty[s], 1);
  }
  for (int i = 0; i < 2; ++i) {
    mbar_init(&b.tmem_full[i], 1);
    mbar_init(&b.tmem_empty[i], kEpiThreads);
  }
  mbar_init(&b.route_ready, 1);
  mbar_init(&b.b_ready, kEpiThreads);
  mbar_init(&b.drain, 1);
  fence_mbar_init();
}

// The routing table, built by one warp (lane = its lane index).
__device__ __forceinline__ void build_route(const DecodeRouting& rt, int T, SmemRoute* r, int lane, bool with_ids) {
  if (rt.logits != nullptr) {
    const bool out = with_ids && blockIdx.x == 0;
    route_from_logits(rt.logits, T, rt.experts, rt.top_k, rt.renormalize, r, lane, 32, 0,
                      out ? rt.ids_out : nullptr, out ? rt.weights_out : nullptr);
  } else {
    route_from_table(rt.table, T, r, lane, 32, 0);
  }
}

// Element (row r, column k) of a K-major, 128-byte-swizzled tile set with
// 64-element K blocks of `rows` rows each.
__device__ __forceinline__ uint32_t sw128_offset(int r, int k, int rows) {
  const int kb = k >> 6, kk = k & 63;
  const int chunk = (kk >> 3) ^ (r & 7);
  return static_cast<uint32_t>(kb * rows * 128 + r * 128 + chunk * 16 + (kk & 7) * 2);
}

// ---------------------------------------------------------------------------
struct GateUpArgs {
  CUtensorMap gate, up, sgate, sup;  // [E*F, H] and [S, H], box 64 x 128
  const float* x;                    // [T, H] fp32
  int T, H, F, S;
  DecodeRouting routing;
  __nv_bfloat16* act;                // [kMaxActive][16][F]
  __nv_bfloat16* act_s;              // [16][S]
  float* partial;                    // [items][2][16][128]
  unsigned* tickets;                 // [groups]
  int max_items;
  int stages;
  int sm_count;
  ErrorWord* err;
};

__global__ void __launch_bounds__(kThreads, 1) gate_up_tc_kernel(const __grid_constant__ GateUpArgs a) {
  extern __shared__ unsigned char dyn_raw[];
  __shared__ DBars bars;
  __shared__ SmemRoute sroute;
  __shared__ uint32_t tmem_holder;
  __shared__ int last_flag;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* xb = smem;                              // x^ [16 x H] bf16, swizzled, 1024-aligned
  unsigned char* ring = smem + kRowsB * a.H * 2;         // stages x (gate 16 KB + up 16 KB)
  constexpr int kTile = 128 * 64 * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = a.H / 64;
  const int sh_units = a.S / 128, fb_per_expert = a.F / 128;

  if (threadIdx.x == 0) init_bars(bars, a.stages);
  if (warp == 1) tmem_alloc(&tmem_holder, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  // Shared units are known now; routed units once the routing table exists.
  const Split sh_split = choose_split(sh_units, kblocks, a.sm_count, a.max_items / 2);
  const int sh_items = sh_units * sh_split.ksplit;

  if (warp == 0) {
    // ---- producer ----
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto load_item = [&](const CUtensorMap* g, const CUtensorMap* u, int row, int kb0, int kb1) {
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        if (lane == 0) {
          if (!mbar_wait(&bars.empty[stage], phase ^ 1)) {
            raise_error(a.err, kDevWaitTimeout, 50, kb, 0);
            ok = false;
          } else {
            mbar_arrive_expect_tx(&bars.full[stage], 2 * kTile);
            unsigned char* d = ring + stage * 2 * kTile;
            tma_load_2d(d, g, kb * 64, row, &bars.full[stage]);
            tma_load_2d(d + kTile, u, kb * 64, row, &bars.full[stage]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (++stage == a.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    };
    for (int i = blockIdx.x; i < sh_items && ok; i += gridDim.x) {
      const int unit = i / sh_split.ksplit, ks = i % sh_split.ksplit;
      int kb0, kb1;
      kb_range(kblocks, sh_split.ksplit, ks, kb0, kb1);
      load_item(&a.sgate, &a.sup, unit * 128, kb0, kb1);
    }
    pdl_wait();  // the router's logits are complete from here on
    build_route(a.routing, a.T, &sroute, lane, true);
    if (lane == 0) mbar_arrive(&bars.route_ready);
    pdl_launch_dependents();
    const int units = sroute.count * fb_per_expert;
    const Split sp = choose_split(units, kblocks, a.sm_count, a.max_items / 2);
    const int items = units * sp.ksplit;
    // Routed items continue the block's round-robin after the shared ones.
    const int first = (blockIdx.x - sh_items % gridDim.x + gridDim.x) % gridDim.x;
    for (int i = first; i < items && ok; i += gridDim.x) {
      const int unit = i / sp.ksplit, ks = i % sp.ksplit;
      const int u = unit / fb_per_expert, fb = unit % fb_per_expert;
      int kb0, kb1;
      kb_range(kblocks, sp.ksplit, ks, kb0, kb1);
      load_item(&a.gate, &a.up, sroute.expert[u] * a.F + fb * 128, kb0, kb1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (!mbar_wait(&bars.b_ready, 0)) raise_error(a.err, kDevWaitTimeout, 51, 0, 0);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    const uint32_t xb_addr = smem_addr(xb);
    auto mma_item = [&](int kb0, int kb1) {
      const int acc = local & 1;
      if (lane == 0) {
        if (!mbar_wait(&bars.tmem_empty[acc], ((local >> 1) & 1) ^ 1)) {
          raise_error(a.err, kDevWaitTimeout, 52, local, 0);
          ok = false;
        }
        tc_fence_after();
        const uint32_t dg = tmem + acc * 32, du = dg + 16;
        for (int kb = kb0; kb < kb1 && ok; ++kb) {
          if (!mbar_wait(&bars.full[stage], phase)) {
            raise_error(a.err, kDevWaitTimeout, 53, kb, 0);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(ring + stage * 2 * kTile);
          const uint64_t gdesc = sw128_kmajor_desc(sa), udesc = sw128_kmajor_desc(sa + kTile);
          const uint64_t xdesc = sw128_kmajor_desc(xb_addr + kb * kRowsB * 128);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            umma_bf16(dg, gdesc + 2 * k, xdesc + 2 * k, kIdesc, accum);
            umma_bf16(du, udesc + 2 * k, xdesc + 2 * k, kIdesc, accum);
          }
          umma_commit(&bars.empty[stage]);
          if (++stage == a.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&bars.tmem_full[acc]);
      } else {
        for (int kb = kb0; kb < kb1; ++kb)
          if (++stage == a.stages) {
            stage = 0;
            phase ^= 1;
          }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++local;
    };
    for (int i = blockIdx.x; i < sh_items && ok; i += gridDim.x) {
      int kb0, kb1;
      kb_range(kblocks, sh_split.ksplit, i % sh_split.ksplit, kb0, kb1);
      mma_item(kb0, kb1);
    }
    if (!mbar_wait(&bars.route_ready, 0)) raise_error(a.err, kDevWaitTimeout, 54, 0, 0);
    pdl_launch_dependents();
    const int units = sroute.count * fb_per_expert;
    const Split sp = choose_split(units, kblocks, a.sm_count, a.max_items / 2);
    const int items = units * sp.ksplit;
    const int first = (blockIdx.x - sh_items % gridDim.x + gridDim.x) % gridDim.x;
    for (int i = first; i < items && ok; i += gridDim.x) {
      int kb0, kb1;
      kb_range(kblocks, sp.ksplit, i % sp.ksplit, kb0, kb1);
      mma_item(kb0, kb1);
    }
    if (lane == 0) {
      umma_commit(&bars.drain);
      if (!mbar_wait(&bars.drain, 0)) raise_error(a.err, kDevWaitTimeout, 55, 0, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue warps: x^ into shared memory, then per item the results ----
    const int et = threadIdx.x - 64;  // 0..127
    for (int i = et; i < kRowsB * a.H; i += kEpiThreads) {
      const int r = i / a.H, k = i % a.H;
      const float v = r < a.T ? __ldcg(a.x + static_cast<int64_t>(r) * a.H + k) : 0.0f;
      *reinterpret_cast<__nv_bfloat16*>(xb + sw128_offset(r, k, kRowsB)) = __float2bfloat16_rn(v);
    }
    fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
    mbar_arrive(&bars.b_ready);
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    // Item `i` of a part whose partial slots start at `slot0`; the K splits of
    // one (part, row block) are the ksplit consecutive items from a multiple of ksplit.
    auto epi_item = [&](int slot0, int i, int ksplit, bool shared_part, int u, int fb, int group) {
      const int item = slot0 + i;
      const int acc = local & 1;
      if (!mbar_wait(&bars.tmem_full[acc], (local >> 1) & 1)) {
        raise_error(a.err, kDevWaitTimeout, 56, item, 0);
        return false;
      }
      tc_fence_after();
      float g[32], uu[32];
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 32;
      tmem_ld32(base, g);  // columns 0..15 gate, 16..31 up
      tc_fence_before();
      mbar_arrive(&bars.tmem_empty[acc]);
      ++local;
#pragma unroll
      for (int t = 0; t < kRowsB; ++t) uu[t] = g[16 + t];
      const int f = fb * 128 + row;
      bool last = true;
      if (ksplit > 1) {
        float* pp = a.partial + static_cast<int64_t>(item) * 2 * kRowsB * 128;
        for (int t = 0; t < a.T; ++t) {
          pp[t * 128 + row] = g[t];
          pp[(kRowsB + t) * 128 + row] = uu[t];
        }
        __threadfence();
        named_bar_sync(kBarEpi, kEpiThreads);
        if (et == 0) last_flag = atomicAdd(&a.tickets[group], 1u) == static_cast<unsigned>(ksplit - 1);
        named_bar_sync(kBarEpi, kEpiThreads);
        last = last_flag != 0;
        if (last) {
          __threadfence();
          const int item0 = slot0 + i - i % ksplit;
          for (int t = 0; t < a.T; ++t) {
            float gs = 0.0f, us = 0.0f;
            for (int s = 0; s < ksplit; ++s) {
              const float* q = a.partial + static_cast<int64_t>(item0 + s) * 2 * kRowsB * 128;
              gs = __fadd_rn(gs, __ldcg(q + t * 128 + row));
              us = __fadd_rn(us, __ldcg(q + (kRowsB + t) * 128 + row));
            }
            g[t] = gs;
            uu[t] = us;
          }
          if (et == 0) a.tickets[group] = 0u;  // ready for the next launch
        }
      }
      if (last) {
        for (int t = 0; t < a.T; ++t) {
          const __nv_bfloat16 v = __float2bfloat16_rn(swiglu(g[t], uu[t]));
          if (shared_part)
            a.act_s[static_cast<int64_t>(t) * a.S + f] = v;
          else
            a.act[(static_cast<int64_t>(u) * kRowsB + t) * a.F + f] = v;
        }
      }
      return true;
    };
    bool ok = true;
    for (int i = blockIdx.x; i < sh_items && ok; i += gridDim.x) {
      const int unit = i / sh_split.ksplit;
      ok = epi_item(0, i, sh_split.ksplit, true, 0, unit, unit);
    }
    if (!mbar_wait(&bars.route_ready, 0)) raise_error(a.err, kDevWaitTimeout, 57, 0, 0);
    pdl_launch_dependents();
    const int units = sroute.count * fb_per_expert;
    const Split sp = choose_split(units, kblocks, a.sm_count, a.max_items / 2);
    const int items = units * sp.ksplit;
    const int first = (blockIdx.x - sh_items % gridDim.x + gridDim.x) % gridDim.x;
    for (int i = first; i < items && ok; i += gridDim.x) {
      const int unit = i / sp.ksplit;
      ok = epi_item(sh_items, i, sp.ksplit, false, unit / fb_per_expert, unit % fb_per_expert, sh_units + unit);
    }
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
struct DownArgs {
  CUtensorMap down, sdown;  // A: [E*H, F] and [H, S], box 64 x 128
  CUtensorMap act, act_s;   // B: [kMaxActive*16, F] and [16, S], box 64 x 16
  int T, H, F, S;
  DecodeRouting routing;
  const float* resid;
  float* y;
  float* partial;           // [items][16][128]
  unsigned* tickets;        // [H / 128]
  int max_items;
  int stages;
  int sm_count;
  ErrorWord* err;
};

// Items: channel block cb (outer), part p (shared = 0 when S > 0, then the
// experts), K split (inner), so one channel block's items are consecutive.
__global__ void __launch_bounds__(kThreads, 1) down_tc_kernel(const __grid_constant__ DownArgs a) {
  extern __shared__ unsigned char dyn_raw[];
  __shared__ DBars bars;
  __shared__ SmemRoute sroute;
  __shared__ uint32_t tmem_holder;
  __shared__ int last_flag;
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kATile = 128 * 64 * 2;     // 16 KB
  constexpr int kBTile = kRowsB * 64 * 2;  // 2 KB
  constexpr int kStage = kATile + kBTile;  // 18 KB, keeps 1024-byte alignment
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cblocks = a.H / 128;
  const int sh_parts = a.S > 0 ? 1 : 0;

  if (threadIdx.x == 0) init_bars(bars, a.stages);
  if (warp == 1) tmem_alloc(&tmem_holder, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  // The router grid finished before this grid started (the gate/up grid
  // released it only after its own wait): the whole block builds the table.
  if (warp == 0) {
    build_route(a.routing, a.T, &sroute, lane, false);
    if (lane == 0) mbar_arrive(&bars.route_ready);
  }
  if (!mbar_wait(&bars.route_ready, 0)) raise_error(a.err, kDevWaitTimeout, 60, 0, 0);
  const int parts = sh_parts + sroute.count;
  // Every part's K range is split the same number of ways over its own K, at
  // most the K blocks of the shortest part so that no split is empty.
  const int kmax = (a.S > 0 && a.S < a.F ? a.S : a.F) / 64;
  const Split sp = choose_split(cblocks * parts, kmax, a.sm_count, a.max_items);
  const int items = cblocks * parts * sp.ksplit;
  auto decode_item = [&](int i, int& cb, int& p, int& ks) {
    ks = i % sp.ksplit;
    p = (i / sp.ksplit) % parts;
    cb = i / (sp.ksplit * parts);
  };
  auto part_kblocks = [&](int p) { return (p < sh_parts ? a.S : a.F) / 64; };

  if (warp == 0) {
    // ---- producer: A tiles (weights) may stream before the activations exist ----
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true, waited = false;
    for (int i = blockIdx.x; i < items && ok; i += gridDim.x) {
      int cb, p, ks;
      decode_item(i, cb, p, ks);
      const int kbs = part_kblocks(p);
      const int kb0 = kbs * ks / sp.ksplit, kb1 = kbs * (ks + 1) / sp.ksplit;
      const bool shared_part = p < sh_parts;
      const int u = p - sh_parts;
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        if (lane == 0) {
          if (!mbar_wait(&bars.empty[stage], phase ^ 1)) {
            raise_error(a.err, kDevWaitTimeout, 61, kb, 0);
            ok = false;
          } else {
            mbar_arrive_expect_tx(&bars.full[stage], kStage);
            unsigned char* d = ring + stage * kStage;
            if (shared_part)
              tma_load_2d(d, &a.sdown, kb * 64, cb * 128, &bars.full[stage]);
            else
              tma_load_2d(d, &a.down, kb * 64, sroute.expert[u] * a.H + cb * 128, &bars.full[stage]);
            if (!waited) {
              pdl_wait();  // the activations come from the gate/up grid
              waited = true;
            }
            if (shared_part)
              tma_load_2d(d + kATile, &a.act_s, kb * 64, 0, &bars.full[stage]);
            else
              tma_load_2d(d + kATile, &a.act, kb * 64, u * kRowsB, &bars.full[stage]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (++stage == a.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    __syncwarp();
    pdl_wait();
    pdl_launch_dependents();
  } else if (warp == 1) {
    // ---- MMA issuer ----
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < items && ok; i += gridDim.x, ++local) {
      int cb, p, ks;
      decode_item(i, cb, p, ks);
      const int kbs = part_kblocks(p);
      const int kb0 = kbs * ks / sp.ksplit, kb1 = kbs * (ks + 1) / sp.ksplit;
      const int acc = local & 1;
      if (lane == 0) {
        if (!mbar_wait(&bars.tmem_empty[acc], ((local >> 1) & 1) ^ 1)) {
          raise_error(a.err, kDevWaitTimeout, 62, i, 0);
          ok = false;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * 16;
        for (int kb = kb0; kb < kb1 && ok; ++kb) {
          if (!mbar_wait(&bars.full[stage], phase)) {
            raise_error(a.err, kDevWaitTimeout, 63, kb, 0);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(ring + stage * kStage);
          const uint64_t adesc = sw128_kmajor_desc(sa), bdesc = sw128_kmajor_desc(sa + kATile);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_bf16(d, adesc + 2 * k, bdesc + 2 * k, kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&bars.empty[stage]);
          if (++stage == a.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&bars.tmem_full[acc]);
      } else {
        for (int kb = kb0; kb < kb1; ++kb)
          if (++stage == a.stages) {
            stage = 0;
            phase ^= 1;
          }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0) {
      umma_commit(&bars.drain);
      if (!mbar_wait(&bars.drain, 0)) raise_error(a.err, kDevWaitTimeout, 64, 0, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue ----
    const int et = threadIdx.x - 64;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    pdl_wait();
    pdl_launch_dependents();
    for (int i = blockIdx.x; i < items; i += gridDim.x, ++local) {
      int cb, p, ks;
      decode_item(i, cb, p, ks);
      const int acc = local & 1;
      if (!mbar_wait(&bars.tmem_full[acc], (local >> 1) & 1)) {
        raise_error(a.err, kDevWaitTimeout, 65, i, 0);
        break;
      }
      tc_fence_after();
      float d[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 16, d);  // columns 0..15 used
      tc_fence_before();
      mbar_arrive(&bars.tmem_empty[acc]);
      float* pp = a.partial + static_cast<int64_t>(i) * kRowsB * 128;
      for (int t = 0; t < a.T; ++t) pp[t * 128 + row] = d[t];
      __threadfence();
      named_bar_sync(kBarEpi, kEpiThreads);
      if (et == 0)
        last_flag = atomicAdd(&a.tickets[cb], 1u) == static_cast<unsigned>(parts * sp.ksplit - 1);
      named_bar_sync(kBarEpi, kEpiThreads);
      if (last_flag == 0) continue;
      __threadfence();
      // Last item of this channel block: shared part, then the experts in
      // ascending id, each summed over its K splits in order.
      const int c = cb * 128 + row;
      const int item0 = cb * parts * sp.ksplit;
      for (int t = 0; t < a.T; ++t) {
        float shared = 0.0f, routed = 0.0f;
        for (int q = 0; q < parts; ++q) {
          float s = 0.0f;
          for (int k2 = 0; k2 < sp.ksplit; ++k2)
            s = __fadd_rn(s, __ldcg(a.partial + static_cast<int64_t>(item0 + q * sp.ksplit + k2) * kRowsB * 128 +
                                    t * 128 + row));
          if (q < sh_parts) {
            shared = s;
          } else {
            const int u = q - sh_parts;
            for (int j = 0; j < sroute.ntok[u]; ++j)
              if (sroute.slot_tok[sroute.base[u] + j] == t)
                routed = __fadd_rn(routed, __fmul_rn(sroute.slot_w[sroute.base[u] + j], s));
          }
        }
        const int64_t o = static_cast<int64_t>(t) * a.H + c;
        float out = __fadd_rn(shared, routed);
        if (a.resid != nullptr) out = __fadd_rn(a.resid[o], out);
        a.y[o] = out;
      }
      if (et == 0) a.tickets[cb] = 0u;
    }
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

size_t decode_tc_scratch_bytes(int H, int F, int S) {
  DecodeTcScratch s{};
  carve_decode_tc_scratch(H, F, S, nullptr, &s);
  return s.bytes;
}

void carve_decode_tc_scratch(int H, int F, int S, void* base, DecodeTcScratch* s) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    off = (off + 255) / 256 * 256;
    char* p = base == nullptr ? nullptr : static_cast<char*>(base) + off;
    off += bytes;
    return p;
  };
  s->act = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(kMaxActive) * kRowsB * F * 2));
  s->act_s = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(kRowsB) * (S > 0 ? S : 64) * 2));
  s->max_items = kDecodeTcMaxItems;
  s->partial = reinterpret_cast<float*>(take(static_cast<size_t>(kDecodeTcMaxItems) * 2 * kRowsB * 128 * 4));
  const int groups = (S > 0 ? S / 128 : 0) + kMaxActive * (F / 128);
  s->tickets_gu = reinterpret_cast<unsigned*>(take(static_cast<size_t>(groups) * 4));
  s->tickets_dn = reinterpret_cast<unsigned*>(take(static_cast<size_t>(H / 128) * 4));
  s->bytes = off;
}

bool decode_tc_shapes_ok(int H, int F, int S) { return H % 128 == 0 && F % 128 == 0 && S % 128 == 0 && H <= 8192; }

cudaError_t launch_decode_tc(const DecodeTcCall& c, cudaStream_t stream) {
  static std::once_flag once;
  static EncodeTiled enc = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<EncodeTiled>(p);
  });
  if (enc == nullptr) return cudaErrorNotSupported;
  auto tmap = [&](CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows > 0 ? rows : 1)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attrs[kMaxDevices] = {};
  const int gu_stages = 3, dn_stages = 6;
  const size_t gu_smem = 1024 + static_cast<size_t>(kRowsB) * c.H * 2 + gu_stages * 2 * 128 * 64 * 2;
  const size_t dn_smem = 1024 + static_cast<size_t>(dn_stages) * (128 * 64 * 2 + kRowsB * 64 * 2);
  if (dev < kMaxDevices && !attrs[dev]) {
    cudaError_t st = allow_max_dynamic_smem(gate_up_tc_kernel);
    if (st == cudaSuccess) st = allow_max_dynamic_smem(down_tc_kernel);
    if (st != cudaSuccess) return st;
    attrs[dev] = true;
  }
  const int S = c.S;
  GateUpArgs g{};
  bool ok = tmap(&g.gate, c.gate, static_cast<int64_t>(c.E) * c.F, c.H, 128) &&
            tmap(&g.up, c.up, static_cast<int64_t>(c.E) * c.F, c.H, 128);
  if (ok && S > 0) ok = tmap(&g.sgate, c.sgate, S, c.H, 128) && tmap(&g.sup, c.sup, S, c.H, 128);
  if (!ok) return cudaErrorInvalidValue;
  g.x = c.x;
  g.T = c.T;
  g.H = c.H;
  g.F = c.F;
  g.S = S;
  g.routing = c.routing;
  g.act = c.scratch.act;
  g.act_s = c.scratch.act_s;
  g.partial = c.scratch.partial;
  g.tickets = c.scratch.tickets_gu;
  g.max_items = c.scratch.max_items;
  g.stages = gu_stages;
  g.sm_count = c.sm_count;
  g.err = c.err;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(c.sm_count);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = gu_smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = c.pdl ? 1 : 0;
  cudaError_t st = cudaLaunchKernelEx(&cfg, gate_up_tc_kernel, g);
  if (st != cudaSuccess) return st;
  if (c.between != nullptr && (st = cudaEventRecord(c.between, stream)) != cudaSuccess) return st;

  DownArgs d{};
  ok = tmap(&d.down, c.down, static_cast<int64_t>(c.E) * c.H, c.F, 128) &&
       tmap(&d.act, c.scratch.act, static_cast<int64_t>(kMaxActive) * kRowsB, c.F, kRowsB);
  if (ok && S > 0) ok = tmap(&d.sdown, c.sdown, c.H, S, 128) && tmap(&d.act_s, c.scratch.act_s, kRowsB, S, kRowsB);
  if (!ok) return cudaErrorInvalidValue;
  d.T = c.T;
  d.H = c.H;
  d.F = c.F;
  d.S = S;
  d.routing = c.routing;
  d.routing.ids_out = nullptr;
  d.routing.weights_out = nullptr;
  d.resid = c.resid;
  d.y = c.y;
  d.partial = c.scratch.partial;
  d.tickets = c.scratch.tickets_dn;
  d.max_items = c.scratch.max_items;
  d.stages = dn_stages;
  d.sm_count = c.sm_count;
  d.err = c.err;
  cfg.dynamicSmemBytes = dn_smem;
  cfg.numAttrs = (c.pdl && c.between == nullptr) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, down_tc_kernel, d);
}

}  // namespace uocr_b200
