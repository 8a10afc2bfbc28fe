// Softmax, top-k selection and the decode routing table, as device functions.
//
// Selection follows src/model/feed_forward.cpp:43-48 and the reference's
// softmax (src/backend/reference/ops.cpp:169-187): max shift, float exp,
// a double-precision total summed in index order, multiply by float(1/total);
// then k rounds of "best remaining", lower id on a tie. Renormalisation (the
// BASELINE semantics, absent in the reference) divides each selected weight
// by the rank-order float sum of the k weights.
//
// Every block of the decode expert kernels runs route_from_logits on the same
// logits and so holds the same table; nothing is exchanged between blocks.
#pragma once

#include "moe_common.cuh"

namespace uocr_b200 {

// Routing table in shared memory: experts in ascending id order, each with
// the batch rows routed to it in row order. Expert u's rows occupy slots
// base[u] .. base[u] + ntok[u] - 1; a slot indexes the [slots, F] activation
// rows and names its batch row and combine weight.
struct SmemRoute {
  int count;
  int expert[kMaxActive];
  int ntok[kMaxActive];
  int base[kMaxActive];
  int slot_tok[kMaxActive];
  float slot_w[kMaxActive];
  // scratch of route_from_logits
  int ids[kDecodeMaxRows * kMaxTopK];
  float w[kDecodeMaxRows * kMaxTopK];
  int slot_of[kMaxExperts];
  alignas(16) float ebuf[8][kMaxExperts];  // 16-byte rows: read as float4 by softmax_topk_warp
};

// Softmax + top-k of one row by one warp; lanes 0..K-1 write ids/weights
// (rank order). Every intermediate stays in registers.
template <typename IdT>
__device__ void softmax_topk_warp(const float* logits, int E, int K, int renorm, float* ebuf, IdT* ids,
                                  float* weights) {
  const int lane = threadIdx.x & 31;
  float v[4];
  float peak = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __ldcg(logits + e) : -INFINITY;
    peak = fmaxf(peak, v[i]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
  if (peak == -INFINITY) {
    // A fully masked row softmaxes to zeros (ops.cpp:175-177).
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = lane + 32 * i < E ? 0.0f : -INFINITY;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        v[i] = expf(v[i] - peak);
        ebuf[e] = v[i];
      }
    }
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      // The reference's double total in index order (ops.cpp:179-183); the
      // 16-byte reads are issued ahead of the dependent adds.
      double total = 0.0;
      int e = 0;
      for (; e + 3 < E; e += 4) {
        const float4 q = *reinterpret_cast<const float4*>(ebuf + e);
        total += static_cast<double>(q.x);
        total += static_cast<double>(q.y);
        total += static_cast<double>(q.z);
        total += static_cast<double>(q.w);
      }
      for (; e < E; ++e) total += static_cast<double>(ebuf[e]);
      inv = static_cast<float>(1.0 / total);
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < E) v[i] = v[i] * inv;
    __syncwarp();
  }
  // K rounds of warp argmax (lower id on a tie); lane j keeps round j's winner.
  float sum = 0.0f, my_w = 0.0f;
  int my_id = 0;
  for (int j = 0; j < K; ++j) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < best_e))) {
        best = v[i];
        best_e = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    // Remove the winner from its owner lane (a removed slot can never win again).
    if ((best_e & 31) == lane) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i == (best_e >> 5)) v[i] = -INFINITY;
    }
    if (lane == j) {
      my_w = best;
      my_id = best_e;
    }
    sum += best;
  }
  if (lane < K) {
    ids[lane] = static_cast<IdT>(my_id);
    weights[lane] = renorm ? my_w / sum : my_w;
  }
}

// Synchronises the threads building a routing table: one warp (nthreads 32)
// uses __syncwarp, more use named barrier `bar`.
__device__ __forceinline__ void route_sync(int bar, int nthreads) {
  if (nthreads == 32)
    __syncwarp();
  else
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
}

// Builds the routing table of T rows from logits [T, E] with `nthreads`
// threads (one warp, or a multiple of 32 synchronising on named barrier
// `bar`; tid < nthreads) that all call this function. When ids_out is not
// null the rank-order ids/weights are also written there.
__device__ inline void route_from_logits(const float* logits, int T, int E, int K, int renorm, SmemRoute* r, int tid,
                                         int nthreads, int bar, int* ids_out, float* w_out) {
  const int warp = tid >> 5, lane = tid & 31;
  const int row_warps = (nthreads >> 5) < 8 ? (nthreads >> 5) : 8;
  if (warp < row_warps)
    for (int t = warp; t < T; t += row_warps)
      softmax_topk_warp<int>(logits + static_cast<int64_t>(t) * E, E, K, renorm, r->ebuf[warp], r->ids + t * K,
                             r->w + t * K);
  for (int i = tid; i < kMaxExperts; i += nthreads) r->slot_of[i] = 0;
  for (int i = tid; i < kMaxActive; i += nthreads) r->ntok[i] = 0;
  route_sync(bar, nthreads);
  const int n = T * K;
  for (int i = tid; i < n; i += nthreads) {
    const int e = r->ids[i];
    if (e >= 0 && e < E) r->slot_of[e] = 1;  // the same value from every writer
    if (ids_out != nullptr) {
      ids_out[i] = e;
      w_out[i] = r->w[i];
    }
  }
  route_sync(bar, nthreads);
  if (warp == 0) {
    // Experts in ascending id order: exclusive scan of the used flags.
    int flags[4], local = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = lane * 4 + q;
      flags[q] = e < E ? r->slot_of[e] : 0;
      local += flags[q];
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int pos = incl - local;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = lane * 4 + q;
      if (flags[q]) {
        r->expert[pos] = e;
        r->slot_of[e] = pos++;
      }
    }
    if (lane == 31) r->count = incl;
  }
  route_sync(bar, nthreads);
  for (int i = tid; i < n; i += nthreads) {
    const int e = r->ids[i];
    if (e >= 0 && e < E) atomicAdd(&r->ntok[r->slot_of[e]], 1);
  }
  route_sync(bar, nthreads);
  if (warp == 0) {
    // base = exclusive scan of ntok over the experts in ascending id.
    const int U = r->count;
    int cnt[4], local = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int u = lane * 4 + q;
      cnt[q] = u < U ? r->ntok[u] : 0;
      local += cnt[q];
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int acc = incl - local;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int u = lane * 4 + q;
      if (u < U) r->base[u] = acc;
      acc += cnt[q];
    }
  }
  route_sync(bar, nthreads);
  // A selection's place among its expert's rows = how many earlier rows chose
  // that expert (ids within a row are distinct), so rows stay in row order.
  for (int i = tid; i < n; i += nthreads) {
    const int t = i / K, e = r->ids[i];
    if (e < 0 || e >= E) continue;
    int place = 0;
    for (int q = 0; q < t * K; ++q) place += r->ids[q] == e;
    const int slot = r->base[r->slot_of[e]] + place;
    r->slot_tok[slot] = t;
    r->slot_w[slot] = r->w[i];
  }
  route_sync(bar, nthreads);
}

// Writes a table built in shared memory to its global form (route_from_table's input).
__device__ inline void route_to_table(const SmemRoute* r, DecodeRoute* g, int tid, int nthreads) {
  const int U = r->count;
  if (tid == 0) {
    g->active_count = U;
    g->slot_total = U > 0 ? r->base[U - 1] + r->ntok[U - 1] : 0;
  }
  for (int u = tid; u < U; u += nthreads) {
    const int base = r->base[u], cnt = r->ntok[u];
    g->active_expert[u] = r->expert[u];
    g->tok_count[u] = cnt;
    g->slot_base[u] = base;
    for (int j = 0; j < cnt; ++j) {
      g->tok_index[u][j] = r->slot_tok[base + j];
      g->tok_weight[u][j] = r->slot_w[base + j];
    }
  }
}

// Copies a precomputed routing table (the expert_ffn_one mirrors) into shared memory.
__device__ inline void route_from_table(const DecodeRoute* g, int T, SmemRoute* r, int tid, int nthreads, int bar) {
  const int U = __ldcg(&g->active_count);
  if (tid == 0) r->count = U;
  for (int u = tid; u < U; u += nthreads) {
    const int base = __ldcg(&g->slot_base[u]);
    const int cnt = __ldcg(&g->tok_count[u]);
    r->expert[u] = __ldcg(&g->active_expert[u]);
    r->ntok[u] = cnt;
    r->base[u] = base;
    for (int j = 0; j < cnt; ++j) {
      r->slot_tok[base + j] = __ldcg(&g->tok_index[u][j]);
      r->slot_w[base + j] = __ldcg(&g->tok_weight[u][j]);
    }
  }
  (void)T;
  route_sync(bar, nthreads);
}

}  // namespace uocr_b200
