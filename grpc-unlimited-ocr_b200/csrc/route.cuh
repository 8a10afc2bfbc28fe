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

#include <cstddef>

#include "moe_common.cuh"

namespace uocr_b200 {

// Routing table in shared memory. Its leading members have DecodeRoute's
// layout (the global form written by the router), so the table moves between
// the two as a flat copy of 16-byte words. Expert u (ascending id) owns slots
// base[u] .. base[u] + ntok[u] - 1; a slot indexes the [slots, F] activation
// rows and names its batch row and combine weight.
struct SmemRoute {
  int count;
  int slot_total;
  int reserved[2];
  int expert[kMaxActive];
  int ntok[kMaxActive];
  int base[kMaxActive];
  int slot_tok[kMaxActive];
  float slot_w[kMaxActive];
  // scratch of route_from_logits
  int ids[kDecodeMaxRows * kMaxTopK];
  float w[kDecodeMaxRows * kMaxTopK];
  alignas(16) unsigned rowmask[kDecodeMaxRows][4];  // experts of each row, 128-bit mask
  alignas(16) float ebuf[8][kTopkScratch];
};
static_assert(offsetof(SmemRoute, count) == offsetof(DecodeRoute, active_count), "table layout");
static_assert(offsetof(SmemRoute, expert) == offsetof(DecodeRoute, active_expert), "table layout");
static_assert(offsetof(SmemRoute, ntok) == offsetof(DecodeRoute, tok_count), "table layout");
static_assert(offsetof(SmemRoute, base) == offsetof(DecodeRoute, slot_base), "table layout");
static_assert(offsetof(SmemRoute, slot_tok) == offsetof(DecodeRoute, slot_tok), "table layout");
static_assert(offsetof(SmemRoute, slot_w) == offsetof(DecodeRoute, slot_w), "table layout");
static_assert(sizeof(DecodeRoute) % 16 == 0, "table copied in 16-byte words");

// Logits of a row: from global memory through L2 (written by another block or
// an earlier grid), or from shared memory.
template <bool kShared>
__device__ __forceinline__ float load_logit(const float* p) {
  if constexpr (kShared)
    return *p;
  else
    return __ldcg(p);
}

// Nonzero softmax numerators at or above this make every partial sum of a
// row exact in double: each is then a multiple of 2^-45 (a float >= 2^-22 has
// an ulp >= 2^-45), and each of at most 128 terms is below 2 (the max-shifted
// exp), so every partial sum is an integer multiple of 2^-45 below 2^8,
// i.e. below 2^53 units. Exact sums do not depend on the order of the adds.
constexpr float kExactSumFloor = 2.384185791015625e-07f;  // 2^-22

// Selection key of expert e with probability p: the bits of p (a
// non-negative float orders like its bits) above ~e, so that a higher
// probability, then a lower id, gives a larger key and no two keys tie. A NaN
// probability keys as 0, below every number; padding entries are 0 as a whole.
__device__ __forceinline__ unsigned long long topk_key(float p, int e) {
  const unsigned hi = p > 0.0f ? __float_as_uint(p) : 0u;
  return (static_cast<unsigned long long>(hi) << 32) | (0xffffffffu - static_cast<unsigned>(e));
}

// Rank of each of the lane's N keys among the row's keys in shared memory
// (padded to an even count with 0): the number of larger keys.
template <int N>
__device__ __forceinline__ void rank_keys(const unsigned long long* keys, int Epad, const unsigned long long (&key)[4],
                                          int (&rank)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) rank[i] = 0;
#pragma unroll 4
  for (int c = 0; c < Epad; c += 2) {
    const ulonglong2 q = *reinterpret_cast<const ulonglong2*>(keys + c);
#pragma unroll
    for (int i = 0; i < N; ++i) rank[i] += static_cast<int>(q.x > key[i]) + static_cast<int>(q.y > key[i]);
  }
}

// Softmax + top-k of one row by one warp; lanes 0..K-1 write ids/weights in
// rank order. `scratch` is kTopkScratch floats of shared memory (16-byte
// aligned) owned by the warp.
//   softmax: max shift, float exp, the reference's double total in index
//     order (ops.cpp:179-183) — as a warp tree when every numerator is 0 or
//     at least kExactSumFloor (then the total is exact and equals the
//     sequential one bit for bit), else sequentially by lane 0 — and a
//     multiply by float(1 / total);
//   top-k: each element's rank is counted directly (higher probability first,
//     lower id on a tie, feed_forward.cpp:46-48) as the number of larger
//     64-bit keys (topk_key); ranks below K are the selection. A NaN
//     probability (NaN logits) ranks after every number.
//   renormalisation divides by the rank-order float sum of the k weights.
template <typename IdT, bool kSharedLogits = false>
__device__ void softmax_topk_warp(const float* logits, int E, int K, int renorm, float* scratch, IdT* ids,
                                  float* weights) {
  const int lane = threadIdx.x & 31;
  float* sums = scratch;                                                       // [kMaxExperts]
  auto* keys = reinterpret_cast<unsigned long long*>(scratch);                 // [kMaxExperts]
  float* sel_w = scratch + 2 * kMaxExperts;                                    // [kMaxTopK]
  int* sel_id = reinterpret_cast<int*>(scratch + 2 * kMaxExperts + kMaxTopK);  // [kMaxTopK]
  float v[4];
  float peak = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? load_logit<kSharedLogits>(logits + e) : -INFINITY;
    peak = fmaxf(peak, v[i]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
  if (peak == -INFINITY) {
    // A fully masked row softmaxes to zeros (ops.cpp:175-177).
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = 0.0f;
  } else {
    bool exact = true;
    double part = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (lane + 32 * i < E) {
        v[i] = expf(v[i] - peak);
        exact &= v[i] == 0.0f || v[i] >= kExactSumFloor;
        part += static_cast<double>(v[i]);
      }
    }
    double total;
    if (__all_sync(0xffffffffu, exact)) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      total = part;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (lane + 32 * i < E) sums[lane + 32 * i] = v[i];
      __syncwarp();
      total = 0.0;
      if (lane == 0)
        for (int e = 0; e < E; ++e) total += static_cast<double>(sums[e]);
      total = __shfl_sync(0xffffffffu, total, 0);
      __syncwarp();
    }
    const float inv = static_cast<float>(1.0 / total);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = v[i] * inv;
  }
  const int Epad = (E + 1) & ~1;
  unsigned long long key[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = lane + 32 * i;
    key[i] = e < E ? topk_key(v[i], e) : 0ull;
    if (e < Epad) keys[e] = key[i];
  }
  __syncwarp();
  int rank[4];
  if (E <= 64)
    rank_keys<2>(keys, Epad, key, rank);
  else
    rank_keys<4>(keys, Epad, key, rank);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = lane + 32 * i;
    if (e < E && rank[i] < K) {
      sel_w[rank[i]] = v[i];
      sel_id[rank[i]] = e;
    }
  }
  __syncwarp();
  if (lane < K) {
    float sum = 0.0f;
    for (int j = 0; j < K; ++j) sum += sel_w[j];
    const float w = sel_w[lane];
    ids[lane] = static_cast<IdT>(sel_id[lane]);
    weights[lane] = renorm ? w / sum : w;
  }
  __syncwarp();
}

// Synchronises the threads building a routing table: one warp (nthreads 32)
// uses __syncwarp, more use named barrier `bar`.
__device__ __forceinline__ void route_sync(int bar, int nthreads) {
  if (nthreads == 32)
    __syncwarp();
  else
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
}

// Number of set bits of a 128-bit mask below bit e.
__device__ __forceinline__ int popc_below(const uint4& m, int e) {
  const unsigned w[4] = {m.x, m.y, m.z, m.w};
  const int q = e >> 5;
  int n = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < q) n += __popc(w[i]);
    if (i == q) n += __popc(w[i] & ((1u << (e & 31)) - 1u));
  }
  return n;
}

// Builds the routing table of T rows from logits [T, E] (global memory, or
// shared memory when kSharedLogits) with `nthreads` threads (one warp, or a
// multiple of 32 synchronising on named barrier `bar`; tid < nthreads) that
// all call this function. When ids_out is not null the rank-order
// ids/weights are also written there.
//
// Each selection i (row t, expert e) finds its slot directly: slot = the
// number of selections of experts below e (= the expert's base) plus the
// number of earlier rows that chose e, so an expert's rows stay in row order;
// the expert's place among the active experts is the number of active experts
// below it (the union of the rows' masks).
template <bool kSharedLogits = false>
__device__ inline void route_from_logits(const float* logits, int T, int E, int K, int renorm, SmemRoute* r, int tid,
                                         int nthreads, int bar, int* ids_out, float* w_out) {
  const int warp = tid >> 5, lane = tid & 31;
  const int row_warps = (nthreads >> 5) < 8 ? (nthreads >> 5) : 8;
  if (warp < row_warps)
    for (int t = warp; t < T; t += row_warps) {
      softmax_topk_warp<int, kSharedLogits>(logits + static_cast<int64_t>(t) * E, E, K, renorm, r->ebuf[warp],
                                            r->ids + t * K, r->w + t * K);
      const int e = lane < K ? r->ids[t * K + lane] : -1;
      const bool valid = e >= 0 && e < E;
      unsigned m[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) m[q] = __reduce_or_sync(0xffffffffu, valid && (e >> 5) == q ? 1u << (e & 31) : 0u);
      if (lane == 0) *reinterpret_cast<uint4*>(r->rowmask[t]) = make_uint4(m[0], m[1], m[2], m[3]);
    }
  route_sync(bar, nthreads);
  uint4 used = make_uint4(0u, 0u, 0u, 0u);
  int slots = 0;
  for (int t = 0; t < T; ++t) {
    const uint4 m = *reinterpret_cast<const uint4*>(r->rowmask[t]);
    used.x |= m.x;
    used.y |= m.y;
    used.z |= m.z;
    used.w |= m.w;
    slots += __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w);
  }
  if (tid == 0) {
    r->count = __popc(used.x) + __popc(used.y) + __popc(used.z) + __popc(used.w);
    r->slot_total = slots;
  }
  const int n = T * K;
  for (int i = tid; i < n; i += nthreads) {
    const int e = r->ids[i];
    const float wi = r->w[i];
    if (ids_out != nullptr) {
      ids_out[i] = e;
      w_out[i] = wi;
    }
    if (e < 0 || e >= E) continue;
    int less = 0, same = 0, cnt = 0;
    for (int j = 0; j < n; ++j) {
      const int ej = r->ids[j];
      less += (ej >= 0) & (ej < e);
      cnt += ej == e;
      same += (ej == e) & (j < i);
    }
    const int slot = less + same;
    r->slot_tok[slot] = i / K;
    r->slot_w[slot] = wi;
    if (same == 0) {
      const int u = popc_below(used, e);
      r->expert[u] = e;
      r->ntok[u] = cnt;
      r->base[u] = less;
    }
  }
  route_sync(bar, nthreads);
}

// Writes a table built in shared memory to its global form (route_from_table's input).
__device__ inline void route_to_table(const SmemRoute* r, DecodeRoute* g, int tid, int nthreads) {
  constexpr int kWords = static_cast<int>(sizeof(DecodeRoute) / 16);
  const uint4* src = reinterpret_cast<const uint4*>(r);
  uint4* dst = reinterpret_cast<uint4*>(g);
  for (int i = tid; i < kWords; i += nthreads) dst[i] = src[i];
}

// Copies a table from its global form into shared memory: every load is
// issued before the first store, so the copy costs one trip to L2.
__device__ inline void route_from_table(const DecodeRoute* g, int T, SmemRoute* r, int tid, int nthreads, int bar) {
  constexpr int kWords = static_cast<int>(sizeof(DecodeRoute) / 16);
  constexpr int kPer = (kWords + 31) / 32;
  const uint4* src = reinterpret_cast<const uint4*>(g);
  uint4* dst = reinterpret_cast<uint4*>(r);
  for (int base = 0; base < kWords; base += kPer * nthreads) {
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = base + k * nthreads + tid;
      if (i < kWords) v[k] = __ldcg(src + i);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = base + k * nthreads + tid;
      if (i < kWords) dst[i] = v[k];
    }
  }
  (void)T;
  route_sync(bar, nthreads);
}

}  // namespace uocr_b200
