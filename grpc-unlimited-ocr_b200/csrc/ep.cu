// Expert-parallel prefill: the exchange between the route and expert phases
// and the barrier between the ranks' exchange regions. Rows cross NVLink as
// plain peer loads (the pull) and as plain peer stores (the down GEMM's
// epilogue sending each output row home, and the barrier's flags); no TMA
// touches peer memory — the grouped GEMMs read only this GPU's xrecv / act.
#include "ep.h"

#include "combine.cuh"
#include "moe_kernels.h"
#include "ptx.cuh"

namespace uocr_b200 {
namespace {

constexpr uint32_t kEpWaitPolls = 1u << 27;

__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int2 ld_relaxed_sys2(const int2* p) {
  int2 v;
  asm volatile("ld.relaxed.sys.global.v2.s32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_cg16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Every rank's per-expert counts and starts (peer loads) and the receive
// layout of this rank's expert slots. One block.
__global__ void __launch_bounds__(256) ep_prepare_kernel(EpMap m, EpPeers peers, EpLayout lay, EpScratch es,
                                                         ErrorWord* err) {
  __shared__ int cnt[kMaxEpRanks][kMaxExperts];
  __shared__ int tot[kMaxEpRanks * kMaxExperts];     // [d * max_local + i] rows slot i of rank d receives
  __shared__ int rstart[kMaxEpRanks * kMaxExperts];  // its first row in rank d's xrecv
  __shared__ int overflow;
  const int W = m.world, E = m.experts, ML = m.max_local;
  if (threadIdx.x == 0) overflow = 0;
  for (int idx = threadIdx.x; idx < W * E; idx += blockDim.x) {
    const int s = idx / E, e = idx % E;
    const int c = ld_relaxed_sys(reinterpret_cast<const int*>(peers.base[s] + lay.seg_count) + e);
    const int st = ld_relaxed_sys(reinterpret_cast<const int*>(peers.base[s] + lay.seg_start) + e);
    cnt[s][e] = c;
    es.cnt_all[idx] = c;
    es.seg_start_all[idx] = st;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < W * ML; q += blockDim.x) {
    const int d = q / ML, e = m.slot_expert[q];
    int t = 0;
    if (e >= 0)
      for (int s = 0; s < W; ++s) t += m.owner[e * W + s] == d ? cnt[s][e] : 0;
    tot[q] = t;
  }
  __syncthreads();
  if (threadIdx.x < W) {
    const int d = threadIdx.x;
    int64_t acc = 0;
    for (int i = 0; i < ML; ++i) {
      rstart[d * ML + i] = static_cast<int>(acc);
      acc += tot[d * ML + i];
    }
    if (acc > lay.max_recv) {
      raise_error(err, kDevCapacity, 60, d, static_cast<int>(acc));
      atomicExch(&overflow, 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < m.local; i += blockDim.x) {
    // On overflow nothing is received (the error word reports it).
    es.recv_count[i] = overflow ? 0 : tot[m.rank * ML + i];
    es.recv_start[i] = overflow ? 0 : rstart[m.rank * ML + i];
  }
  __syncthreads();
  // (slot i, source s) segments of this rank's receive layout: slot-major,
  // then source rank (the sources the owner table sends to this rank; the
  // others' segments are empty).
  for (int q = threadIdx.x; q < m.local * W; q += blockDim.x) {
    const int i = q / W, s = q % W, e = m.slot_expert[m.rank * ML + i];
    int d = overflow ? 0 : rstart[m.rank * ML + i];
    for (int s2 = 0; s2 < s; ++s2) d += m.owner[e * W + s2] == m.rank ? cnt[s2][e] : 0;
    es.seg_dst[q] = d;
    es.seg_src[q] = es.seg_start_all[s * E + e];
  }
}

// src_of of this rank's permuted positions: the row's index, and the position
// of its first selection on the same owner — the selections one owner takes
// reach its receive rows in ascending expert order (its slots are in
// ascending id), so the lowest expert id's position is the one the owner
// pulls over NVLink; the others point at it. Thread per row.
__global__ void ep_first_kernel(EpMap m, int T, int K, const int* __restrict__ ids, const int* __restrict__ pos_of,
                                int2* __restrict__ src_of) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int e[kMaxTopK], d[kMaxTopK], p[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j >= K) break;
    e[j] = ids[static_cast<int64_t>(t) * K + j];
    p[j] = pos_of[static_cast<int64_t>(t) * K + j];
    d[j] = (e[j] >= 0 && e[j] < m.experts) ? m.owner[e[j] * m.world + m.rank] : -1;
  }
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j >= K) break;
    if (p[j] < 0 || d[j] < 0) continue;
    int best = j;
#pragma unroll
    for (int i = 0; i < kMaxTopK; ++i) {
      if (i >= K) break;
      if (d[i] == d[j] && p[i] >= 0 && e[i] < e[best]) best = i;
    }
    src_of[p[j]] = make_int2(p[best], t);
  }
}

// xrecv rows of this rank's expert slots: slot-major, then source rank (the
// sources this slot takes; the others' segments are empty), each (slot,
// source) segment the source's selections of that expert in permuted order
// (= row order), each row fetched from the source's x^ by the index src_of
// gives. One warp per row, grid-stride; 16-byte peer loads, all of a row in
// flight at once.
__global__ void __launch_bounds__(256) ep_pull_kernel(EpMap m, EpPeers peers, EpLayout lay, EpScratch es, int H) {
  __shared__ int seg_dst[kMaxEpRanks * kMaxExperts];
  __shared__ int seg_src[kMaxEpRanks * kMaxExperts];
  __shared__ int seg_rank[kMaxEpRanks * kMaxExperts];
  __shared__ int total;
  const int W = m.world, L = m.local, n = W * L, E = m.experts;
  for (int q = threadIdx.x; q < n; q += blockDim.x) {
    seg_dst[q] = es.seg_dst[q];
    seg_src[q] = es.seg_src[q];
    seg_rank[q] = q % W;
  }
  if (threadIdx.x == 0) total = es.recv_start[L - 1] + es.recv_count[L - 1];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nch = H / 8;  // 16-byte chunks per row
  for (int r = warp; r < total; r += nwarps) {
    int lo = 0, hi = n - 1;  // last segment starting at or before r (empty segments share the next one's start)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg_dst[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int s = seg_rank[lo];
    const int src_row = seg_src[lo] + (r - seg_dst[lo]);
    // A row this rank takes for several experts crosses once: the position
    // of its lowest-id selection owned here is pulled, the others copied
    // from xrecv afterwards (ep_dup_kernel).
    // The copy source is a receive row before r (its expert id is lower); a
    // position that does not resolve to one is pulled like any other.
    int from = -1, tok = 0;
    if (lane == 0) {
      const int2 so = ld_relaxed_sys2(reinterpret_cast<const int2*>(peers.base[s] + lay.src_of) + src_row);
      const int fp = so.x;
      tok = so.y;
      if (fp >= 0 && fp < src_row) {
        // fp's expert: the last expert of source s whose segment starts at
        // or before it (empty segments start where the next one does).
        const int* st = es.seg_start_all + s * E;
        int a = 0, b = E - 1;
        while (a < b) {
          const int mid = (a + b + 1) >> 1;
          if (st[mid] <= fp) a = mid;
          else b = mid - 1;
        }
        if (m.owner[a * W + s] == m.rank) {
          const int q = m.slot[a * W + s] * W + s;
          const int r0 = es.seg_dst[q] + (fp - es.seg_src[q]);
          if (r0 >= 0 && r0 < r) from = r0;
        }
      }
      es.dup[r] = from;
    }
    from = __shfl_sync(0xffffffffu, from, 0);
    if (from >= 0) continue;
    tok = __shfl_sync(0xffffffffu, tok, 0);
    if (tok < 0 || tok >= lay.max_rows) continue;  // never for a consistent table
    const uint4* src = reinterpret_cast<const uint4*>(peers.base[s] + lay.xhat) + static_cast<int64_t>(tok) * nch;
    uint4* dst = reinterpret_cast<uint4*>(es.xrecv) + static_cast<int64_t>(r) * nch;
    for (int c0 = 0; c0 < nch; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = c0 + lane + 32 * u;
        if (idx < nch) v[u] = ld_cg16(src + idx);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = c0 + lane + 32 * u;
        if (idx < nch) dst[idx] = v[u];
      }
    }
  }
}

// The rows ep_pull_kernel left to copy locally: each from the receive row
// that pulled it. One warp per row, grid-stride.
__global__ void __launch_bounds__(256) ep_dup_kernel(EpMap m, EpScratch es, int H) {
  const int total = es.recv_start[m.local - 1] + es.recv_count[m.local - 1];
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nch = H / 8;
  for (int r = warp; r < total; r += nwarps) {
    const int from = es.dup[r];
    if (from < 0 || from >= r) continue;  // pulled (a copy always comes from an earlier row)
    const uint4* src = reinterpret_cast<const uint4*>(es.xrecv) + static_cast<int64_t>(from) * nch;
    uint4* dst = reinterpret_cast<uint4*>(es.xrecv) + static_cast<int64_t>(r) * nch;
    for (int c0 = 0; c0 < nch; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = c0 + lane + 32 * u;
        if (idx < nch) v[u] = ld_cg16(src + idx);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = c0 + lane + 32 * u;
        if (idx < nch) dst[idx] = v[u];
      }
    }
  }
}

__global__ void ep_arrive_kernel(EpPeers peers, EpLayout lay, int rank, int world, unsigned* epoch) {
  unsigned e = 0;
  if (threadIdx.x == 0) {
    e = *epoch + 1;
    *epoch = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  __threadfence_system();
  if (static_cast<int>(threadIdx.x) < world)
    st_release_sys(reinterpret_cast<unsigned*>(peers.base[threadIdx.x] + lay.flags) + rank, e);
}

__global__ void ep_wait_kernel(const unsigned* flags, int world, const unsigned* epoch, ErrorWord* err, int site,
                               uint64_t wait_ns) {
  if (static_cast<int>(threadIdx.x) >= world) return;
  const unsigned target = *epoch;
  const unsigned* f = flags + threadIdx.x;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (static_cast<int>(ld_acquire_sys(f) - target) >= 0) break;
    if (i >= kEpWaitPolls || ((i & 63u) == 63u && global_timer_ns() - start > wait_ns)) {
      raise_error(err, kDevWaitTimeout, site, static_cast<int>(threadIdx.x), static_cast<int>(target));
      break;
    }
    __nanosleep(200);
  }
  __threadfence_system();
}

}  // namespace

bool build_ep_tables(int experts, int world, const int32_t* owner_in, bool strided, EpTables* t, std::string* why) {
  const int E = experts, W = world;
  t->world = W;
  t->experts = E;
  t->owner.assign(static_cast<size_t>(E) * W, 0);
  for (int e = 0; e < E; ++e)
    for (int s = 0; s < W; ++s) {
      int d;
      if (owner_in != nullptr) {
        d = owner_in[e * W + s];
        if (d < 0 || d >= W) {
          *why = "owner of expert " + std::to_string(e) + " for rank " + std::to_string(s) + " is not a rank";
          return false;
        }
      } else {
        if (E % W != 0) {
          *why = "routed_experts must be a multiple of ep_world without an owner table";
          return false;
        }
        d = strided ? e % W : e / (E / W);
      }
      t->owner[static_cast<size_t>(e) * W + s] = d;
    }
  // Slots: rank d's experts in ascending id.
  std::vector<std::vector<int>> held(static_cast<size_t>(W));
  for (int e = 0; e < E; ++e)
    for (int d = 0; d < W; ++d)
      for (int s = 0; s < W; ++s)
        if (t->owner[static_cast<size_t>(e) * W + s] == d) {
          held[static_cast<size_t>(d)].push_back(e);
          break;
        }
  t->max_local = 0;
  t->slot_count.assign(static_cast<size_t>(W), 0);
  for (int d = 0; d < W; ++d) {
    const int n = static_cast<int>(held[static_cast<size_t>(d)].size());
    if (n == 0) {
      *why = "rank " + std::to_string(d) + " holds no expert";
      return false;
    }
    t->slot_count[static_cast<size_t>(d)] = n;
    if (n > t->max_local) t->max_local = n;
  }
  t->slot_expert.assign(static_cast<size_t>(W) * t->max_local, -1);
  t->slot.assign(static_cast<size_t>(E) * W, 0);
  for (int d = 0; d < W; ++d)
    for (size_t i = 0; i < held[static_cast<size_t>(d)].size(); ++i)
      t->slot_expert[static_cast<size_t>(d) * t->max_local + i] = held[static_cast<size_t>(d)][i];
  for (int e = 0; e < E; ++e)
    for (int s = 0; s < W; ++s) {
      const int d = t->owner[static_cast<size_t>(e) * W + s];
      const auto& h = held[static_cast<size_t>(d)];
      int i = 0;
      while (h[static_cast<size_t>(i)] != e) ++i;
      t->slot[static_cast<size_t>(e) * W + s] = i;
    }
  uint64_t h = 1469598103934665603ull;  // FNV-1a over the owner table
  for (int v : t->owner) {
    h ^= static_cast<uint64_t>(static_cast<uint32_t>(v));
    h *= 1099511628211ull;
  }
  t->hash = h;
  return true;
}

EpLayout ep_layout(const PrefillDims& d, const EpMap& m) {
  EpLayout l{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = align256(off);
    const size_t at = off;
    off += bytes;
    return at;
  };
  const size_t T = static_cast<size_t>(d.max_rows), K = d.top_k, E = d.experts, H = d.hidden;
  l.flags = take(kMaxEpRanks * sizeof(unsigned));
  l.seg_count = take(E * 4);
  l.seg_start = take(E * 4);
  l.max_rows = static_cast<int64_t>(T);
  l.xhat = take(T * H * 2);
  l.src_of = take(T * K * 8);
  l.max_recv = static_cast<int64_t>(m.world) * static_cast<int64_t>(T) *
               (K < static_cast<size_t>(m.max_local) ? static_cast<int64_t>(K) : static_cast<int64_t>(m.max_local));
  l.yback = take(T * K * H * 2);
  l.bytes = align256(off);
  return l;
}

size_t ep_scratch_bytes(const PrefillDims& d, const EpLayout& lay, const EpMap& m) {
  EpScratch s{};
  carve_ep_scratch(d, lay, m, nullptr, &s);
  return s.bytes;
}

void carve_ep_scratch(const PrefillDims& d, const EpLayout& lay, const EpMap& m, void* base, EpScratch* s) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    off = align256(off);
    char* p = base == nullptr ? nullptr : static_cast<char*>(base) + off;
    off += bytes;
    return p;
  };
  const size_t W = m.world, E = d.experts, L = m.local, H = d.hidden, F = d.ffn, R = lay.max_recv;
  s->cnt_all = reinterpret_cast<int*>(take(W * E * 4));
  s->seg_start_all = reinterpret_cast<int*>(take(W * E * 4));
  s->recv_count = reinterpret_cast<int*>(take(L * 4));
  s->recv_start = reinterpret_cast<int*>(take(L * 4));
  s->seg_dst = reinterpret_cast<int*>(take(L * W * 4));
  s->seg_src = reinterpret_cast<int*>(take(L * W * 4));
  s->dup = reinterpret_cast<int*>(take(static_cast<size_t>(R) * 4));
  s->epoch = reinterpret_cast<unsigned*>(take(sizeof(unsigned)));
  s->xrecv = reinterpret_cast<__nv_bfloat16*>(take(R * H * 2));
  s->act = reinterpret_cast<__nv_bfloat16*>(take(R * F * 2));
  s->bytes = align256(off);
}

cudaError_t ep_route(const EpCall& c, cudaStream_t stream) {
  cudaError_t st = launch_prefill_route(c.pc, stream);
  if (st != cudaSuccess || c.pc.rows <= 0) return st;
  const int T = c.pc.rows;
  ep_first_kernel<<<(T + 255) / 256, 256, 0, stream>>>(c.map, T, c.pc.dims.top_k, c.pc.ids, c.pc.scratch.pos_of,
                                                     reinterpret_cast<int2*>(c.peers.base[c.map.rank] + c.lay.src_of));
  return cudaGetLastError();
}

cudaError_t ep_experts(const EpCall& c, cudaStream_t stream, cudaEvent_t after_pull) {
  const PrefillDims& d = c.pc.dims;
  ep_prepare_kernel<<<1, 256, 0, stream>>>(c.map, c.peers, c.lay, c.es, c.pc.err);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  ep_pull_kernel<<<c.pc.sm_count * 4, 256, 0, stream>>>(c.map, c.peers, c.lay, c.es, d.hidden);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  ep_dup_kernel<<<c.pc.sm_count * 4, 256, 0, stream>>>(c.map, c.es, d.hidden);
  if ((st = cudaGetLastError()) != cudaSuccess) return st;
  if (after_pull != nullptr && (st = cudaEventRecord(after_pull, stream)) != cudaSuccess) return st;
  const int L = c.map.local;
  GroupedGemm g1 = prefill_gate_up_gemm(c.pc, true, false);
  g1.experts = L;
  g1.seg_count = c.es.recv_count;
  g1.seg_start = c.es.recv_start;
  g1.a_routed = c.es.xrecv;
  g1.a_routed_rows = c.lay.max_recv;
  g1.b0_routed = c.gate_local;
  g1.b1_routed = c.up_local;
  g1.b_routed_rows = static_cast<int64_t>(L) * d.ffn;
  g1.out_routed = c.es.act;
  if ((st = launch_grouped_gemm(g1, stream)) != cudaSuccess) return st;
  GroupedGemm g2 = prefill_down_gemm(c.pc, true, false);
  g2.experts = L;
  g2.seg_count = c.es.recv_count;
  g2.seg_start = c.es.recv_start;
  g2.a_routed = c.es.act;
  g2.a_routed_rows = c.lay.max_recv;
  g2.b0_routed = c.down_local;
  g2.b1_routed = c.down_local;
  g2.b_routed_rows = static_cast<int64_t>(L) * d.hidden;
  g2.out_routed = nullptr;  // every row goes home through the scatter
  g2.scatter.world = c.map.world;
  g2.scatter.seg_dst = c.es.seg_dst;
  g2.scatter.seg_src = c.es.seg_src;
  for (int s = 0; s < c.map.world; ++s) g2.scatter.base[s] = c.peers.base[s] + c.lay.yback;
  return launch_grouped_gemm(g2, stream);
}

cudaError_t ep_shared(const EpCall& c, cudaStream_t stream) {
  if (c.pc.rows <= 0 || c.pc.dims.shared_ffn <= 0) return cudaSuccess;
  cudaError_t st = launch_grouped_gemm(prefill_gate_up_gemm(c.pc, false, true), stream);
  if (st != cudaSuccess) return st;
  return launch_grouped_gemm(prefill_down_gemm(c.pc, false, true), stream);
}

cudaError_t ep_combine(const EpCall& c, cudaStream_t stream) { return launch_prefill_combine(c.pc, stream); }

cudaError_t ep_arrive(const EpCall& c, cudaStream_t stream) {
  ep_arrive_kernel<<<1, 32, 0, stream>>>(c.peers, c.lay, c.map.rank, c.map.world, c.es.epoch);
  return cudaGetLastError();
}

cudaError_t ep_wait(const EpCall& c, int site, cudaStream_t stream) {
  const auto* flags = reinterpret_cast<const unsigned*>(c.peers.base[c.map.rank] + c.lay.flags);
  ep_wait_kernel<<<1, 32, 0, stream>>>(flags, c.map.world, c.es.epoch, c.pc.err, site, c.wait_ns);
  return cudaGetLastError();
}

cudaError_t ep_forward(const EpCall& c, cudaStream_t stream, cudaEvent_t* ev) {
  auto mark = [&](int i) { return ev != nullptr ? cudaEventRecord(ev[i], stream) : cudaSuccess; };
  cudaError_t st;
  if ((st = ep_route(c, stream)) != cudaSuccess || (st = mark(0)) != cudaSuccess) return st;
  if ((st = ep_arrive(c, stream)) != cudaSuccess || (st = ep_wait(c, 61, stream)) != cudaSuccess ||
      (st = mark(1)) != cudaSuccess)
    return st;
  // The shared expert needs only this rank's own rows (x^): on the side
  // stream it runs while the pull, which NVLink bounds, crosses to this rank
  // and the routed GEMMs follow. The measurement path keeps one stream so
  // that its phases stay separable.
  const bool overlap = ev == nullptr && c.side != nullptr && c.pc.rows > 0 && c.pc.dims.shared_ffn > 0;
  if (overlap) {
    if ((st = cudaEventRecord(c.fork, stream)) != cudaSuccess ||
        (st = cudaStreamWaitEvent(c.side, c.fork, 0)) != cudaSuccess || (st = ep_shared(c, c.side)) != cudaSuccess ||
        (st = cudaEventRecord(c.join, c.side)) != cudaSuccess)
      return st;
  }
  if ((st = ep_experts(c, stream, ev != nullptr ? ev[2] : nullptr)) != cudaSuccess || (st = mark(3)) != cudaSuccess)
    return st;
  if ((st = ep_arrive(c, stream)) != cudaSuccess) return st;
  if (overlap) {
    if ((st = cudaStreamWaitEvent(stream, c.join, 0)) != cudaSuccess) return st;
  } else if ((st = ep_shared(c, stream)) != cudaSuccess) {
    return st;
  }
  if ((st = ep_wait(c, 62, stream)) != cudaSuccess || (st = mark(4)) != cudaSuccess) return st;
  if ((st = ep_combine(c, stream)) != cudaSuccess) return st;
  return mark(5);
}

}  // namespace uocr_b200
