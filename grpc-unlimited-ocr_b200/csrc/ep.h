// Expert-parallel prefill across the GPUs of one node (ep.cu): one process
// per GPU, each owning a slice of the rows and routed_experts / world of the
// experts. The reference has no multi-GPU path (no NCCL or MPI anywhere in
// its src/); this is the dispatch/combine exchange that expert sharding needs.
//
// Every rank holds one exchange region (a cudaMalloc block shared through
// CUDA IPC) with the same layout on every rank:
//   flags     [kMaxEpRanks] u32   barrier epochs, flags[s] written by rank s
//   seg_count [E] i32, seg_start [E] i32   this rank's rows per global expert
//   xhat      [max_rows, H] bf16          this rank's rows, bf16-rounded
//   src_of    [max_rows*k] {i32, i32}     per permuted position (the expert-
//                                          grouped order of the selections):
//                                          the position of the same row's
//                                          selection with the lowest expert id
//                                          among those the same rank owns, and
//                                          the row's index in xhat
//   yback     [max_rows*k, H] bf16        the selections' expert outputs, by
//                                          permuted position
// Per layer, on rank r:
//   route    router + top-k + the permutation of its own rows, x^ (the
//            single-GPU prefill stages)
//   barrier  (arrive, wait)
//   experts  for each of its experts, the rows of every rank's segment of
//            that expert are pulled over NVLink (peer loads of x^ rows) into
//            xrecv, source rank order, so an expert's rows are in global row
//            order as on one GPU — a row that several of its experts take
//            crosses once (src_of), the other copies are made from xrecv
//            itself; the
//            down GEMM's epilogue stores each output row into the yback of
//            the rank it came from (peer stores, tile by tile), at the
//            permuted position of the selection on that rank
//   (the shared expert on its own rows runs alongside, on a second stream)
//   arrive, wait
//   combine  the single-GPU combine over its own yback: every selection's
//            output row is local by then.
// Each output row of the grouped GEMM depends on its own input row only, so
// the result is bitwise the single-GPU result for the same rows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "prefill.h"

namespace uocr_b200 {

constexpr int kMaxEpRanks = 8;

// Which rank computes which rows. The rows of expert e that rank s routed go
// to rank owner[e * world + s], into that rank's expert slot
// slot[e * world + s]; rank d holds slot_count[d] experts, its slot i being
// expert slot_expert[d * max_local + i] (slots in ascending expert id). An
// expert may live on several ranks (a hot expert's rows split by source
// rank), and ranks may hold different numbers of experts. The tables live in
// device memory (the plan's arena); every rank builds the same ones.
struct EpMap {
  int world, rank, experts;
  int local;      // this rank's slot count
  int max_local;  // the largest slot count of any rank
  const int* owner;        // [experts * world]
  const int* slot;         // [experts * world]
  const int* slot_expert;  // [world * max_local], -1 past a rank's slot count
};

// The host copy of the tables, from an owner table [experts * world] or, when
// owner_in is null, from contiguous ranges (e / (experts / world)) or the
// strided map (e % world), both with every source going to the one owner.
struct EpTables {
  int world = 0, experts = 0, max_local = 0;
  std::vector<int> owner, slot, slot_expert, slot_count;
  uint64_t hash = 0;  // of the owner table: ranks connect only with the same map
};
// False (with the reason) when an owner is outside [0, world), a rank holds
// no expert, or the experts cannot be split by the rules above.
bool build_ep_tables(int experts, int world, const int32_t* owner_in, bool strided, EpTables* t, std::string* why);

// Exchange region base of every rank (this rank's own included).
struct EpPeers {
  char* base[kMaxEpRanks];
};

struct EpLayout {
  size_t flags, seg_count, seg_start, xhat, src_of, yback, bytes;
  int64_t max_recv;  // rows one rank's experts can receive: world * max_rows * min(k, local)
  int64_t max_rows;  // rows of xhat
};
EpLayout ep_layout(const PrefillDims& d, const EpMap& m);

// Per-rank scratch outside the exchange region.
struct EpScratch {
  int* cnt_all;      // [world, E] every rank's rows per global expert, read after the first barrier
  int* seg_start_all;  // [world, E] and where they start in that rank's permuted order
  int* recv_count;   // [local] rows each local expert receives
  int* recv_start;   // [local] its first row in xrecv
  int* seg_dst;      // [local * world] first xrecv row of (slot i, source s)
  int* seg_src;      // [local * world] that segment's first permuted position in source s
  int* dup;          // [max_recv] receive row to copy this one from (a row pulled once), -1: pulled
  unsigned* epoch;   // barrier epoch counter
  __nv_bfloat16* xrecv;  // [max_recv, H]
  __nv_bfloat16* act;    // [max_recv, F]
  size_t bytes;
};
size_t ep_scratch_bytes(const PrefillDims& d, const EpLayout& lay, const EpMap& m);
void carve_ep_scratch(const PrefillDims& d, const EpLayout& lay, const EpMap& m, void* base, EpScratch* s);

struct EpCall {
  PrefillCall pc;  // this rank's rows; pc.scratch's seg_count/seg_start/xhat/yperm point into its exchange
                   // region, xperm is null (owners pull rows from x^)
  EpMap map;
  EpPeers peers;
  EpLayout lay;
  EpScratch es;
  // This rank's experts only: gate/up [local*F, H], down [local*H, F].
  const __nv_bfloat16* gate_local;
  const __nv_bfloat16* up_local;
  const __nv_bfloat16* down_local;
  uint64_t wait_ns;  // how long a barrier waits for the other ranks
  // A stream of the plan's own and two events: ep_forward runs the shared
  // expert there while the pull and the routed GEMMs run on the caller's
  // stream (null: everything on the caller's stream).
  cudaStream_t side;
  cudaEvent_t fork, join;
};

// The phases of one layer; ep_forward runs them with the barriers between.
cudaError_t ep_route(const EpCall& c, cudaStream_t stream);
cudaError_t ep_experts(const EpCall& c, cudaStream_t stream, cudaEvent_t after_pull = nullptr);
cudaError_t ep_shared(const EpCall& c, cudaStream_t stream);
cudaError_t ep_combine(const EpCall& c, cudaStream_t stream);
// Barrier over the ranks' exchange regions: arrive publishes this rank's
// next epoch to every rank; wait spins (bounded: wait_ns, then an error word)
// until every rank published it. Data written before arrive on any rank is
// visible to every rank's kernels after its wait.
cudaError_t ep_arrive(const EpCall& c, cudaStream_t stream);
cudaError_t ep_wait(const EpCall& c, int site, cudaStream_t stream);
// Optional events (6): after route, the first wait, the pull of the rows
// over NVLink, the expert GEMMs, the shared expert and second wait, combine.
cudaError_t ep_forward(const EpCall& c, cudaStream_t stream, cudaEvent_t* events = nullptr);

}  // namespace uocr_b200
