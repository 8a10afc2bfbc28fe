"""Host side of expert parallelism (the prefill path sharded over the GPUs of
one node): which rows and experts each rank owns, and the handle exchange that
connects the ranks' plans.

torch.distributed is only the plumbing here — it carries the 256-byte
handles once at set-up. Rows and expert outputs cross NVLink inside the
library's kernels (peer loads from CUDA IPC mappings), with device-side
barriers between the phases of a layer.

The reference has no multi-GPU path (its src/ has no NCCL or MPI); one
process drives one device (src/backend/cuda/context.cu:50-56), which is the
model kept here: one process per GPU, each with its own plan.
"""
from __future__ import annotations


def rows_of(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s contiguous slice of `total` rows;
    the first total % world ranks take one row more."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def expert_owner(e: int, experts: int, world: int, strided: bool = False) -> int:
    """Rank holding expert e: contiguous ranges, or e % world when strided
    (the same map as EpMap in the library)."""
    return e % world if strided else e // (experts // world)


def local_experts(rank: int, experts: int, world: int, strided: bool = False) -> list[int]:
    """Global ids of `rank`'s experts in its local order (ascending)."""
    local = experts // world
    return [i * world + rank if strided else rank * local + i for i in range(local)]


def owner_table(experts: int, world: int, strided: bool = False) -> list[int]:
    """The built-in maps as an owner table [experts * world]: entry
    e * world + s = the rank computing expert e's rows from source rank s."""
    return [expert_owner(e, experts, world, strided) for e in range(experts) for _ in range(world)]


def slots_of(owner: list[int], experts: int, world: int, rank: int) -> list[int]:
    """Global ids of the experts `rank` holds under an owner table (its slots,
    in ascending id), as the library derives them."""
    return [e for e in range(experts) if any(owner[e * world + s] == rank for s in range(world))]


def rows_received(owner: list[int], counts_by_source, experts: int, world: int) -> list[int]:
    """Rows each rank's experts receive: counts_by_source[s][e] = rows source
    rank s routed to expert e."""
    got = [0] * world
    for e in range(experts):
        for s in range(world):
            got[owner[e * world + s]] += int(counts_by_source[s][e])
    return got


def rows_pulled_from(ids, owner: list[int], world: int, rank: int) -> list[int]:
    """How many of source `rank`'s rows each rank pulls over NVLink: a row
    crosses once to every other rank that owns at least one of its selected
    experts (for this source), however many of them it owns. ids [rows, k]."""
    import numpy as np
    ids = np.asarray(ids, np.int64).reshape(len(ids), -1) if len(ids) else np.zeros((0, 1), np.int64)
    own = np.asarray(owner, np.int64)[ids * world + rank]
    return [int((own == d).any(axis=1).sum()) if d != rank else 0 for d in range(world)]


def balanced_owner_table(counts_by_source, world: int, share: float = 0.5) -> list[int]:
    """An owner table that evens out the rows the ranks' experts receive,
    from a calibration histogram counts_by_source[s][e] (rows source rank s
    routes to expert e; a Zipf-skewed router gives the same shape on every
    batch, so one batch calibrates).

    Hot experts are replicated: expert e with load L_e gets the smallest
    number of replicas r dividing world with L_e / r <= share * (total /
    world), replica j taking the rows of sources s with s % r == j (so each
    replica sees whole source segments and the single-GPU row order within
    them). Then longest-processing-time first: the replica loads in
    descending order, each to the least-loaded rank that does not already hold
    that expert (ties: fewer experts, then lower rank). Deterministic, so every
    rank computes the same table from the same histogram."""
    W = world
    E = len(counts_by_source[0])
    load = [sum(int(counts_by_source[s][e]) for s in range(W)) for e in range(E)]
    target = max(1.0, sum(load) / W)
    divisors = [r for r in range(1, W + 1) if W % r == 0]
    items = []
    for e in range(E):
        r = next((r for r in divisors if load[e] / r <= share * target), W)
        for j in range(r):
            srcs = [s for s in range(W) if s % r == j]
            items.append((sum(int(counts_by_source[s][e]) for s in srcs), e, j, srcs))
    items.sort(key=lambda it: (-it[0], it[1], it[2]))
    rank_load = [0] * W
    held = [set() for _ in range(W)]
    owner = [0] * (E * W)
    for ld, e, _, srcs in items:
        d = min((d for d in range(W) if e not in held[d]), key=lambda d: (rank_load[d], len(held[d]), d))
        rank_load[d] += ld
        held[d].add(e)
        for s in srcs:
            owner[e * W + s] = d
    # A rank that drew no expert (more ranks than replicas) takes a copy of the
    # lightest expert held twice or more, or else one of a rank with several.
    for d in range(W):
        if held[d]:
            continue
        e = min(range(E), key=lambda e: (load[e], e))
        srcs = [s for s in range(W) if owner[e * W + s] != d][:1]
        for s in srcs:
            owner[e * W + s] = d
        held[d].add(e)
    return owner


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (any torch.distributed backend)."""
    import torch.distributed as dist
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def connect(plan, group=None) -> None:
    """Connects this rank's plan to the others' and meets them, so that no
    rank forwards before every rank has mapped every other's memory."""
    import torch.distributed as dist
    plan.ep_connect(exchange_handles(plan.ep_handle(), group))
    dist.barrier(group)
