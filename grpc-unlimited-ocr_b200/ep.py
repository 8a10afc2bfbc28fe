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
