"""Expert-parallel group set-up over torch.distributed (one process per GPU of one node).

The batched decode step of every rank computes the experts it owns for the rows of every
rank, reading and writing the other ranks' memory directly (libdismoen_cuda.so maps the
peers' arenas with CUDA IPC).  The host side only has to exchange the 64-byte memory
handles once, in rank order, and join the ranks before the first step:

    group = attach_group(engine, dist)          # torch.distributed initialised (any backend)
    ...  engine.decode_batch(slots, tokens) on every rank, same row count ...
    engine.ep_detach()

Expert ownership (reference layout of the sharded MoE: expert e on GPU e // (E / G)) and
the even split of sequences over ranks are plain functions so they are testable on CPU.
"""
from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class Group:
    rank: int
    world: int


def expert_owner(expert: int, num_experts: int, world: int) -> int:
    """Rank that computes `expert` (contiguous blocks of num_experts / world experts)."""
    if num_experts % world:
        raise ValueError("the world size must divide the number of experts")
    return expert // (num_experts // world)


def rows_of_rank(total_rows: int, rank: int, world: int) -> range:
    """This rank's share of `total_rows` sequences (equal shares: every rank runs the same
    row count through the batched step)."""
    if total_rows % world:
        raise ValueError("the world size must divide the number of sequences")
    per = total_rows // world
    return range(rank * per, (rank + 1) * per)


def gather_handles(handle: bytes, dist) -> list[bytes]:
    """All ranks' handles in rank order (all_gather_object over the default group)."""
    world = dist.get_world_size()
    out: list = [None] * world
    dist.all_gather_object(out, handle)
    return [bytes(h) for h in out]


def attach_group(engine, dist) -> Group:
    """Joins `engine` to the expert-parallel group of the default process group."""
    rank, world = dist.get_rank(), dist.get_world_size()
    handles = gather_handles(engine.ep_ipc_handle(), dist)
    engine.ep_attach(rank, world, handles)
    dist.barrier()  # every rank's barrier flags are reset before anyone signals
    return Group(rank, world)
