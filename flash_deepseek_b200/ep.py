"""Host-side helpers of the expert-parallel layout (one process per GPU).

Routed expert e lives on rank e // (n_experts / world) (whole routing groups
per rank when world divides n_group); the router and the shared expert are
replicated.  A global decode batch is split evenly over the ranks, or, when
it is smaller than the world, one token goes to each of the first B ranks
and the others join the exchanges with none.  The reference has one process
and no counterpart; its MoE call site is infer.m:1878-1923.
"""
from __future__ import annotations

import numpy as np


def local_tokens(batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first global token, token count) of `rank`."""
    if world < 1 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"bad batch/world/rank {batch}/{world}/{rank}")
    if batch >= world:
        if batch % world:
            raise ValueError(f"global batch {batch} does not divide over {world} ranks")
        n = batch // world
        return rank * n, n
    return min(rank, batch), (1 if rank < batch else 0)


def expert_owner(expert, n_experts: int, world: int):
    """Rank holding routed expert `expert` (scalar or array)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    return np.asarray(expert) // (n_experts // world)


def experts_hit(idx_global: np.ndarray, n_experts: int, world: int, rank: int) -> list[int]:
    """Routed experts of `rank` that any token of the global batch selects."""
    idx = np.asarray(idx_global).reshape(-1)
    mine = idx[expert_owner(idx, n_experts, world) == rank]
    return sorted(set(int(e) for e in mine))


def share_unique_id(pg, rank: int, make_id) -> bytes:
    """Rank 0 makes the NCCL unique id (`make_id()`), every rank receives it
    over the host process group `pg` (torch.distributed, any backend)."""
    obj = [make_id() if rank == 0 else None]
    pg.broadcast_object_list(obj, src=0)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("unique id exchange failed")
    return bytes(uid)
