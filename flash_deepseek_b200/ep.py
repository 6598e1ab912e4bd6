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


class PeerLost(RuntimeError):
    """A rank stopped taking steps; `ranks` lists the ones that did not arrive."""

    def __init__(self, step: int, ranks: list[int], left: list[int]):
        self.step, self.ranks, self.left = step, ranks, left
        super().__init__(f"step {step}: rank(s) {ranks} did not arrive" + (f" ({left} left)" if left else ""))


class PeerWatch:
    """Host-side liveness of the expert-parallel ranks, checked between steps.

    Every rank calls `beat(step)` before it launches step `step` and
    `wait(step)` before the launch: `wait` returns once every rank has beaten
    `step`, or raises PeerLost naming the ranks that have not within
    `timeout` seconds (or that called `leave()`).  Because the check sits
    before this rank's launches, none of its kernels or exchanges of that
    step are in flight when the failure is seen, and the context can be
    destroyed at once.  `store` is a torch.distributed key-value store
    (TCPStore, FileStore or a process group's store).  The reference runs one
    process and has no counterpart."""

    def __init__(self, store, rank: int, world: int, timeout: float = 5.0, prefix: str = "moe/step"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"bad rank/world {rank}/{world}")
        self.store, self.rank, self.world, self.timeout, self.prefix = store, rank, world, timeout, prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), str(int(step)))

    def leave(self) -> None:
        """A clean exit: the peers' next wait fails at once instead of timing out."""
        self.store.set(self._key(self.rank), "-1")

    def wait(self, step: int) -> None:
        import time
        deadline = time.monotonic() + self.timeout
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            left, still = [], []
            for r in pending:
                k = self._key(r)
                v = int(self.store.get(k)) if self.store.check([k]) else None
                if v == -1:
                    left.append(r)
                elif v is None or v < step:
                    still.append(r)
            if left:
                raise PeerLost(step, sorted(left + still), left)
            if not still:
                return
            if time.monotonic() > deadline:
                raise PeerLost(step, still, [])
            pending = still
            time.sleep(0.001)
