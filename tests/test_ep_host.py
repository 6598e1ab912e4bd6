"""Expert-parallel host logic on CPU: token split, expert ownership, the
unique-id exchange over a world-size-2 gloo group, and the decomposition the
library uses at N > 1 (each rank sums the slots it owns in slot order, the
token's rank adds the per-rank partials in rank order, then the shared
expert), checked with the oracle against the one-process layer."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from flash_deepseek_b200 import ep


def test_local_tokens_split():
    assert [ep.local_tokens(64, 8, r) for r in range(8)] == [(8 * r, 8) for r in range(8)]
    assert [ep.local_tokens(1, 8, r) for r in range(8)] == [(0, 1)] + [(1, 0)] * 7
    assert [ep.local_tokens(3, 4, r) for r in range(4)] == [(0, 1), (1, 1), (2, 1), (3, 0)]
    with pytest.raises(ValueError):
        ep.local_tokens(6, 4, 0)
    with pytest.raises(ValueError):
        ep.local_tokens(4, 2, 2)


def test_expert_owner_and_hits():
    assert ep.expert_owner(np.arange(256), 256, 8).tolist() == sorted(list(range(8)) * 32)
    idx = np.array([[0, 31, 32, 255], [33, 34, 0, 200]])
    assert ep.experts_hit(idx, 256, 8, 0) == [0, 31]
    assert ep.experts_hit(idx, 256, 8, 1) == [32, 33, 34]
    assert ep.experts_hit(idx, 256, 8, 7) == [255]
    assert ep.experts_hit(idx, 256, 8, 3) == []
    with pytest.raises(ValueError):
        ep.expert_owner(3, 10, 4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        uid = ep.share_unique_id(dist, rank, lambda: bytes(range(128)))
        # the decomposition: routing and expert outputs are stand-ins here
        # (random); only the summation structure is under test
        rng = np.random.default_rng(5)
        E, K, H, T = 16, 4, 64, 3
        idx = np.stack([rng.permutation(E)[:K] for _ in range(T * world)]).astype(np.int32)
        w = rng.random((T * world, K)).astype(np.float32)
        eo = rng.standard_normal((T * world, K, H)).astype(np.float32)
        shared = rng.standard_normal((T * world, H)).astype(np.float32)
        own = ep.expert_owner(idx, E, world) == rank
        part = np.zeros((T * world, H), np.float32)
        for t in range(T * world):
            for k in range(K):  # slot order
                if own[t, k]:
                    part[t] += w[t, k] * eo[t, k]
        import torch
        parts = [torch.zeros(T * world, H) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        t0, n = ep.local_tokens(T * world, world, rank)
        out = np.zeros((n, H), np.float32)
        for r in range(world):  # rank order
            out += parts[r].numpy()[t0:t0 + n]
        out += shared[t0:t0 + n]
        full = np.zeros((n, H), np.float32)
        for t in range(n):
            for k in range(K):
                full[t] += w[t0 + t, k] * eo[t0 + t, k]
        full += shared[t0:t0 + n]
        err = float(np.max(np.abs(out - full)) / np.max(np.abs(full)))
        dist.destroy_process_group()
        q.put((rank, uid, err, None))
    except Exception as e:
        q.put((rank, None, None, repr(e)))


def test_gloo_world2_uid_and_decomposition():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, uid, err, exc = q.get(timeout=120)
            assert exc is None, exc
            res[rank] = (uid, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    assert res[0][0] == res[1][0] == bytes(range(128))
    for rank in (0, 1):
        assert res[rank][1] < 1e-6, res[rank]


def test_ep_decomposition_matches_oracle_layer(oracle):
    """Per-rank pre-combine + rank-order sum over real oracle expert outputs
    equals the one-process layer within the summation-order tolerance."""
    O = oracle
    H, I, E, K, dt = 256, 256, 8, 4, 12
    cfg = dict(H=H, I=I, n_experts=E, n_group=4, topk_group=2, K=K, routed_scale=2.5, down_type=dt)
    blobs = {e: O.gen_expert(3, 0, e, H, I, dt) for e in range(E + 1)}
    router = O.normal(3, O.stream(0, 0, O.KIND_ROUTER), E * H, 0.05).reshape(E, H)
    bias = O.normal(3, O.stream(0, 0, O.KIND_BIAS), E, 0.01)
    x = O.normal(4, O.stream(0, 0, O.KIND_ACT), 4 * H, 1.0).reshape(4, H)
    full, idx, w, _ = O.moe_layer(cfg, blobs, router, bias, x, acc_double=False)
    world = 2
    eo = {(t, e): O.expert_forward(blobs[e], H, I, dt, x[t], acc_double=False) for t in range(4) for e in idx[t]}
    sh = np.stack([O.expert_forward(blobs[E], H, I, dt, x[t], acc_double=False) for t in range(4)])
    out = np.zeros_like(full)
    for t in range(4):
        for r in range(world):
            part = np.zeros(H, np.float32)
            for k in range(K):
                if ep.expert_owner(idx[t, k], E, world) == r:
                    part += w[t, k] * eo[(t, int(idx[t, k]))]
            out[t] += part
        out[t] += sh[t]
    err = float(np.max(np.abs(out - full)) / np.max(np.abs(full)))
    assert err < 1e-5, err


def _watch_rank(rank, world, port, mode, q):
    """Three good steps, then rank 1 fails in `mode`: "exit" (dies without a
    word), "raise" (an exception, handled by leaving) or "late" (arrives
    after the timeout)."""
    try:
        import time
        from datetime import timedelta
        from torch.distributed import TCPStore
        store = TCPStore("127.0.0.1", port, world, rank == 0, timedelta(seconds=30))
        w = ep.PeerWatch(store, rank, world, timeout=3.0)
        for step in range(3):
            w.beat(step)
            w.wait(step)
        if rank == 1:
            if mode == "exit":
                q.put((rank, "exited", 0.0))
                q.close()
                q.join_thread()   # the message is out before the process dies
                os._exit(0)
            if mode == "raise":
                try:
                    raise RuntimeError("planted failure")
                except RuntimeError:
                    w.leave()
                q.put((rank, "left", 0.0))
                time.sleep(6)   # keep the store's peer alive while rank 0 checks
                return
            time.sleep(4.5)      # late: past the 3 s timeout
            w.beat(3)
            q.put((rank, "late", 0.0))
            time.sleep(1)
            return
        w.beat(3)
        t0 = time.monotonic()
        try:
            w.wait(3)
            got = "no error"
        except ep.PeerLost as e:
            got = f"lost {e.ranks} left {e.left}"
        q.put((rank, got, time.monotonic() - t0))
        time.sleep(0.5)
    except Exception as e:
        q.put((rank, "EXC " + repr(e), 0.0))


@pytest.mark.parametrize("mode", ["exit", "raise", "late"])
def test_peer_watch_detects_a_lost_rank(mode):
    """Host-side failure detection between steps (no GPU): a rank that dies,
    leaves after an exception, or misses the timeout is reported to the
    others by PeerWatch.wait before their next launch."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watch_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, got, dt = q.get(timeout=120)
            res[rank] = (got, dt)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    got, dt = res[0]
    if mode == "raise":
        assert got == "lost [1] left [1]", got
        assert dt < 2.5, dt      # at once, not after the 3 s timeout (margin for a loaded host)
    else:
        assert got == "lost [1] left []", got
        assert 2.9 < dt < 20, dt


def test_peer_watch_validates_arguments():
    with pytest.raises(ValueError):
        ep.PeerWatch(None, 2, 2)
