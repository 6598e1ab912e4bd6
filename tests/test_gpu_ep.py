"""Expert parallelism over NCCL (2 GPUs): each rank holds n_experts / world
routed experts plus the replicated router and shared expert, its tokens go
to the owning ranks in the dispatch exchange and come back weighted in the
combine exchange.  Every rank's output is checked against the oracle on the
same tokens, with ragged and empty batches on one rank.

Skipped with fewer than 2 GPUs.  The ranks are child processes started with
`spawn`; NVLink SHARP stays off (NCCL_NVLS_ENABLE=0) so a rank that dies
cannot leave a multicast object bound on its peer.
"""
import multiprocessing as mp
import os
import subprocess

import numpy as np
import pytest

from test_gpu_moe import GUARD, TOL, check_routing, oracle_cfg, rel_err, router_of, small_cfg

SEED = 21


def _gpu_count() -> int:
    try:
        r = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=30)
        return sum(1 for ln in r.stdout.splitlines() if ln.startswith("GPU "))
    except Exception:
        return 0


def _load_shard(F, O, m, cfg_kw, down_type):
    """This rank's slice of the stacked expert tensors (the bytes a host
    would pread at moe_shard_range's offset), loaded with
    moe_load_layer_shard; the weights are the synthetic layer's, made on the
    host by the oracle's generator."""
    H, I, E = cfg_kw["hidden"], cfg_kw["intermediate"], cfg_kw["n_experts"]
    gb, db = O.row_bytes(12, H) * I, O.row_bytes(down_type, I) * H
    off, nbytes = m.shard_range(gb)
    e0, n = off // gb, nbytes // gb
    assert m.shard_range(db) == (e0 * db, n * db) and n == E // m.lib.moe_world_size(m.ctx)
    blobs = [O.gen_expert(SEED, 0, e, H, I, down_type) for e in range(e0, e0 + n)]
    sh = O.gen_expert(SEED, 0, E, H, I, down_type)
    router = O.normal(SEED, O.stream(0, 0, O.KIND_ROUTER), E * H, 0.006).reshape(E, H)
    bias = O.normal(SEED, O.stream(0, 0, O.KIND_BIAS), E, 0.01)
    m.load_layer_shard(0, np.concatenate([b[:gb] for b in blobs]), np.concatenate([b[gb:2 * gb] for b in blobs]),
                       np.concatenate([b[2 * gb:] for b in blobs]), down_type, router, bias, sh[:gb], sh[gb:2 * gb],
                       sh[2 * gb:], down_type)


def _ep_rank(rank, world, uid, cfg_kw, down_type, batches, q, mode="synthetic"):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import flash_deepseek_b200 as F
        m = F.MoE(F.MoeConfig(**cfg_kw), device=rank, rank=rank, world_size=world, unique_id=uid)
        if mode == "shard":
            from oracle import oracle as O
            _load_shard(F, O, m, cfg_kw, down_type)
        else:
            m.init_layer_synthetic(0, seed=SEED, down_type=down_type)
        if mode == "graph":
            # device-pointer steps on the same buffers: the first runs directly,
            # the second is captured, the rest replay the graph; the step
            # number the peer exchange needs lives in device memory
            import torch
            torch.cuda.set_device(rank)
            res = []
            for h in batches[rank]:
                d_h = torch.from_numpy(h).cuda(rank) if h.shape[0] else torch.empty(1, h.shape[1], device=rank)
                d_out = torch.empty_like(d_h)
                d_idx = torch.empty(max(1, h.shape[0]), cfg_kw["top_k"], dtype=torch.int32, device=rank)
                d_w = torch.empty(max(1, h.shape[0]), cfg_kw["top_k"], dtype=torch.float32, device=rank)
                outs = []
                for _ in range(5):
                    m.forward_device(0, d_h, h.shape[0], d_out, d_idx=d_idx, d_w=d_w)
                    torch.cuda.synchronize(rank)
                    outs.append(d_out[:h.shape[0]].cpu().numpy().copy())
                m.check_error()
                for o in outs[1:]:
                    assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32)), "graph replay differs"
                res.append((outs[-1], d_idx[:h.shape[0]].cpu().numpy(), d_w[:h.shape[0]].cpu().numpy()))
        else:
            res = [m.forward(0, h) for h in batches[rank]]
        m.close()
        q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def run_ranks(cuda_lib, cfg, down_type, batches, world=2, timeout=240, mode="synthetic"):
    uid = cuda_lib.get_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    kw = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, n_experts=cfg.n_experts, n_group=cfg.n_group,
              topk_group=cfg.topk_group, top_k=cfg.top_k, n_layers=cfg.n_layers, max_tokens=cfg.max_tokens)
    procs = [ctx.Process(target=_ep_rank, args=(r, world, uid, kw, down_type, batches, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=timeout)
            assert err is None, f"rank {rank}: {err}"
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    return got


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [12, 14])
def test_ep2_matches_oracle(cuda_lib, oracle, down_type):
    if _gpu_count() < 2:
        pytest.skip("expert parallelism needs 2 GPUs")
    cfg = small_cfg(intermediate=2048 if down_type == 14 else 512)
    H, E = cfg.hidden, cfg.n_experts
    O = oracle

    def toks(strm, T):
        return O.normal(strm, O.stream(0, 0, O.KIND_ACT), max(T, 1) * H, 1.0)[:T * H].reshape(T, H)

    # step 0: ragged (5 and 2 tokens); step 1: rank 1 has no tokens; step 2: full batches
    batches = {0: [toks(100, 5), toks(101, 3), toks(102, cfg.max_tokens)],
               1: [toks(200, 2), toks(201, 0), toks(202, cfg.max_tokens)]}
    got = run_ranks(cuda_lib, cfg, down_type, batches)
    check_ranks(O, cfg, down_type, batches, got)


@pytest.mark.gpu
def test_ep2_graph_replay_matches_oracle(cuda_lib, oracle):
    """The peer-memory EP step replayed as a CUDA graph (device buffers, five
    steps per batch, bit-identical every time), a rank without tokens
    included, against the oracle."""
    if _gpu_count() < 2:
        pytest.skip("expert parallelism needs 2 GPUs")
    cfg = small_cfg()
    H, O = cfg.hidden, oracle
    toks = lambda strm, T: O.normal(strm, O.stream(0, 0, O.KIND_ACT), max(T, 1) * H, 1.0)[:T * H].reshape(T, H)
    batches = {0: [toks(300, 6), toks(301, 4)], 1: [toks(400, 3), toks(401, 0)]}
    got = run_ranks(cuda_lib, cfg, 14, batches, mode="graph")
    check_ranks(O, cfg, 14, batches, got)


@pytest.mark.gpu
def test_ep2_shard_loader_matches_oracle(cuda_lib, oracle):
    """moe_load_layer_shard: each rank loads only its slice of the stacked
    expert tensors (the byte range moe_shard_range gives); the outputs match
    the oracle on the same weights."""
    if _gpu_count() < 2:
        pytest.skip("expert parallelism needs 2 GPUs")
    cfg = small_cfg()
    H, O = cfg.hidden, oracle
    toks = lambda strm, T: O.normal(strm, O.stream(0, 0, O.KIND_ACT), max(T, 1) * H, 1.0)[:T * H].reshape(T, H)
    batches = {0: [toks(500, 5)], 1: [toks(600, 4)]}
    got = run_ranks(cuda_lib, cfg, 14, batches, mode="shard")
    check_ranks(O, cfg, 14, batches, got)


def check_ranks(O, cfg, down_type, batches, got):
    """every rank's output of every step against the oracle layer on its tokens"""
    H, E = cfg.hidden, cfg.n_experts
    router, bias = router_of(O, SEED, 0, cfg)
    blobs = {}
    for rank in sorted(batches):
        for step, h in enumerate(batches[rank]):
            out, idx, w = got[rank][step]
            if h.shape[0] == 0:
                assert out.shape == (0, H)
                continue
            logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
            check_routing(O, cfg, logits, bias, idx, w)
            for e in set(idx.reshape(-1).tolist()) | {E}:
                if e not in blobs:
                    blobs[e] = O.gen_expert(SEED, 0, e, H, cfg.intermediate, down_type)
            ref, _, _, _ = O.moe_layer(oracle_cfg(cfg, down_type), blobs, router, bias, h, force_idx=idx, force_w=w)
            err = rel_err(out, ref)
            assert err < TOL and err < GUARD, (rank, step, err)


def _ep_prefill_rank(rank, world, uid, cfg_kw, down_type, batches, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import flash_deepseek_b200 as F
        m = F.MoE(F.MoeConfig(**cfg_kw), device=rank, rank=rank, world_size=world, unique_id=uid)
        m.init_layer_synthetic(0, seed=SEED, down_type=down_type)
        res = [m.prefill(0, h) for h in batches[rank]]
        m.close()
        q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [12, 14])
def test_ep2_prefill_matches_oracle(cuda_lib, oracle, down_type):
    """Expert-parallel prefill (tensor-core GEMMs) at 2 GPUs: ragged token
    counts, then a step where rank 1 has none; every rank's output against the
    oracle within the prefill bound."""
    if _gpu_count() < 2:
        pytest.skip("expert parallelism needs 2 GPUs")
    from test_gpu_prefill import PREFILL_TOL
    cfg = small_cfg(intermediate=2048 if down_type == 14 else 512)
    H, E, O = cfg.hidden, cfg.n_experts, oracle

    def toks(strm, T):
        return O.normal(strm, O.stream(0, 0, O.KIND_ACT), max(T, 1) * H, 1.0)[:T * H].reshape(T, H)

    batches = {0: [toks(300, 300), toks(301, 40)], 1: [toks(400, 170), toks(401, 0)]}
    uid = cuda_lib.get_unique_id()
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    kw = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, n_experts=cfg.n_experts, n_group=cfg.n_group,
              topk_group=cfg.topk_group, top_k=cfg.top_k, n_layers=cfg.n_layers, max_tokens=cfg.max_tokens)
    procs = [ctx.Process(target=_ep_prefill_rank, args=(r, 2, uid, kw, down_type, batches, qq)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            rank, res, err = qq.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    router, bias = router_of(O, SEED, 0, cfg)
    blobs = {}
    for rank in (0, 1):
        for step, h in enumerate(batches[rank]):
            out, idx, w = got[rank][step]
            if h.shape[0] == 0:
                assert out.shape == (0, H)
                continue
            logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
            check_routing(O, cfg, logits, bias, idx, w)
            for e in set(idx.reshape(-1).tolist()) | {E}:
                if e not in blobs:
                    blobs[e] = O.gen_expert(SEED, 0, e, H, cfg.intermediate, down_type)
            ref, _, _, _ = O.moe_layer(oracle_cfg(cfg, down_type), blobs, router, bias, h, force_idx=idx, force_w=w)
            err = rel_err(out, ref)
            assert err < PREFILL_TOL, (rank, step, err)

