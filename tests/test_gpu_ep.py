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


def _ep_rank(rank, world, uid, cfg_kw, down_type, batches, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import flash_deepseek_b200 as F
        m = F.MoE(F.MoeConfig(**cfg_kw), device=rank, rank=rank, world_size=world, unique_id=uid)
        m.init_layer_synthetic(0, seed=SEED, down_type=down_type)
        res = [m.forward(0, h) for h in batches[rank]]
        m.close()
        q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def run_ranks(cuda_lib, cfg, down_type, batches, world=2, timeout=240):
    uid = cuda_lib.get_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    kw = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, n_experts=cfg.n_experts, n_group=cfg.n_group,
              topk_group=cfg.topk_group, top_k=cfg.top_k, n_layers=cfg.n_layers, max_tokens=cfg.max_tokens)
    procs = [ctx.Process(target=_ep_rank, args=(r, world, uid, kw, down_type, batches, q)) for r in range(world)]
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

