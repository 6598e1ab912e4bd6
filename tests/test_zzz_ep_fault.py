"""GPU failure detection of the expert-parallel decode (2 GPUs), with rank 1
skipping a step: the peer-memory exchange waits for its peers' step flags
with a bounded spin (about 2 s by %globaltimer), so rank 0's call must come
back with the peer-exchange timeout error instead of hanging, and the
context must then refuse further expert-parallel calls (the ranks' step
numbers no longer agree).  No GPU fault is involved: every buffer stays
mapped and in bounds, and rank 1 only frees its memory after rank 0's step
has finished.

The NCCL exchange (used when the peers cannot be mapped) has no bounded wait
of its own, so it is not made to stall here: its host-side poll / abort /
refuse policy is tested on the CPU against fakes (tests/test_wait_policy.py).

Skipped with fewer than 2 GPUs.  The ranks are child processes started with
`spawn`, NVLink SHARP stays off (NCCL_NVLS_ENABLE=0) and the exchange uses
plain peer stores, so a rank that goes away leaves nothing bound on its
peer.  Collected last so that a failure here cannot stop the other GPU
tests."""
import multiprocessing as mp
import os
import time

import pytest

from test_gpu_ep import SEED, _gpu_count
from test_gpu_moe import small_cfg


def _fault_rank(rank, world, uid, cfg_kw, h, q, done):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ.pop("MOE_EP_NCCL", None)
    try:
        import flash_deepseek_b200 as F
        m = F.MoE(F.MoeConfig(**cfg_kw), device=rank, rank=rank, world_size=world, unique_id=uid)
        m.init_layer_synthetic(0, seed=SEED, down_type=F.TYPE_Q6_K)
        if not m.ep_peer_memory:
            # the NCCL exchange has no bounded wait: skipping a step would
            # leave the peer's kernel waiting, so the test does not run it
            m.close()
            q.put((rank, "no peer memory", 0.0))
            return
        m.forward(0, h)  # one step that both ranks take
        if rank == 0:
            t0 = time.monotonic()
            try:
                m.forward(0, h)  # rank 1 does not take this step
                got = "no error"
            except F.MoeError as e:
                got = str(e)
            dt = time.monotonic() - t0
            try:
                m.forward(0, h)  # refused on the host: no kernel is launched
                again = "ran"
            except F.MoeError as e:
                again = str(e)
            done.set()  # rank 0's kernels are finished: rank 1 may free its mailbox
            m.close()
            q.put((rank, (got, again), dt))
        else:
            done.wait(120)
            m.close()
            q.put((rank, "skipped a step", 0.0))
    except Exception as e:  # reported to the parent, which fails the test
        done.set()
        q.put((rank, "EXC " + repr(e), 0.0))


@pytest.mark.gpu
def test_peer_exchange_wait_times_out_when_a_rank_skips_a_step(cuda_lib, oracle):
    if _gpu_count() < 2:
        pytest.skip("expert parallelism needs 2 GPUs")
    cfg = small_cfg()
    H = cfg.hidden
    h = oracle.normal(7, oracle.stream(0, 0, oracle.KIND_ACT), 4 * H, 1.0).reshape(4, H)
    uid = cuda_lib.get_unique_id()
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    kw = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, n_experts=cfg.n_experts, n_group=cfg.n_group,
              topk_group=cfg.topk_group, top_k=cfg.top_k, n_layers=cfg.n_layers, max_tokens=cfg.max_tokens)
    procs = [ctx.Process(target=_fault_rank, args=(r, 2, uid, kw, h, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            rank, msg, dt = q.get(timeout=240)
            got[rank] = (msg, dt)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    if "no peer memory" in (got[0][0], got[1][0]):
        pytest.skip("the peer mappings were refused; the NCCL exchange has no bounded wait")
    assert got[1][0] == "skipped a step", got
    (msg, again), dt = got[0]
    assert "peer exchange wait timed out" in msg, msg
    assert "out of step" in again, again
    assert dt < 60, dt  # two bounded waits of ~2 s each, plus the step
