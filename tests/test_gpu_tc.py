"""The tcgen05 kernels of the busy experts (chunks of more than 8 tokens,
moe_experts_tc.cu) against the oracle, and against the GEMVs' fp16 path on
the same inputs (MOE_TC=0 at context creation): chunk sizes 9..32 (MMA N =
16 and 32), an expert split into two chunks, Q4_K and Q6_K down matrices,
the shared expert, and the full DeepSeek shape."""
import os

import numpy as np
import pytest

from test_gpu_moe import GUARD, TOL, oracle_cfg, rel_err, small_cfg


def _ctx(cuda_lib, cfg, tc):
    old = os.environ.get("MOE_TC")
    os.environ["MOE_TC"] = "1" if tc else "0"
    try:
        return cuda_lib.MoE(cfg)
    finally:
        if old is None:
            del os.environ["MOE_TC"]
        else:
            os.environ["MOE_TC"] = old


def _busy_routing(T, K, E, rng, busy):
    """Token t goes to every expert e of `busy` = [(e, n)] with t < n, and
    to random other experts (ids past the busy ones) for its remaining slots."""
    nb = len(busy)
    idx = np.zeros((T, K), np.int32)
    for t in range(T):
        mine = [e for e, n in busy if t < n][:K]
        rest = [e for e in rng.permutation(np.arange(nb, E)) if e not in mine]
        idx[t] = (mine + rest)[:K]
    w = rng.uniform(0.1, 1.0, (T, K)).astype(np.float32)
    return idx, w


@pytest.mark.gpu
@pytest.mark.parametrize("down_type,inter", [(12, 512), (14, 2048), (12, 2048)])
def test_tc_chunks_routing_given(cuda_lib, oracle, down_type, inter):
    """Expert 0 takes 40 tokens (two chunks of 20), expert 1 nine (N = 16),
    expert 2 thirty-two (N = 32), expert 3 seventeen; the shared expert 48
    (two chunks of 24)."""
    cfg = small_cfg(intermediate=inter, max_tokens=48)
    H, I, T = cfg.hidden, cfg.intermediate, 48
    rng = np.random.default_rng(17)
    idx, w = _busy_routing(T, cfg.top_k, cfg.n_experts, rng, [(0, 40), (1, 9), (2, 32), (3, 17)])
    h = oracle.normal(5, oracle.stream(0, 3, oracle.KIND_ACT), T * H, 1.0).reshape(T, H)
    outs = {}
    for tc in (1, 0):
        m = _ctx(cuda_lib, cfg, tc)
        m.init_layer_synthetic(0, seed=21, down_type=down_type)
        outs[tc] = (m.experts_forward(0, h, idx, w), m.shared_forward(0, h))
        if tc:
            experts = {e: m.read_expert(0, e) for e in range(cfg.n_experts + 1)}
        m.close()
    ref = np.zeros((T, H), np.float32)
    sd = np.zeros((T, H), np.float32)
    for t in range(T):
        for k in range(cfg.top_k):
            ref[t] += w[t, k] * oracle.expert_forward(experts[int(idx[t, k])], H, I, down_type, h[t])
        sd[t] = oracle.expert_forward(experts[cfg.n_experts], H, I, down_type, h[t])
    e_tc, e_sd = rel_err(outs[1][0], ref), rel_err(outs[1][1], sd)
    assert e_tc < TOL and e_tc < GUARD, e_tc
    assert e_sd < TOL and e_sd < GUARD, e_sd
    # the two engines differ in summation order only
    assert rel_err(outs[1][0], outs[0][0]) < 1e-5
    assert rel_err(outs[1][1], outs[0][1]) < 1e-5
    rows = [rel_err(outs[1][0][t], ref[t]) for t in range(T)]
    assert max(rows) < 10 * GUARD, max(rows)


@pytest.mark.gpu
def test_tc_full_size_hot_experts(cuda_lib, oracle):
    """DeepSeek shapes, routing given: 64 tokens, the first four experts take
    64, 33, 20 and 9 of them (chunks 32 + 32, 17 + 16, 20, 9), the shared
    expert all 64; every output row against the oracle."""
    import torch
    cfg = cuda_lib.MoeConfig(n_layers=1, max_tokens=64)
    H, T, K, E = cfg.hidden, 64, cfg.top_k, cfg.n_experts
    idx, w = _busy_routing(T, K, E, np.random.default_rng(3), [(0, 64), (1, 33), (2, 20), (3, 9)])
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=0, down_type=14)
    h = torch.randn(T, H, generator=torch.Generator().manual_seed(11)).numpy()
    out = m.experts_forward(0, h, idx, w)
    sd = m.shared_forward(0, h)
    experts = {e: m.read_expert(0, e) for e in sorted(set(idx.reshape(-1).tolist())) + [E]}
    ref = oracle.moe_layer_given(oracle_cfg(cfg, 14), experts, h, idx, w)  # includes the shared expert
    e = rel_err(out + sd, ref)
    assert e < TOL and e < GUARD, e
    m.close()
