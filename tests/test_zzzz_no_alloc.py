"""GPU: moe_route_hidden_noalloc -- routing for callers that cannot allocate
device memory (a fixed memory pool, or a decode loop where cudaMalloc may
synchronize the device) -- gives the same routing as moe_forward, through the
C ABI, at DeepSeek-V3 shapes (above 4 tokens moe_forward's logits come from
the tensor-core router, fp32-accurate in another summation order; these
seeded inputs hold no near tie, so indices match exactly and weights to 1e-6).  Calls follow each other on one shared scratch
array that keeps the last call's contents: 3 tokens (one-pass router kernel,
no scratch), then 5 and 64 tokens (split-K router: partial sums and
completion counters in the array), then 64 tokens again with other inputs.
Collected last on purpose."""
import ctypes as C

import numpy as np
import pytest


@pytest.mark.gpu
def test_route_hidden_noalloc_matches_forward(cuda_lib, oracle):
    import torch
    from flash_deepseek_b200 import MoeConfig, _lib

    cfg = MoeConfig(n_layers=1, max_tokens=64)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=3, down_type=cuda_lib.TYPE_Q6_K)
    O = oracle
    # the synthetic router / bias, regenerated bit-identically on the host
    router = O.normal(3, O.stream(0, 0, O.KIND_ROUTER), cfg.n_experts * cfg.hidden, 0.006)
    bias = O.normal(3, O.stream(0, 0, O.KIND_BIAS), cfg.n_experts, 0.01)
    dev = torch.device("cuda", 0)
    d_router = torch.from_numpy(router).to(dev)
    d_bias = torch.from_numpy(bias).to(dev)
    lib = _lib.load()
    ccfg = cfg.c()
    for call, T in enumerate((3, 5, 64, 64)):
        h = O.normal(40 + call, O.stream(0, 0, O.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
        _, idx_ref, w_ref = m.forward(0, h)          # existing entry point
        d_h = torch.from_numpy(h).to(dev)
        d_idx = torch.full((T, cfg.top_k), -1, dtype=torch.int32, device=dev)
        d_w = torch.zeros((T, cfg.top_k), dtype=torch.float32, device=dev)
        rc = lib.moe_route_hidden_noalloc(C.byref(ccfg), d_router.data_ptr(), d_bias.data_ptr(), d_h.data_ptr(), T,
                                          d_idx.data_ptr(), d_w.data_ptr(), None)
        assert rc == 0
        torch.cuda.synchronize()
        idx, w = d_idx.cpu().numpy(), d_w.cpu().numpy()
        assert np.array_equal(idx, idx_ref), (call, T)
        assert np.allclose(w, w_ref, rtol=1e-6, atol=0), (call, T)
    # sizes beyond the fixed scratch are rejected, not truncated
    big = MoeConfig(n_experts=1024, n_group=8, max_tokens=64).c()
    d_h = torch.zeros((64, cfg.hidden), dtype=torch.float32, device=dev)
    d_idx = torch.zeros((64, 8), dtype=torch.int32, device=dev)
    d_w = torch.zeros((64, 8), dtype=torch.float32, device=dev)
    assert lib.moe_route_hidden_noalloc(C.byref(big), d_router.data_ptr(), None, d_h.data_ptr(), 64,
                                        d_idx.data_ptr(), d_w.data_ptr(), None) != 0
    m.close()
