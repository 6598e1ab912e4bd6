"""tcgen05 (fifth-generation tensor core) building blocks used by the
prefill GEMMs: a one-CTA fp16 GEMM through tensor memory, with the A tile
written by threads either into 128-byte-swizzled shared memory or straight
into tensor memory, and B loaded by TMA, against an fp32 product of the same
fp16 values; then the prefill path against the oracle."""
import ctypes as C
import os
import subprocess
import tempfile

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def selftest_lib():
    so = os.path.join(tempfile.mkdtemp(), "umma_selftest.so")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                    "-shared", "-Xcompiler", "-fPIC", "-o", so, os.path.join(HERE, "umma_selftest.cu"),
                    "-cudart", "static"], check=True, capture_output=True)
    lib = C.CDLL(so)
    lib.umma_selftest.restype = C.c_int
    lib.umma_selftest.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
    lib.umma_selftest_pair.restype = C.c_int
    lib.umma_selftest_pair.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
    return lib


@pytest.mark.gpu
@pytest.mark.parametrize("a_in_tmem", [0, 1])
def test_umma_f16_gemm_selftest(selftest_lib, a_in_tmem):
    import torch
    g = torch.Generator().manual_seed(3)
    A = torch.randn(128, 256, generator=g).half()
    B = torch.randn(128, 256, generator=g).half()
    dA, dB = A.cuda(), B.cuda()
    dC = torch.zeros(128, 128, device="cuda")
    rc = selftest_lib.umma_selftest(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), a_in_tmem)
    assert rc == 0, rc
    ref = A.double() @ B.double().T
    err = float((dC.cpu().double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-5, err


@pytest.mark.gpu
@pytest.mark.parametrize("N,dcol,acol", [(128, 0, 256), (96, 0, 384), (160, 0, 384), (160, 160, 384),
                                         (96, 160, 320)])
def test_umma_pair_selftest(selftest_lib, N, dcol, acol):
    """The CTA-pair MMA (cta_group::2, M = 256, A in tensor memory): each CTA
    holds 128 rows of A and N/2 rows of B and gets its 128 rows of C over all
    N columns; accumulator and A at the column offsets the prefill GEMM uses."""
    import torch
    g = torch.Generator().manual_seed(5)
    A = torch.randn(256, 256, generator=g).half()
    B = torch.randn(N, 256, generator=g).half()
    dA, dB = A.cuda(), B.cuda()
    dC = torch.zeros(256, N, device="cuda")
    rc = selftest_lib.umma_selftest_pair(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), N, dcol, acol)
    assert rc == 0, rc
    ref = A.double() @ B.double().T
    err = float((dC.cpu().double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-5, err


PREFILL_TOL = 2e-3   # north-star bound; fp16 weights and activations, fp32 accumulation


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [12, 14])
def test_prefill_matches_oracle(cuda_lib, oracle, down_type):
    from test_gpu_moe import check_routing, oracle_layer, rel_err, router_of, small_cfg
    cfg = small_cfg(intermediate=2048 if down_type == 14 else 512)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=11, down_type=down_type)
    router, bias = router_of(oracle, 11, 0, cfg)
    T = 300   # the shared expert spans two tiles of 150 pairs
    h = oracle.normal(4, oracle.stream(0, 0, oracle.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
    out, idx, w = m.prefill(0, h)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx, w)
    ref = oracle_layer(oracle, m, cfg, 0, down_type, h, idx, w, router, bias)
    e = rel_err(out, ref)
    assert e < PREFILL_TOL, e
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 2, 17])
def test_prefill_short_prompts_match_oracle(cuda_lib, oracle, T):
    """Ragged tiny tiles: one to a few pairs per expert, so the pair MMA's N
    (rounded up to 32) is mostly padding and the peer CTA of a pair holds no
    pair of the tile (it loads no activation box); the same call object is
    reused across sizes by the workspace."""
    from test_gpu_moe import check_routing, oracle_layer, rel_err, router_of, small_cfg
    cfg = small_cfg(intermediate=2048)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=13, down_type=14)
    router, bias = router_of(oracle, 13, 0, cfg)
    h = oracle.normal(30 + T, oracle.stream(0, 0, oracle.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
    out, idx, w = m.prefill(0, h)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx, w)
    ref = oracle_layer(oracle, m, cfg, 0, 14, h, idx, w, router, bias)
    e = rel_err(out, ref)
    assert e < PREFILL_TOL, (T, e)
    m.close()


@pytest.mark.gpu
def test_prefill_matches_decode_path_full_size(cuda_lib, oracle):
    """DeepSeek shapes: the tensor-core prefill (tensor-core router with fp16
    hi/lo splits, tcgen05 expert GEMMs) agrees with the exact decode path on
    the same 64 tokens; both routings match the fp64 logits up to near ties."""
    import torch
    from test_gpu_moe import check_routing, router_of
    cfg = cuda_lib.MoeConfig(n_layers=1, max_tokens=64)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=0, down_type=14)
    g = torch.Generator().manual_seed(7)
    h = torch.randn(64, cfg.hidden, generator=g).numpy()
    out_d, idx_d, w_d = m.forward(0, h)
    out_p, idx_p, w_p = m.prefill(0, h)
    router, bias = router_of(oracle, 0, 0, cfg)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx_d, w_d)
    check_routing(oracle, cfg, logits, bias, idx_p, w_p)
    same = np.array([set(a.tolist()) == set(b.tolist()) for a, b in zip(idx_d, idx_p)])
    assert same.mean() > 0.9, same.mean()
    e = float(np.max(np.abs(out_p[same] - out_d[same])) / np.max(np.abs(out_d[same])))
    assert e < PREFILL_TOL, e
    m.close()


@pytest.mark.gpu
def test_prefill_router_logits_accuracy(cuda_lib, oracle):
    """The tensor-core router's routing weights at full size agree with the
    fp64 reference to 1e-6 (the fp32 sgemv's own accuracy)."""
    from test_gpu_moe import check_routing, router_of
    cfg = cuda_lib.MoeConfig(n_layers=1, max_tokens=64)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=3, down_type=14)
    T = 300
    h = oracle.normal(9, oracle.stream(0, 0, oracle.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
    _, idx, w = m.prefill(0, h)
    router, bias = router_of(oracle, 3, 0, cfg)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx, w)
    m.close()


def _prefill_sample(idx, n_experts, rng, per_group=16):
    """Rows that cover the hottest expert's tiles, the coldest experts and the
    batch edges (tile boundaries of the shared expert), plus random rows."""
    counts = np.bincount(idx.reshape(-1), minlength=n_experts)
    hot = int(np.argmax(counts))
    rows = set(np.nonzero((idx == hot).any(axis=1))[0][:per_group].tolist())
    live = np.nonzero(counts)[0]
    for e in live[np.argsort(counts[live])][:per_group]:
        rows.add(int(np.nonzero((idx == e).any(axis=1))[0][0]))
    T = idx.shape[0]
    rows |= {0, 127, 128, T - 1}
    rows |= set(rng.choice(T, per_group, replace=False).tolist())
    return sorted(rows), hot, int(counts[hot])


@pytest.mark.gpu
@pytest.mark.parametrize("down_type,T", [(14, 4096), (12, 2048)])
def test_prefill_full_size_matches_oracle(cuda_lib, oracle, down_type, T):
    """Config 5 at its own shape: DeepSeek-V3 layer (hidden 7168, 256 + 1
    experts, Q4_K gate/up, Q6_K or Q4_K down), 4096 (2048) tokens, so that
    experts average 128 (64) pairs and most fill one tile of up to 160 pairs
    (pair MMA N = 160), the shared expert 26 (13) tiles.  The routing of every
    token against fp64 logits; the outputs of a sample of rows (the hottest
    expert's tokens, the coldest experts' tokens, tile edges, random rows)
    against the oracle on the same routing."""
    from test_gpu_moe import check_routing, oracle_cfg, rel_err, router_of
    cfg = cuda_lib.MoeConfig(n_layers=1, max_tokens=64)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=0, down_type=down_type)
    h = oracle.normal(21, oracle.stream(0, 0, oracle.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
    out, idx, w = m.prefill(0, h)
    router, bias = router_of(oracle, 0, 0, cfg)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx, w)
    rows, hot, n_hot = _prefill_sample(idx, cfg.n_experts, np.random.default_rng(5))
    assert n_hot >= (128 if T >= 4096 else 64)  # the busiest expert fills (or half fills) a tile
    experts = {e: m.read_expert(0, e) for e in sorted(set(idx[rows].reshape(-1).tolist())) + [cfg.n_experts]}
    ref = oracle.moe_layer_given(oracle_cfg(cfg, down_type), experts, h[rows], idx[rows], w[rows])
    e = rel_err(out[rows], ref)
    assert e < PREFILL_TOL, e
    print(f"prefill T={T} down={down_type}: {len(rows)} rows, hottest expert {hot} with {n_hot} pairs, err {e:.2e}")
    m.close()
