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


PREFILL_TOL = 2e-3   # north-star bound; fp16 weights and activations, fp32 accumulation


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [12, 14])
def test_prefill_matches_oracle(cuda_lib, oracle, down_type):
    from test_gpu_moe import check_routing, oracle_layer, rel_err, router_of, small_cfg
    cfg = small_cfg(intermediate=2048 if down_type == 14 else 512)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(0, seed=11, down_type=down_type)
    router, bias = router_of(oracle, 11, 0, cfg)
    T = 300   # the shared expert spans three 128-pair tiles
    h = oracle.normal(4, oracle.stream(0, 0, oracle.KIND_ACT), T * cfg.hidden, 1.0).reshape(T, cfg.hidden)
    out, idx, w = m.prefill(0, h)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(oracle, cfg, logits, bias, idx, w)
    ref = oracle_layer(oracle, m, cfg, 0, down_type, h, idx, w, router, bias)
    e = rel_err(out, ref)
    assert e < PREFILL_TOL, e
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
