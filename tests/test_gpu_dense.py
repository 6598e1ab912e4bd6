"""Dense FFN layers (the first layers of DeepSeek-V3, infer.m:1786-1793 and
1852-1868) through the C ABI against the oracle: the fp16 weights the loader
keeps for every GGUF type the reference decodes (bit-exact), the FFN of a
few tokens across the kernels' token passes, DeepSeek-V3's own shape
(hidden 7168, intermediate 18432), and the layer stack with dense and MoE
slots."""
import numpy as np
import pytest

# fp16 weights and fp32 activations as in the reference's mv_f16; fp32
# accumulation against the oracle's fp64 dot: order-only differences
DENSE_TOL = 1e-5


def _matrices(O, H, Id, seed, qtype):
    """Host GGUF bytes of gate [Id x H], up [Id x H], down [H x Id] of `qtype`,
    with the fp16 bits the reference's dequant_tensor_f16 makes of them."""
    rng = np.random.default_rng(seed)
    mats, bits = [], []
    for rows, cols in ((Id, H), (Id, H), (H, Id)):
        v = (rng.standard_normal(rows * cols) * 0.05).astype(np.float32)
        if qtype == O.TYPE_F32:
            blob = v
        elif qtype == O.TYPE_F16:
            blob = v.astype(np.float16)
        elif qtype == O.TYPE_BF16:
            blob = (v.view(np.uint32) >> 16).astype(np.uint16)
        else:
            blob = O.quantize(v, qtype)
        mats.append(blob)
        bits.append(O.to_f16(blob, qtype, rows * cols).reshape(rows, cols))
    return mats, bits


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [0, 1, 30, 12, 14])
def test_dense_load_keeps_reference_fp16(cuda_lib, oracle, qtype):
    from test_gpu_moe import small_cfg
    cfg = small_cfg()
    H, Id = cfg.hidden, 2048
    m = cuda_lib.MoE(cfg)
    mats, bits = _matrices(oracle, H, Id, 3 + qtype, qtype)
    m.load_dense_layer(0, mats[0], qtype, mats[1], qtype, mats[2], qtype, intermediate=Id)
    for which in range(3):
        got = m.read_dense_weight(0, which, Id)
        assert np.array_equal(got, bits[which]), (qtype, which)
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 2, 3, 5, 9, 16])
def test_dense_forward_matches_oracle(cuda_lib, oracle, T):
    """Token counts below, at and across the passes of 4 (gate/up) and 2
    (down) tokens; mixed GGUF types per matrix."""
    from test_gpu_moe import rel_err, small_cfg
    cfg = small_cfg()
    H, Id = cfg.hidden, 2560
    m = cuda_lib.MoE(cfg)
    mats, bits = _matrices(oracle, H, Id, 7, oracle.TYPE_Q4_K)
    m.load_dense_layer(1, mats[0], oracle.TYPE_Q4_K, mats[1], oracle.TYPE_Q4_K, mats[2], oracle.TYPE_Q4_K,
                       intermediate=Id)
    h = oracle.normal(40 + T, oracle.stream(1, 0, oracle.KIND_ACT), T * H, 1.0).reshape(T, H)
    out = m.dense_forward(1, h)
    ref = oracle.dense_ffn(bits[0], bits[1], bits[2], h)
    e = rel_err(out, ref)
    assert e < DENSE_TOL, (T, e)
    m.close()


@pytest.mark.gpu
def test_dense_full_size_matches_oracle(cuda_lib, oracle):
    """DeepSeek-V3's dense layer (hidden 7168, DENSE_INTERMEDIATE 18432) on the
    synthetic generator: sampled rows of the kept fp16 weights against the
    oracle's generator, then the FFN of 2 tokens against the oracle on the
    weights read back."""
    from test_gpu_moe import rel_err
    cfg = cuda_lib.MoeConfig(n_layers=3, max_tokens=4)
    H, Id = cfg.hidden, 18432
    m = cuda_lib.MoE(cfg)
    m.init_dense_synthetic(0, Id, seed=9, w_sigma=0.02)
    W = [m.read_dense_weight(0, k, Id) for k in range(3)]
    kinds = (oracle.KIND_GATE, oracle.KIND_UP, oracle.KIND_DOWN)
    for k in range(3):
        cols = W[k].shape[1]
        for r in (0, 1, W[k].shape[0] // 2, W[k].shape[0] - 1):
            v = oracle.normal(9, oracle.stream(0, cfg.n_experts + 1, kinds[k]), cols, 0.02, first=r * cols)
            assert np.array_equal(W[k][r], oracle.to_f16(v, oracle.TYPE_F32, cols)), (k, r)
    h = oracle.normal(11, oracle.stream(0, 0, oracle.KIND_ACT), 2 * H, 1.0).reshape(2, H)
    out = m.dense_forward(0, h)
    ref = oracle.dense_ffn(W[0], W[1], W[2], h)
    e = rel_err(out, ref)
    assert e < DENSE_TOL, e
    m.close()


@pytest.mark.gpu
def test_stack_with_dense_layers(cuda_lib, oracle):
    """Layers 0-1 dense, layer 2 MoE, in one moe_forward_stack call: per layer
    RMSNorm then hidden += FFN(h_post) (infer.m:1850-1868, 1922)."""
    from test_gpu_moe import oracle_layer, rel_err, router_of, small_cfg
    cfg = small_cfg(n_layers=3)
    H, Id = cfg.hidden, 1536
    m = cuda_lib.MoE(cfg)
    bits = {}
    for L in range(2):
        mats, b = _matrices(oracle, H, Id, 20 + L, oracle.TYPE_F16)
        m.load_dense_layer(L, mats[0], oracle.TYPE_F16, mats[1], oracle.TYPE_F16, mats[2], oracle.TYPE_F16,
                           intermediate=Id)
        bits[L] = b
    m.init_layer_synthetic(2, seed=5, down_type=14)
    norms = []
    for L in range(3):
        nw = (1.0 + 0.1 * oracle.normal(5, oracle.stream(L, 0, oracle.KIND_NORM), H, 1.0)).astype(np.float32)
        m.set_norm_weight(L, nw)
        norms.append(nw)
    T = 3
    h0 = oracle.normal(6, oracle.stream(0, 0, oracle.KIND_ACT), T * H, 1.0).reshape(T, H)
    got = m.forward_stack(0, 3, h0)
    hid = h0.copy()
    for L in range(3):
        post = np.empty_like(hid)
        for t in range(T):
            r = np.empty(H, np.float32)
            oracle.lib().or_rms_norm(np.ascontiguousarray(hid[t]), norms[L].ctypes.data, r, H, 1e-6)
            post[t] = r
        if L < 2:
            hid = hid + oracle.dense_ffn(*bits[L], post)
        else:
            _, idx, w = m.forward(L, post)
            router, bias = router_of(oracle, 5, L, cfg)
            hid = hid + oracle_layer(oracle, m, cfg, L, 14, post, idx, w, router, bias)
    assert rel_err(got, hid) < 1e-4
    # a MoE call on a dense slot is refused, and loading a MoE block frees the dense FFN
    with pytest.raises(cuda_lib.MoeError):
        m.forward(0, post)
    m.init_layer_synthetic(0, seed=5, down_type=12)
    with pytest.raises(cuda_lib.MoeError):
        m.dense_forward(0, post)
    m.close()


@pytest.mark.gpu
def test_dense_shape_errors(cuda_lib, oracle):
    from test_gpu_moe import small_cfg
    cfg = small_cfg()
    m = cuda_lib.MoE(cfg)
    with pytest.raises(cuda_lib.MoeError):
        m.init_dense_synthetic(0, 1000)        # intermediate % 256 != 0
    with pytest.raises(cuda_lib.MoeError):
        m.dense_forward(0, np.zeros((1, cfg.hidden), np.float32))   # not loaded
    with pytest.raises(cuda_lib.MoeError):
        m.load_dense_layer(0, np.zeros(4), 7, np.zeros(4), 7, np.zeros(4), 7, intermediate=256)  # type 7
    m.close()
