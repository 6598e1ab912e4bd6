"""CPU: pins the oracle (the checker) against the reference's own outputs --
golden fixtures made by tests/golden/make_golden.py from gguf-py and from the
reference's quant.c / route() built in place -- and, where the reference
build is present, against it directly."""
import ctypes as C
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def gold(name):
    return np.load(os.path.join(GOLD, name))


def test_fp16_all_patterns(oracle):
    t = gold("fp16_table.npz")["bits"]
    L = oracle.lib()
    mine = np.array([L.or_fp16_to_fp32(h) for h in range(65536)], np.float32).view(np.uint32)
    assert np.array_equal(mine, t)


@pytest.mark.parametrize("name,qtype", [("dequant_q4k.npz", 12), ("dequant_q6k.npz", 14)])
def test_dequant_golden(oracle, name, qtype):
    g = gold(name)
    blocks, exp = g["blocks"], g["expected"]
    got = oracle.dequant(blocks.reshape(-1), qtype, exp.size).reshape(exp.shape)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref", "libref_moe.so")),
                    reason="reference build not present")
@pytest.mark.parametrize("qtype,bsz", [(12, 144), (14, 210)])
def test_dequant_vs_reference_random(oracle, qtype, bsz):
    rng = np.random.default_rng(qtype)
    b = rng.integers(0, 256, size=(4096, bsz), dtype=np.uint8)
    off = 0 if qtype == 12 else 208
    b[:, off:off + 2] = (rng.standard_normal(4096) * 1e-2).astype(np.float16).view(np.uint8).reshape(-1, 2)
    a = oracle.dequant(b.reshape(-1), qtype, 4096 * 256)
    r = oracle.ref_dequant(b.reshape(-1), qtype, 4096 * 256)
    assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


def test_route_golden(oracle):
    g = gold("route_golden.npz")
    for i in range(len(g["logits"])):
        idx, w = oracle.route(g["logits"][i], g["bias"][i])
        assert np.array_equal(idx, g["idx"][i]), i
        assert np.array_equal(w.view(np.uint32), g["w"][i].view(np.uint32)), i


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref", "libref_moe.so")),
                    reason="reference build not present")
def test_route_vs_reference_random(oracle):
    rng = np.random.default_rng(7)
    for _ in range(500):
        lg = (rng.standard_normal(256) * rng.uniform(0.1, 4)).astype(np.float32)
        b = (rng.standard_normal(256) * 0.01).astype(np.float32)
        i1, w1 = oracle.route(lg, b)
        i2, w2 = oracle.ref_route(lg, b)
        assert np.array_equal(i1, i2) and np.array_equal(w1.view(np.uint32), w2.view(np.uint32))


def test_activation_golden(oracle):
    g = gold("act_golden.npz")
    L = oracle.lib()
    o = np.empty_like(g["g"])
    L.or_silu_mul(g["g"], g["u"], o, o.size)
    assert np.array_equal(o.view(np.uint32), g["silu"].view(np.uint32))
    x, nw = g["x"], g["norm_w"]
    r = np.empty_like(x)
    L.or_rms_norm(x, nw.ctypes.data, r, r.size, 1e-6)
    assert np.array_equal(r.view(np.uint32), g["rms"].view(np.uint32))
    s = np.array([L.or_sigmoidf(float(v)) for v in g["sig_in"]], np.float32)
    assert np.array_equal(s.view(np.uint32), g["sig"].view(np.uint32))


def test_synth_golden(oracle):
    g = gold("synth_golden.npz")
    O = oracle
    assert np.array_equal(O.gen_matrix(0, O.stream(0, 0, O.KIND_GATE), O.TYPE_Q4_K, 1, 1024, 0.02), g["gate_q4k"])
    assert np.array_equal(O.gen_matrix(0, O.stream(0, 0, O.KIND_DOWN), O.TYPE_Q6_K, 1, 1024, 0.02), g["down_q6k"])
    assert np.array_equal(O.normal(0, O.stream(0, 0, O.KIND_ROUTER), 64, 0.006).view(np.uint32),
                          g["router"].view(np.uint32))


def test_generator_statistics(oracle):
    x = oracle.normal(0, oracle.stream(1, 2, 3), 400000, 0.02)
    assert abs(x.mean()) < 2e-4 and abs(x.std() - 0.02) < 2e-4
    y = oracle.normal(0, oracle.stream(1, 2, 4), 400000, 0.02)
    assert abs(np.corrcoef(x, y)[0, 1]) < 0.01
    z = oracle.normal(1, oracle.stream(1, 2, 3), 400000, 0.02)
    assert not np.array_equal(x, z)
    # deterministic and position-addressable
    part = oracle.normal(0, oracle.stream(1, 2, 3), 1000, 0.02, first=5000)
    assert np.array_equal(part, x[5000:6000])


def test_det_log(oracle):
    L = oracle.lib()
    for s in np.concatenate([np.linspace(1e-12, 1.0, 997), [2.0 ** -62, 0.5, 0.7071067811865476]]):
        assert abs(L.or_det_log(float(s)) - np.log(s)) <= 4e-16 * max(1.0, abs(np.log(s)))


@pytest.mark.parametrize("qtype", [12, 14])
def test_quantizer_roundtrip(oracle, qtype):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(256 * 512) * 0.02).astype(np.float32)
    x[:256] = 0.0                      # all-zero super-block
    x[256:512] = np.abs(x[256:512])    # all positive (min clamps to 0)
    q = oracle.quantize(x, qtype)
    y = oracle.dequant(q, qtype, x.size)
    assert np.all(y[:256] == 0.0)
    rel = np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < (0.1 if qtype == 12 else 0.03), rel
    # every reconstructed value is within one quantization step of the input
    blocks = x.reshape(-1, 256)
    err = np.abs(y - x).reshape(-1, 256).max(axis=1)
    span = blocks.max(axis=1) - np.minimum(blocks.min(axis=1), 0)
    assert np.all(err <= span / 4 + 1e-6)


def test_expert_forward_precision_variants(oracle):
    """fp32 and fp64 accumulation of the oracle agree far inside the 2e-3
    tolerance: the tolerance covers summation order only."""
    H, I = 512, 512
    O = oracle
    blob = O.gen_expert(0, 0, 0, H, I, O.TYPE_Q4_K)
    x = O.normal(0, O.stream(0, 0, O.KIND_ACT), H, 1.0)
    a = O.expert_forward(blob, H, I, O.TYPE_Q4_K, x, acc_double=True)
    b = O.expert_forward(blob, H, I, O.TYPE_Q4_K, x, acc_double=False)
    assert np.max(np.abs(a - b)) / np.max(np.abs(a)) < 1e-5


@pytest.mark.parametrize("down_type", [12, 14])
def test_grouped_layer_equals_per_token_layer(oracle, down_type):
    """moe_layer_given (rows dequantized once per expert, all of its tokens
    at once) is the per-token or_moe_layer restatement, bit for bit."""
    O = oracle
    H, I, E, K = 512, 256, 8, 3
    cfg = dict(H=H, I=I, n_experts=E, n_group=4, topk_group=2, K=K, routed_scale=2.5, down_type=down_type)
    experts = {e: O.gen_expert(5, 0, e, H, I, down_type) for e in range(E + 1)}
    router = O.normal(5, O.stream(0, 0, O.KIND_ROUTER), E * H, 0.05).reshape(E, H)
    x = O.normal(6, O.stream(0, 0, O.KIND_ACT), 7 * H, 1.0).reshape(7, H)
    out, idx, w, _ = O.moe_layer(cfg, experts, router, None, x)
    for dbl in (True, False):
        ref, _, _, _ = O.moe_layer(cfg, experts, router, None, x, force_idx=idx, force_w=w, acc_double=dbl)
        got = O.moe_layer_given(cfg, experts, x, idx, w, acc_double=dbl)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_to_f16_pins(oracle):
    """dequant_tensor_f16 (infer.m:314-348, 519-538): the fp32 value of each
    GGUF type, rounded to fp16 to nearest even -- against numpy's float16
    cast (IEEE RNE, subnormals and overflow included) and the gguf-py
    golden dequant of the Q4_K / Q6_K blocks."""
    rng = np.random.default_rng(4)
    v = np.concatenate([rng.standard_normal(4096) * s for s in (1e-7, 1e-4, 1.0, 3e4, 1e5)]).astype(np.float32)
    assert np.array_equal(oracle.to_f16(v, oracle.TYPE_F32, v.size), v.astype(np.float16).view(np.uint16))
    bf = (v.view(np.uint32) >> 16).astype(np.uint16)
    want = (bf.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.to_f16(bf, oracle.TYPE_BF16, bf.size), want)
    h = v[(np.abs(v) < 6e4)].astype(np.float16)
    assert np.array_equal(oracle.to_f16(h, oracle.TYPE_F16, h.size), h.view(np.uint16))
    for name, qtype in (("dequant_q4k.npz", oracle.TYPE_Q4_K), ("dequant_q6k.npz", oracle.TYPE_Q6_K)):
        g = gold(name)
        blob, ref = g["blocks"].reshape(-1), g["expected"].reshape(-1)
        n = ref.size
        assert np.array_equal(oracle.to_f16(blob, qtype, n), ref.astype(np.float32).astype(np.float16).view(np.uint16))


def test_dense_ffn_composition(oracle):
    """infer.m:1855-1865 (mv_f16, silu_mul, mv_f16) against a float64 numpy
    composition of the same fp16 weights; silu_mul on the fp32 projections is
    the pinned or_silu_mul."""
    rng = np.random.default_rng(8)
    H, Id, T = 512, 768, 3
    g = (rng.standard_normal((Id, H)) * 0.05).astype(np.float16)
    u = (rng.standard_normal((Id, H)) * 0.05).astype(np.float16)
    d = (rng.standard_normal((H, Id)) * 0.05).astype(np.float16)
    x = rng.standard_normal((T, H)).astype(np.float32)
    out = oracle.dense_ffn(g.view(np.uint16), u.view(np.uint16), d.view(np.uint16), x)
    G = (x.astype(np.float64) @ g.astype(np.float64).T).astype(np.float32)
    U = (x.astype(np.float64) @ u.astype(np.float64).T).astype(np.float32)
    A = np.empty_like(G)
    for t in range(T):
        oracle.lib().or_silu_mul(np.ascontiguousarray(G[t]), np.ascontiguousarray(U[t]), A[t], Id)
    ref = (A.astype(np.float64) @ d.astype(np.float64).T).astype(np.float32)
    assert np.array_equal(out, ref) or float(np.max(np.abs(out - ref)) / np.max(np.abs(ref))) < 1e-6
    y = oracle.mv_f16(g.view(np.uint16), x[0], acc_double=False)
    assert float(np.max(np.abs(y - G[0])) / np.max(np.abs(G[0]))) < 1e-5


def test_sampler_vs_reference(oracle):
    """or_sample_top_p / or_argmax against the reference's own sample_top_p
    and argmax (infer.m:390-456, built in place): the same token and the same
    generator state over many draws, logits without equal probabilities (the
    reference's qsort leaves their order open)."""
    if not oracle.ref_available():
        pytest.skip("reference build not present")
    R = oracle.ref()
    rng = np.random.default_rng(12)
    for n, scale in ((1000, 3.0), (129280, 2.0), (50, 0.5)):
        for trial in range(6):
            lg = (rng.standard_normal(n) * scale).astype(np.float32)
            assert R.ref_argmax(lg, n) == oracle.lib().or_argmax(lg, n)
            for temp, top_p in ((0.6, 0.95), (1.0, 0.5), (0.0, 0.9), (2.0, 1.0)):
                s0 = int(rng.integers(1, 2**32))
                st = C.c_uint32(s0)
                want = R.ref_sample_top_p(lg, n, temp, top_p, C.byref(st))
                tok, s1, _, _ = oracle.sample_top_p(lg, temp, top_p, s0)
                assert (tok, s1) == (want, st.value), (n, trial, temp, top_p)
