"""CPU: the oracle's restatement of MLA attention (infer.m:545-903), the next
component after the FFN halves of a decoder layer.  Its pieces are pinned to
the reference's own functions, extracted from infer.m and built in place
(yarn_init_once / yarn_freq / apply_rope_q / apply_rope_k, softmax); the
whole decode step (RMSNorm, q_a / q_b and kv_a projections, interleaved YaRN
RoPE, the latent cache, absorbed attention with k_b and v_b, o_proj and the
residual) is checked against a float64 numpy composition over several
positions of a growing cache."""
import ctypes as C

import numpy as np
import pytest


def _ref(oracle):
    if not oracle.ref_available():
        pytest.skip("reference build not present")
    return oracle.ref()


def test_yarn_band_and_frequencies_match_reference(oracle):
    R = _ref(oracle)
    cfg = oracle.mla_cfg()
    lo, hi, rlo, rhi = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    oracle.lib().or_yarn_band(C.byref(cfg), C.byref(lo), C.byref(hi))
    R.ref_yarn_band(C.byref(rlo), C.byref(rhi))
    assert (lo.value, hi.value) == (rlo.value, rhi.value) == (10, 23)
    for i in range(cfg.qk_rope // 2):
        a = np.float32(oracle.lib().or_yarn_freq(C.byref(cfg), i))
        b = np.float32(R.ref_yarn_freq(i))
        assert a.view(np.uint32) == b.view(np.uint32), i


@pytest.mark.parametrize("pos", [0, 1, 7, 4095, 16000])
def test_rope_matches_reference(oracle, pos):
    R = _ref(oracle)
    cfg = oracle.mla_cfg()
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(cfg.n_heads * cfg.qk_rope).astype(np.float32)
    a, b = q.copy(), q.copy()
    oracle.lib().or_rope(C.byref(cfg), a, cfg.n_heads, pos)
    R.ref_rope_q(b, cfg.n_heads, pos)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    k = rng.standard_normal(cfg.qk_rope).astype(np.float32)
    a, b = k.copy(), k.copy()
    oracle.lib().or_rope(C.byref(cfg), a, 1, pos)
    R.ref_rope_k(b, pos)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_softmax_matches_reference(oracle):
    R = _ref(oracle)
    rng = np.random.default_rng(1)
    for n in (1, 5, 300, 4096):
        x = (rng.standard_normal(n) * 4).astype(np.float32)
        a, b = x.copy(), x.copy()
        oracle.lib().or_softmax(a, n)
        R.ref_softmax(b, n)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n


def _weights(cfg, rng):
    def f16(*shape, s=0.05):
        return (rng.standard_normal(shape) * s).astype(np.float16).view(np.uint16)
    QK = cfg.qk_nope + cfg.qk_rope
    return dict(q_a=f16(cfg.q_lora, cfg.H), q_b=f16(cfg.n_heads * QK, cfg.q_lora),
                kv_a=f16(cfg.kv_lora + cfg.qk_rope, cfg.H), k_b=f16(cfg.n_heads, cfg.kv_lora, cfg.qk_nope, s=0.1),
                v_b=f16(cfg.n_heads, cfg.v_head, cfg.kv_lora, s=0.1), o_proj=f16(cfg.H, cfg.n_heads * cfg.v_head),
                attn_norm=(1 + 0.1 * rng.standard_normal(cfg.H)).astype(np.float32),
                q_a_norm=(1 + 0.1 * rng.standard_normal(cfg.q_lora)).astype(np.float32),
                kv_a_norm=(1 + 0.1 * rng.standard_normal(cfg.kv_lora)).astype(np.float32))


def _np_step(oracle, cfg, w, h, ckv, kr, pos):
    """float64 composition of mla_forward; ckv / kr are lists (the cache)."""
    H16 = lambda a: a.view(np.float16).astype(np.float64)   # noqa: E731
    eps = float(cfg.eps)

    def rms(x, g):
        return x / np.sqrt(np.mean(x * x) + eps) * g.astype(np.float64)

    freqs = np.array([oracle.lib().or_yarn_freq(C.byref(cfg), i) for i in range(cfg.qk_rope // 2)], np.float32)
    ang = (np.float32(pos) * freqs).astype(np.float32).astype(np.float64)
    cs, sn = np.cos(ang), np.sin(ang)

    def rope(x):
        x = x.reshape(-1, cfg.qk_rope // 2, 2)
        a, b = x[..., 0].copy(), x[..., 1].copy()
        return np.stack([a * cs - b * sn, a * sn + b * cs], -1).reshape(-1)

    x = h.astype(np.float64)
    normed = rms(x, w["attn_norm"])
    qan = rms(H16(w["q_a"]) @ normed, w["q_a_norm"])
    QK = cfg.qk_nope + cfg.qk_rope
    qf = (H16(w["q_b"]) @ qan).reshape(cfg.n_heads, QK)
    qn, qr = qf[:, :cfg.qk_nope], rope(qf[:, cfg.qk_nope:]).reshape(cfg.n_heads, cfg.qk_rope)
    kva = H16(w["kv_a"]) @ normed
    ckv.append(rms(kva[:cfg.kv_lora], w["kv_a_norm"]))
    kr.append(rope(kva[cfg.kv_lora:]))
    CKV, KR = np.stack(ckv), np.stack(kr)
    ms = 0.1 * np.log(np.float32(cfg.rope_scale)) + 1.0
    scale = ms * ms / np.sqrt(QK)
    kb, vb = H16(w["k_b"]), H16(w["v_b"])
    att = []
    for hd in range(cfg.n_heads):
        qabs = kb[hd] @ qn[hd]
        sc = scale * (CKV @ qabs) + scale * (KR @ qr[hd])
        p = np.exp(sc - sc.max())
        p /= p.sum()
        att.append(vb[hd] @ (p @ CKV))
    return x + H16(w["o_proj"]) @ np.concatenate(att)


@pytest.mark.parametrize("shape", ["small", "deepseek_heads"])
def test_mla_decode_matches_float64_composition(oracle, shape):
    if shape == "small":
        cfg = oracle.mla_cfg(H=256, n_heads=4, q_lora=128, kv_lora=64, qk_nope=32, qk_rope=64, v_head=32)
    else:   # DeepSeek's per-head sizes and rank, fewer heads and a narrower hidden
        cfg = oracle.mla_cfg(H=512, n_heads=8)
    rng = np.random.default_rng(7)
    w = _weights(cfg, rng)
    cache = oracle.MlaCache(cfg, 16)
    ckv, kr = [], []
    for step, pos in enumerate((0, 1, 2, 3, 100, 101)):
        h = rng.standard_normal(cfg.H).astype(np.float32)
        got = oracle.mla_decode(cfg, w, h, cache, pos)
        want = _np_step(oracle, cfg, w, h, ckv, kr, pos)
        assert cache.len == step + 1
        err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
        assert err < 1e-5, (step, err)
        # the cache rows the oracle appended are the composition's
        assert np.max(np.abs(cache.c_kv[step] - ckv[-1])) < 1e-5 * np.max(np.abs(ckv[-1]))
