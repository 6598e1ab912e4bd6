"""GPU: the device codec, the Q6_K repack and the device generator are bit
exact with the reference's quant.c (through the oracle pinned to it) and with
the oracle's generator."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.gpu
@pytest.mark.parametrize("name,qtype", [("dequant_q4k.npz", 12), ("dequant_q6k.npz", 14)])
def test_dequant_golden(cuda_lib, name, qtype):
    g = np.load(os.path.join(GOLD, name))
    blocks, exp = g["blocks"], g["expected"]
    fn = cuda_lib.dequantize_row_q6_K if qtype == 14 else cuda_lib.dequantize_row_q4_K
    got = fn(blocks.reshape(-1), exp.size).reshape(exp.shape)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("qtype,bsz", [(12, 144), (14, 210)])
def test_dequant_random(cuda_lib, oracle, qtype, bsz):
    rng = np.random.default_rng(100 + qtype)
    n = 8192
    b = rng.integers(0, 256, size=(n, bsz), dtype=np.uint8)
    off = 0 if qtype == 12 else 208
    b[:, off:off + 2] = (rng.standard_normal(n) * 1e-2).astype(np.float16).view(np.uint8).reshape(-1, 2)
    fn = cuda_lib.dequantize_row_q6_K if qtype == 14 else cuda_lib.dequantize_row_q4_K
    got = fn(b.reshape(-1), n * 256)
    exp = oracle.dequant(b.reshape(-1), qtype, n * 256)
    # random dmin bytes include NaN halves; NaN payloads are not compared
    nan = np.isnan(exp)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), exp[~nan].view(np.uint32))


@pytest.mark.gpu
def test_fp16_all_patterns_via_q6k(cuda_lib):
    """d of a Q6_K block with sc = 1 and q = 1 dequantizes to fp16_to_fp32(d)
    exactly: covers all 65536 half patterns (NaN payloads excepted)."""
    t = np.load(os.path.join(GOLD, "fp16_table.npz"))["bits"].view(np.float32)
    n = 65536
    b = np.zeros((n, 210), np.uint8)
    b[:, 0:128] = 0x11      # low nibbles 1
    b[:, 128:192] = 0xAA    # high bits 2 -> q6 = 1 + 32 -> q = 1
    b[:, 192:208] = 1
    b[:, 208:210] = np.arange(n, dtype=np.uint16).view(np.uint8).reshape(n, 2)
    got = cuda_lib.dequantize_row_q6_K(b.reshape(-1), n * 256).reshape(n, 256)[:, 0]
    nan = np.isnan(t)
    assert np.array_equal(got[~nan].view(np.uint32), t[~nan].view(np.uint32))
    assert np.all(np.isnan(got[nan]))


def small_cfg(**kw):
    from flash_deepseek_b200 import MoeConfig
    base = dict(hidden=1024, intermediate=2048, n_experts=16, n_group=4, topk_group=2, top_k=4, n_layers=2,
                max_tokens=8)
    base.update(kw)
    return MoeConfig(**base)


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [12, 14])
def test_synthetic_weights_match_host_generator(cuda_lib, oracle, down_type):
    cfg = small_cfg(intermediate=2048)
    m = cuda_lib.MoE(cfg)
    m.init_layer_synthetic(1, seed=7, down_type=down_type)
    for e in (0, 5, 15, 16):   # 16 = shared expert
        dev = m.read_expert(1, e)[: oracle.expert_bytes(cfg.hidden, cfg.intermediate, down_type)]
        host = oracle.gen_expert(7, 1, e, cfg.hidden, cfg.intermediate, down_type)
        assert np.array_equal(dev, host), e
    m.close()


@pytest.mark.gpu
def test_q6_repack_roundtrip_through_load(cuda_lib, oracle):
    """Raw GGUF bytes loaded with moe_load_layer come back unchanged from
    moe_read_expert (the Q6_K repack is lossless)."""
    cfg = small_cfg()
    H, I, E = cfg.hidden, cfg.intermediate, cfg.n_experts
    rng = np.random.default_rng(5)
    gb = oracle.row_bytes(12, H) * I
    db = oracle.row_bytes(14, I) * H
    gate = rng.integers(0, 256, E * gb, dtype=np.uint8)
    up = rng.integers(0, 256, E * gb, dtype=np.uint8)
    down = rng.integers(0, 256, E * db, dtype=np.uint8)
    sh = [rng.integers(0, 256, n, dtype=np.uint8) for n in (gb, gb, db)]
    router = rng.standard_normal((E, H)).astype(np.float32)
    m = cuda_lib.MoE(cfg)
    m.load_layer(0, gate, up, down, 14, router, None, sh[0], sh[1], sh[2], 14)
    for e in (0, 9, 15):
        back = m.read_expert(0, e)
        assert np.array_equal(back[:gb], gate[e * gb:(e + 1) * gb])
        assert np.array_equal(back[gb:2 * gb], up[e * gb:(e + 1) * gb])
        assert np.array_equal(back[2 * gb:2 * gb + db], down[e * db:(e + 1) * db])
    back = m.read_expert(0, E)
    assert np.array_equal(back[2 * gb:2 * gb + db], sh[2])
    m.close()
