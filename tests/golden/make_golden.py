"""Generates the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference sources (the oracle Makefile builds
oracle/_ref/libref_moe.so from them) and gguf-py:

    python tests/golden/make_golden.py

Fixtures (all seeded, small):
  dequant_q4k.npz / dequant_q6k.npz  random + edge-case super-blocks and their
      dequantization by gguf-py 0.19.0 (gguf.quants.dequantize), asserted
      bit-identical to the reference's quant.c before saving
  fp16_table.npz     quant.c fp16_to_fp32 of all 65536 bit patterns
  route_golden.npz   logits/bias cases (random, exact ties, near ties) and the
      reference route() (infer.m:920-991) outputs in slot order
  act_golden.npz     reference silu_mul / rms_norm / sigmoidf outputs
  synth_golden.npz   first super-blocks of the synthetic generator + quantizer
      (no reference counterpart; pins the generator across machines)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def rand_q4k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(n)) * 1e-3).astype(np.float16)
    dm = (np.abs(rng.standard_normal(n)) * 1e-3).astype(np.float16)
    # edge cases: subnormal d, dmin = 0, negative d, large d
    d[0] = np.float16(3e-7)      # subnormal half
    dm[1] = np.float16(0.0)
    d[2] = np.float16(-0.5)
    d[3] = np.float16(60000.0)
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(n, 2)
    b[4, 4:16] = 0xFF            # all scale/min bits set (top bits of every slot)
    b[5, 4:16] = 0x00
    return b


def rand_q6k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    d = (rng.standard_normal(n) * 1e-3).astype(np.float16)
    d[0] = np.float16(3e-7)
    d[1] = np.float16(0.0)
    d[2] = np.float16(-60000.0)
    b[:, 208:210] = d.view(np.uint8).reshape(n, 2)
    b[3, 192:208] = 0x80         # scales = -128
    b[4, 192:208] = 0x7F         # scales = 127
    b[5, 0:192] = 0xFF           # q = 31 everywhere
    return b


def main():
    import gguf
    from gguf.quants import dequantize
    O.build()
    assert O.ref_available(), "reference build (oracle/_ref) missing"
    rng = np.random.default_rng(20261201)

    q4 = rand_q4k_blocks(rng, 64)
    g4 = dequantize(q4, gguf.GGMLQuantizationType.Q4_K).reshape(64, 256).astype(np.float32)
    r4 = O.ref_dequant(q4.reshape(-1), O.TYPE_Q4_K, 64 * 256).reshape(64, 256)
    assert np.array_equal(g4.view(np.uint32), r4.view(np.uint32)), "gguf-py and quant.c disagree on Q4_K"
    np.savez_compressed(os.path.join(HERE, "dequant_q4k.npz"), blocks=q4, expected=r4,
                        source="gguf-py %s dequantize == reference quant.c" % getattr(gguf, "__version__", "0.19.0"))

    q6 = rand_q6k_blocks(rng, 64)
    g6 = dequantize(q6, gguf.GGMLQuantizationType.Q6_K).reshape(64, 256).astype(np.float32)
    r6 = O.ref_dequant(q6.reshape(-1), O.TYPE_Q6_K, 64 * 256).reshape(64, 256)
    assert np.array_equal(g6.view(np.uint32), r6.view(np.uint32)), "gguf-py and quant.c disagree on Q6_K"
    np.savez_compressed(os.path.join(HERE, "dequant_q6k.npz"), blocks=q6, expected=r6)

    R = O.ref()
    table = np.array([R.fp16_to_fp32(h) for h in range(65536)], np.float32)
    np.savez_compressed(os.path.join(HERE, "fp16_table.npz"), bits=table.view(np.uint32))

    # route cases: random, exact ties, near ties, skewed bias
    cases_l, cases_b = [], []
    for i in range(96):
        cases_l.append((rng.standard_normal(256) * 2).astype(np.float32))
        cases_b.append((rng.standard_normal(256) * 0.01).astype(np.float32))
    for i in range(16):  # exact ties: repeated logits, zero bias
        lg = np.repeat(rng.standard_normal(32).astype(np.float32), 8)
        rng.shuffle(lg)
        cases_l.append(lg)
        cases_b.append(np.zeros(256, np.float32))
    for i in range(16):  # near ties (1e-7 .. 1e-6 apart)
        base = np.float32(rng.standard_normal())
        lg = (base + rng.integers(0, 10, 256) * 1e-7).astype(np.float32)
        cases_l.append(lg)
        cases_b.append((rng.standard_normal(256) * 1e-7).astype(np.float32))
    cases_l.append(np.zeros(256, np.float32))  # all equal
    cases_b.append(np.zeros(256, np.float32))
    L = np.stack(cases_l)
    B = np.stack(cases_b)
    idx = np.zeros((len(L), 8), np.int32)
    w = np.zeros((len(L), 8), np.float32)
    for i in range(len(L)):
        idx[i], w[i] = O.ref_route(L[i], B[i], K=8)
    np.savez_compressed(os.path.join(HERE, "route_golden.npz"), logits=L, bias=B, idx=idx, w=w)

    g = (rng.standard_normal(2048) * 3).astype(np.float32)
    u = rng.standard_normal(2048).astype(np.float32)
    silu = np.empty_like(g)
    R.ref_silu_mul(g, u, silu, g.size)
    x = rng.standard_normal(7168).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(7168)).astype(np.float32)
    rms = np.empty_like(x)
    R.ref_rms_norm(x, nw.ctypes.data_as(O.C.c_void_p), rms, x.size)
    sig_in = np.linspace(-30, 30, 1001).astype(np.float32)
    sig = np.array([R.ref_sigmoidf(float(v)) for v in sig_in], np.float32)
    np.savez_compressed(os.path.join(HERE, "act_golden.npz"), g=g, u=u, silu=silu, x=x, norm_w=nw, rms=rms,
                        sig_in=sig_in, sig=sig)

    seed = 0
    gate4 = O.gen_matrix(seed, O.stream(0, 0, O.KIND_GATE), O.TYPE_Q4_K, 1, 1024, 0.02)
    down6 = O.gen_matrix(seed, O.stream(0, 0, O.KIND_DOWN), O.TYPE_Q6_K, 1, 1024, 0.02)
    router = O.normal(seed, O.stream(0, 0, O.KIND_ROUTER), 64, 0.006)
    np.savez_compressed(os.path.join(HERE, "synth_golden.npz"), gate_q4k=gate4, down_q6k=down6, router=router)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
