"""CPU: the operand and repack maps of moe_common.cuh, and a lane-by-lane
emulation of the tensor-core arithmetic of the expert kernels
(moe_experts.cu: q4_stage, q6_stage, planes_to_vector on the int8 path;
q4w_stage, q6w_stage on the fp16 path) against the quant.c dequantization, so that a fragment-layout or decode error shows up
without a GPU.  The maps come from a host build of the same header; the MMA
fragment layouts are those of the PTX ISA for mma.m16n8k32 / m16n8k16."""
import os
import subprocess
import tempfile
from collections import defaultdict

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def tables():
    exe = os.path.join(tempfile.mkdtemp(), "layout_dump")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-std=c++17", "-o", exe, os.path.join(HERE, "layout_dump.cu")],
                   check=True, capture_output=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    t = defaultdict(dict)
    for line in out:
        if not line:
            continue
        f = line.split()
        if f[0] in ("opq4", "opq6", "xsum", "q4r", "q6r", "opw4", "opw6"):
            t[f[0]][int(f[1])] = int(f[2])
        elif f[0] == "opw":
            t["opw"] = tuple(map(int, f[1:]))
        elif f[0] == "sizes":
            t["sizes"] = tuple(map(int, f[1:]))
        elif f[0] == "f2h":
            t["f2h"][float(f[1])] = int(f[2])
        elif f[0] == "split":
            t["split"] = int(f[1])
    return t


# ------------------------------------------------------------------ maps
def test_operand_maps_are_bijections(tables):
    assert sorted(tables["opq4"].values()) == list(range(256))
    assert sorted(tables["opq6"].values()) == list(range(256))
    xs = sorted(tables["xsum"].values())
    assert xs == [256 + 2 * i for i in range(16)]
    H, ob, op2, sb, plane = 7168, *tables["sizes"][1:]
    assert (sb, plane) == (960, 320) and ob == 28 * 960 and op2 == 8 * 960
    assert plane % 128 == 64  # plane blocks 80 words apart: quarter-warp loads hit distinct banks


def test_q4_operand_matches_weight_lanes(tables):
    # weight side: lane t holds repacked qs chunk j = old bytes 32j + 8t + i;
    # low nibble -> weight 32(2j) + 8t + i, high -> 32(2j+1) + 8t + i (quant.c:49-58).
    # operand side: lane t's 16-byte load j = [8 B of sub-block 2j][8 B of 2j+1].
    for j in range(4):
        for t in range(4):
            for i in range(8):
                for h in range(2):
                    k = 32 * (2 * j + h) + 8 * t + i
                    assert tables["opq4"][k] == 64 * j + 16 * t + 8 * h + i


def test_q4_repack_is_transpose(tables):
    src = tables["q4r"]
    assert sorted(src.values()) == list(range(128))
    for p, s in src.items():
        assert src[s] == p  # its own inverse
        c, i = p // 8, p % 8
        t, j = c // 4, c % 4
        assert s == 32 * j + 8 * t + i


def test_q6_operand_and_repack(tables):
    for s in range(16):
        for t in range(4):
            for i in range(4):
                assert tables["opq6"][16 * s + 4 * t + i] == 64 * (s // 4) + 16 * t + 4 * (s % 4) + i
    src = sorted(tables["q6r"].values())
    assert src == list(range(192))
    assert tables["sizes"][0] == 7168 * 8 * 210   # repacked matrix has the GGUF size
    for p, sb in tables["q6r"].items():
        t, rem = p // 48, p % 48
        h, w, b = rem // 24, (rem % 24) // 4, rem % 4
        if w < 4:
            assert sb == 64 * h + 16 * w + 4 * t + b
        else:
            assert sb == 128 + 32 * h + 16 * (w - 4) + 4 * t + b


def test_f2h_matches_numpy(tables):
    for f, bits in tables["f2h"].items():
        assert bits == int(np.float32(f).astype(np.float16).view(np.uint16)), f


def test_splitmix_matches_oracle(tables, oracle):
    assert tables["split"] == oracle.lib().or_splitmix64(12345)


# ------------------------------------------------------- MMA emulation
def w32(buf, off):
    return int.from_bytes(bytes(buf[off:off + 4]), "little")


def bytes_of(w, signed):
    b = [(w >> (8 * i)) & 0xFF for i in range(4)]
    return [x - 256 if signed and x > 127 else x for x in b]


def halves_of(w):
    return list(np.array([w & 0xFFFF, w >> 16], np.uint16).view(np.float16).astype(np.float64))


def mma(a, b, k, kind):
    """a[lane] = A registers, b[lane] = B registers of one warp; returns
    d[lane] = (D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1])."""
    A = np.zeros((16, k))
    B = np.zeros((k, 8))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        if kind == "k32":      # u8 x s8, m16n8k32
            for r, (row, k0) in enumerate([(g, 4 * t), (g + 8, 4 * t), (g, 16 + 4 * t), (g + 8, 16 + 4 * t)]):
                A[row, k0:k0 + 4] = bytes_of(a[lane][r], False)
            B[4 * t:4 * t + 4, g] = bytes_of(b[lane][0], True)
            B[16 + 4 * t:20 + 4 * t, g] = bytes_of(b[lane][1], True)
        elif kind == "k16s8":  # s8 x s8, m16n8k16
            A[g, 4 * t:4 * t + 4] = bytes_of(a[lane][0], True)
            A[g + 8, 4 * t:4 * t + 4] = bytes_of(a[lane][1], True)
            B[4 * t:4 * t + 4, g] = bytes_of(b[lane][0], True)
        else:                  # f16 m16n8k16
            for r, (row, k0) in enumerate([(g, 2 * t), (g + 8, 2 * t), (g, 2 * t + 8), (g + 8, 2 * t + 8)]):
                A[row, k0:k0 + 2] = halves_of(a[lane][r])
            B[2 * t:2 * t + 2, g] = halves_of(b[lane][0])
            B[2 * t + 8:2 * t + 10, g] = halves_of(b[lane][1])
    D = A @ B
    return [(D[l >> 2, 2 * (l & 3)], D[l >> 2, 2 * (l & 3) + 1], D[(l >> 2) + 8, 2 * (l & 3)],
             D[(l >> 2) + 8, 2 * (l & 3) + 1]) for l in range(32)]


def build_operand(tables, x, style):
    """Operand bytes of one super-block of each vector, as build_op writes them."""
    s = 2.0 ** (20 - np.frexp(np.max(np.abs(x)))[1])
    v = np.rint(x.astype(np.float64) * s).astype(np.int64)
    ops = []
    for vec in v:
        op = np.zeros(960, np.uint8)
        planes = [vec & 127, (vec >> 7) & 127, (vec >> 14) & 255]
        for p in range(3):
            for k in range(256):
                off = tables["opq4" if style == 4 else "opq6"][k]
                op[320 * p + off] = planes[p][k]
            if style == 4:
                pv = [vec & 127, (vec >> 7) & 127, vec >> 14][p]
                for jj in range(16):
                    h = np.float16(int(pv[16 * jj:16 * jj + 16].sum()))
                    op[320 * p + tables["xsum"][jj]:320 * p + tables["xsum"][jj] + 2] = \
                        np.frombuffer(h.tobytes(), np.uint8)
        ops.append(op)
    return np.concatenate(ops), v, 1.0 / s


def planes_to_vector(c0, c1, t_list):
    """planes_to_vector over a quad: c0[t], c1[t] for t = 0..3 -> (vector 2n, 2n+1)."""
    va = [c0[0] + 128 * c1[0], 16384 * c0[1], 0, 0]
    vb = [0, c1[1], 128 * c0[2] + 16384 * c1[2], 0]
    return sum(va), sum(vb)


def header_words(block):
    """q4_stage's word-level unpack of the 12 scale bytes (4 values per word)."""
    y, z, w = w32(block, 4), w32(block, 8), w32(block, 12)
    sc_lo, sc_hi = y & 0x3F3F3F3F, (w & 0x0F0F0F0F) | ((y >> 2) & 0x30303030)
    mn_lo, mn_hi = z & 0x3F3F3F3F, ((w >> 4) & 0x0F0F0F0F) | ((z >> 2) & 0x30303030)
    return sc_lo, sc_hi, mn_lo, mn_hi


def sc_pair(block, j):
    """(16 sc of sub-block 2j, sc of sub-block 2j + 1) as q4_stage extracts them."""
    sc_lo, sc_hi = header_words(block)[:2]
    sw, bl = (sc_lo if j < 2 else sc_hi), 2 * (j & 1)
    return ((sw >> (8 * bl)) & 0x3F) << 4, (sw >> (8 * bl + 8)) & 0x3F


def mins_words(block):
    mn_lo, mn_hi = header_words(block)[2:]
    return [(mn_lo >> (8 * s)) & 0xFF for s in range(4)] + [(mn_hi >> (8 * s)) & 0xFF for s in range(4)]


def test_q4_header_unpack_matches_quant_c():
    # get_scale_min_k4 (quant.c:26-34) on random scale bytes
    rng = np.random.default_rng(3)
    for _ in range(200):
        blk = rng.integers(0, 256, 144, dtype=np.uint8)
        q = blk[4:16].astype(int)
        sc = [(q[s] & 63) if s < 4 else ((q[s + 4] & 0xF) | ((q[s - 4] >> 6) << 4)) for s in range(8)]
        mn = [(q[s + 4] & 63) if s < 4 else ((q[s + 4] >> 4) | ((q[s] >> 6) << 4)) for s in range(8)]
        for j in range(4):
            assert sc_pair(blk, j) == (16 * sc[2 * j], sc[2 * j + 1])
        assert mins_words(blk) == mn


def test_q4_stage_emulation(tables, oracle):
    rng = np.random.default_rng(7)
    W = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(W.reshape(-1), oracle.TYPE_Q4_K).reshape(16, 144)
    wdq = oracle.dequant(blocks.reshape(-1), oracle.TYPE_Q4_K, 16 * 256).reshape(16, 256).astype(np.float64)
    rep = blocks.copy()
    for p, sidx in tables["q4r"].items():
        rep[:, 16 + p] = blocks[:, 16 + sidx]
    x = rng.standard_normal((2, 256)).astype(np.float32)
    opnd, v, inv = build_operand(tables, x, 4)
    acc = [[0, 0, 0, 0] for _ in range(32)]
    a_l, a_h, b_l, b_h = {}, {}, {}, {}
    for j in range(4):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            wg = [w32(rep[g], 16 + 32 * t + 8 * j), w32(rep[g], 20 + 32 * t + 8 * j)]
            w8 = [w32(rep[g + 8], 16 + 32 * t + 8 * j), w32(rep[g + 8], 20 + 32 * t + 8 * j)]
            a_l[lane] = [wg[0] & 0x0F0F0F0F, w8[0] & 0x0F0F0F0F, wg[1] & 0x0F0F0F0F, w8[1] & 0x0F0F0F0F]
            a_h[lane] = [wg[0] & 0xF0F0F0F0, w8[0] & 0xF0F0F0F0, wg[1] & 0xF0F0F0F0, w8[1] & 0xF0F0F0F0]
            tsel, plane = (1 if g >= 3 else 0), g % 3
            ok = g < 6 and tsel < 2
            base = tsel * 960 + plane * 320 + 16 * t + 64 * j
            wv = [w32(opnd, base + 4 * q) if ok else 0 for q in range(4)]
            b_l[lane], b_h[lane] = wv[0:2], wv[2:4]
        dl, dh = mma(a_l, b_l, 32, "k32"), mma(a_h, b_h, 32, "k32")
        for lane in range(32):
            g = lane >> 2
            slg, shg = sc_pair(rep[g], j)
            sl8, sh8 = sc_pair(rep[g + 8], j)
            acc[lane][0] += slg * dl[lane][0] + shg * dh[lane][0]
            acc[lane][1] += slg * dl[lane][1] + shg * dh[lane][1]
            acc[lane][2] += sl8 * dl[lane][2] + sh8 * dh[lane][2]
            acc[lane][3] += sl8 * dl[lane][3] + sh8 * dh[lane][3]
    assert max(abs(a) for l in acc for a in l) < 2 ** 31
    am, bm = {}, {}
    for lane in range(32):
        g, t = lane >> 2, lane & 3

        mg, m8 = mins_words(rep[g]), mins_words(rep[g + 8])
        h2 = lambda m: int(np.array([m, m], np.float16).view(np.uint32)[0])
        am[lane] = [h2(mg[t]), h2(m8[t]), h2(mg[t + 4]), h2(m8[t + 4])]
        tsel, plane = (1 if g >= 3 else 0), g % 3
        base = tsel * 960 + plane * 320 + 256 + 8 * t
        bm[lane] = [w32(opnd, base), w32(opnd, base + 4)] if g < 6 else [0, 0]
    mt = mma(am, bm, 16, "f16")
    out = np.zeros((16, 2))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        hg, h8 = rep[g][:4].view(np.float16).astype(np.float64), rep[g + 8][:4].view(np.float16).astype(np.float64)
        lane_f = [hg[0] / 16 * acc[lane][0] - hg[1] * mt[lane][0], hg[0] / 16 * acc[lane][1] - hg[1] * mt[lane][1],
                  h8[0] / 16 * acc[lane][2] - h8[1] * mt[lane][2], h8[0] / 16 * acc[lane][3] - h8[1] * mt[lane][3]]
        acc[lane] = lane_f
    for g in range(8):
        quad = [acc[4 * g + t] for t in range(4)]
        for half, row in ((0, g), (2, g + 8)):
            va, vb = planes_to_vector([q[half] for q in quad], [q[half + 1] for q in quad], None)
            out[row] = (va, vb)
    ref = np.stack([wdq @ v[0].astype(np.float64), wdq @ v[1].astype(np.float64)], axis=1)
    err = np.max(np.abs(out - ref)) / np.max(np.abs(ref))
    assert err < 1e-12, err


def test_q6_stage_emulation(tables, oracle):
    rng = np.random.default_rng(8)
    W = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(W.reshape(-1), oracle.TYPE_Q6_K).reshape(16, 210)
    wdq = oracle.dequant(blocks.reshape(-1), oracle.TYPE_Q6_K, 16 * 256).reshape(16, 256).astype(np.float64)
    Q = np.zeros((16, 192), np.uint8)
    for p, sidx in tables["q6r"].items():
        Q[:, p] = blocks[:, sidx] ^ (0xAA if sidx >= 128 else 0)
    S = blocks[:, 192:208].view(np.int8)
    D = blocks[:, 208:210].copy().view(np.float16).astype(np.float64)[:, 0]
    x = rng.standard_normal((2, 256)).astype(np.float32)
    opnd, v, inv = build_operand(tables, x, 6)

    def q6_a4(sp, W_, Hw):
        nib = ((W_ << 2) & 0x3C3C3C3C) if sp < 4 else ((W_ >> 2) & 0x3C3C3C3C)
        f = sp >> 1
        hs = [(Hw << 6), (Hw << 4), (Hw << 2), Hw][f] & 0xFFFFFFFF
        return (nib | (hs & 0xC0C0C0C0)) & 0xFFFFFFFF
    acc = [[0, 0, 0, 0] for _ in range(32)]
    for s in range(16):
        h, sp = s // 8, s % 8
        a, b = {}, {}
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            wg = [w32(Q[g], 48 * t + 24 * h + 4 * i) for i in range(6)]
            w8 = [w32(Q[g + 8], 48 * t + 24 * h + 4 * i) for i in range(6)]
            a[lane] = [q6_a4(sp, wg[sp & 3], wg[4 + (sp & 1)]), q6_a4(sp, w8[sp & 3], w8[4 + (sp & 1)])]
            tsel, plane = (1 if g >= 3 else 0), g % 3
            base = tsel * 960 + plane * 320 + 16 * t + 64 * (s // 4) + 4 * (s % 4)
            b[lane] = [w32(opnd, base) if g < 6 else 0]
        dd = mma(a, b, 16, "k16s8")
        for lane in range(32):
            g = lane >> 2
            acc[lane][0] += int(S[g, s]) * dd[lane][0]
            acc[lane][1] += int(S[g, s]) * dd[lane][1]
            acc[lane][2] += int(S[g + 8, s]) * dd[lane][2]
            acc[lane][3] += int(S[g + 8, s]) * dd[lane][3]
    assert max(abs(a_) for l in acc for a_ in l) < 2 ** 31
    out = np.zeros((16, 2))
    for g in range(8):
        quad = [acc[4 * g + t] for t in range(4)]
        for half, row in ((0, g), (2, g + 8)):
            va, vb = planes_to_vector([q[half] for q in quad], [q[half + 1] for q in quad], None)
            out[row] = (D[row] * 0.25 * va, D[row] * 0.25 * vb)
    ref = np.stack([wdq @ v[0].astype(np.float64), wdq @ v[1].astype(np.float64)], axis=1)
    err = np.max(np.abs(out - ref)) / np.max(np.abs(ref))
    assert err < 1e-12, err


# ---------------------------------------------------------------------------
# The prefill GEMMs' dequantization of one 64-column atom into fp16 pairs
# (moe_prefill.cu: pf_q4_consts / pf_deq_q4 and pf_q6_consts / pf_deq_q6),
# emulated step by step with single fp16 roundings, from the repacked bytes
# the kernels read, against the quant.c dequantization.

def f16(x):
    """round to the nearest fp16 (ties to even), as a Python float"""
    return float(np.float16(x))


def hfma(a, b, c):
    return f16(a * b + c)   # a * b is exact in binary64 for fp16 inputs


def byte_perm(x, y, s):
    """__byte_perm(x, y, s): result byte n is byte (s >> 4n) & 7 of y:x"""
    src = x | (y << 32)
    return sum(((src >> (8 * ((s >> (4 * n)) & 7))) & 0xFF) << (8 * n) for n in range(4))


def h2(u):
    """the two fp16 halves of a 32-bit word, low first"""
    return np.array([u & 0xFFFF, u >> 16], np.uint16).view(np.float16).astype(np.float64)


def q4_scale_min(sb, j):
    """get_scale_min_k4 (quant.c:26-34) on the 12 scale bytes"""
    if j < 4:
        return sb[j] & 63, sb[j + 4] & 63
    return (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4), (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4)


def split16(x):
    hi = f16(np.float32(x))
    return hi, f16(np.float32(np.float32(x) - np.float32(hi)))


def weight_blocks(oracle, qtype, rows, seed):
    rng = np.random.default_rng(seed)
    sig = np.array([0.02, 0.5, 1e-3, 3.0, 0.02, 0.1, 2e-4, 0.02][:rows])[:, None]
    W = (rng.standard_normal((rows, 256)) * sig).astype(np.float32)
    W[-1, ::7] = 0.0
    bb = 144 if qtype == oracle.TYPE_Q4_K else 210
    blocks = oracle.quantize(W.reshape(-1), qtype).reshape(rows, bb)
    ref = oracle.dequant(blocks.reshape(-1), qtype, rows * 256).reshape(rows, 256).astype(np.float64)
    return blocks, ref


def check_fp16_dequant(out, ref, max_ulps):
    """error against the fp32 dequantization in units of the fp16 spacing at
    the correctly rounded value (0.5 = correctly rounded)"""
    cr = np.vectorize(f16)(ref)
    ulp = np.maximum(np.spacing(np.abs(cr).astype(np.float16)).astype(np.float64), 2.0 ** -24)
    e = float(np.max(np.abs(out - ref) / ulp))
    assert e <= max_ulps, e


def test_prefill_q4_dequant_emulation(tables, oracle):
    rows = 8
    blocks, ref = weight_blocks(oracle, oracle.TYPE_Q4_K, rows, 21)
    rep = blocks.copy()
    for p, s in tables["q4r"].items():   # the load-time transpose of the qs bytes
        rep[:, 16 + p] = blocks[:, 16 + s]
    out = np.zeros((rows, 256))
    for r in range(rows):
        blk = rep[r]
        d = float(blk[0:2].view(np.float16)[0])
        dmin = np.float32(blk[2:4].view(np.float16)[0])
        sb = [int(b) for b in blk[4:16]]
        for g in range(4):
            sc0, m0 = q4_scale_min(sb, 2 * g)
            sc1, m1 = q4_scale_min(sb, 2 * g + 1)
            c = [f16(sc0), f16(-1024.0 * sc0), *split16(-dmin * np.float32(m0)),
                 f16(0.0625 * sc1), f16(-64.0 * sc1), *split16(-dmin * np.float32(m1))]
            v = np.zeros(64)
            for t in range(4):
                for h in range(2):
                    w = w32(blk, 16 + 32 * t + 8 * g + 4 * h)
                    x01, x23 = byte_perm(w, 0x64, 0x4140), byte_perm(w, 0x64, 0x4342)
                    for reg, x, hi in ((4 * t + 2 * h, x01 & 0xFF0FFF0F, 0), (4 * t + 2 * h + 1, x23 & 0xFF0FFF0F, 0),
                                       (16 + 4 * t + 2 * h, x01 & 0xFFF0FFF0, 1),
                                       (16 + 4 * t + 2 * h + 1, x23 & 0xFFF0FFF0, 1)):
                        cc = c[4 * hi:4 * hi + 4]
                        for i, xv in enumerate(h2(x)):
                            p = hfma(xv, cc[0], cc[1])
                            assert p == (xv - 1024.0) / (16.0 if hi else 1.0) * (sc1 if hi else sc0)  # v * sc, exact
                            v[2 * reg + i] = f16(hfma(p, d, cc[2]) + cc[3])
            out[r, 64 * g:64 * g + 64] = v
    check_fp16_dequant(out, ref, 1.0)   # fma, then the low half of dmin*m: two roundings


def test_prefill_q6_dequant_emulation(tables, oracle):
    rows = 8
    blocks, ref = weight_blocks(oracle, oracle.TYPE_Q6_K, rows, 22)
    Q = np.zeros((rows, 192), np.uint8)
    for p, sidx in tables["q6r"].items():   # the load-time Q plane (qh pairs' high bit inverted)
        Q[:, p] = blocks[:, sidx] ^ (0xAA if sidx >= 128 else 0)
    S = blocks[:, 192:208].view(np.int8)
    D = blocks[:, 208:210].copy().view(np.float16)[:, 0]
    out = np.zeros((rows, 256))
    for r in range(rows):
        for A in range(4):
            h = A >> 1
            q = [w32(Q[r], 48 * t + 24 * h + 4 * u) for t in range(4) for u in range(6)]
            c = [x for u in range(4) for x in split16(np.float32(D[r]) * np.float32(S[r, 4 * A + u]))]
            v = np.zeros(64)
            for t in range(4):
                for s4 in range(4):
                    sp = 4 * (A & 1) + s4
                    f = sp >> 1
                    W, Hq = q[6 * t + s4], q[6 * t + 4 + (s4 & 1)]
                    nib = (W if sp < 4 else W >> 4) & 0x0F0F0F0F
                    hb = ((Hq << (4 - 2 * f)) if 2 * f <= 4 else (Hq >> (2 * f - 4))) & 0x30303030
                    q6 = nib | (hb ^ 0x20202020)
                    fh, fl = c[2 * s4], c[2 * s4 + 1]
                    for reg, sel in ((8 * s4 + 2 * t, 0x4140), (8 * s4 + 2 * t + 1, 0x4342)):
                        for i, xv in enumerate(h2(byte_perm(q6, 0x64, sel))):
                            vq = f16(xv - 1056.0)
                            assert vq == xv - 1056.0   # q - 32 is exact
                            v[2 * reg + i] = hfma(vq, fh, f16(vq * fl))
            out[r, 64 * A:64 * A + 64] = v
    check_fp16_dequant(out, ref, 0.5)   # correctly rounded: one rounding of (q - 32) * d * sc



# ---------------------------------------------------------------------------
# fp16 path of the expert GEMVs (moe_experts.cu: q4w_stage, q6w_stage; the
# operand of moe_kernels.cu: build_opw_sb), lane by lane with single fp16
# roundings, on two 4-token tiles.

def test_wide_operand_maps(tables):
    sb, xsum, scale, lo, top = tables["opw"]
    assert (sb, xsum, scale, lo, top) == (1104, 512, 544, 576, 15)
    assert lo % 128 == 64 and sb % 16 == 0  # planes' quarter-warp loads on distinct banks; bulk-copy size
    assert (4 * sb) % 128 == 64             # x_hi of tokens k, k + 4 (Q6_K residual tiles) on distinct banks
    for name in ("opw4", "opw6"):
        assert sorted(tables[name].values()) == list(range(256))
    for k in range(256):  # style Q4: lane t = (k / 8) % 4 of sub-block k / 32 owns 8 contiguous fp16
        j, t, i = k >> 5, (k >> 3) & 3, k & 7
        assert tables["opw4"][k] == 32 * j + 8 * t + [0, 2, 1, 3, 4, 6, 5, 7][i]
        s, t6, i6 = k >> 4, (k >> 2) & 3, k & 3
        assert tables["opw6"][k] == 32 * (s >> 1) + 8 * t6 + 4 * (s & 1) + i6


OPW = 1104  # OPW_SB, checked against the header by test_wide_operand_maps


def build_wide_operand(tables, xs, style):
    """build_opw_sb for each vector of xs [n, 256]: bytes, and the exact
    values (hi + lo) / s the MMAs see."""
    ops, vals = [], []
    for x in xs.astype(np.float32):
        amax = float(np.max(np.abs(x)))
        s = 2.0 ** (15 - np.frexp(amax)[1])
        xsc = (x.astype(np.float64) * s).astype(np.float32)
        hi = xsc.astype(np.float16)
        lo = (xsc - hi.astype(np.float32)).astype(np.float16)
        op = np.zeros(OPW, np.uint8)
        H = np.zeros(256, np.float16)
        L = np.zeros(256, np.float16)
        m = tables["opw4" if style == 4 else "opw6"]
        for k in range(256):
            H[m[k]], L[m[k]] = hi[k], lo[k]
        op[0:512] = np.frombuffer(H.tobytes(), np.uint8)
        op[576:1088] = np.frombuffer(L.tobytes(), np.uint8)
        v = hi.astype(np.float32) + lo.astype(np.float32)   # exact
        if style == 4:
            for j in range(8):
                lane_sums = [np.float32(0)] * 4
                for t in range(4):   # each lane sums its 8 values in order, then xor 1, xor 2
                    acc = np.float32(0)
                    for i in range(8):
                        acc = np.float32(acc + v[32 * j + 8 * t + i])
                    lane_sums[t] = acc
                a = [np.float32(lane_sums[t] + lane_sums[t ^ 1]) for t in range(4)]
                tot = np.float32(a[0] + a[2])
                s32 = np.float32(tot * np.float32(0.03125))
                sh = np.float16(s32)
                sl = np.float16(np.float32(s32 - np.float32(sh)))
                op[512 + 2 * j:514 + 2 * j] = np.frombuffer(sh.tobytes(), np.uint8)
                op[528 + 2 * j:530 + 2 * j] = np.frombuffer(sl.tobytes(), np.uint8)
        op[544:548] = np.frombuffer(np.float32(1.0 / s).tobytes(), np.uint8)
        ops.append(op)
        vals.append(v.astype(np.float64) / s)
    return np.concatenate(ops), np.stack(vals)


def h2pair(a, b):
    return int(np.array([a, b], np.float16).view(np.uint32)[0])


def test_q4w_stage_emulation(tables, oracle):
    rng = np.random.default_rng(17)
    W = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(W.reshape(-1), oracle.TYPE_Q4_K).reshape(16, 144)
    wdq = oracle.dequant(blocks.reshape(-1), oracle.TYPE_Q4_K, 16 * 256).reshape(16, 256).astype(np.float64)
    rep = blocks.copy()
    for p, sidx in tables["q4r"].items():
        rep[:, 16 + p] = blocks[:, 16 + sidx]
    NTOK = 8
    x = (rng.standard_normal((NTOK, 256)) * np.array([1, 1e-3, 50, 1, 1, 1, 1e-5, 3])[:, None]).astype(np.float32)
    opnd, xv = build_wide_operand(tables, x, 4)

    def sc_of(row, s):
        sc_lo, sc_hi = header_words(rep[row])[:2]
        return ((sc_lo if s < 4 else sc_hi) >> (8 * (s & 3))) & 0x3F

    def dec(word, row, s, high):
        # (w & mask) | 0x6400 pairs -> fma(1024 + v, c, n): q sc exactly
        sc = sc_of(row, s)
        m = 0x00F000F0 if high else 0x000F000F
        u = (word & m) | 0x64006400
        a, b = halves_of(u)
        c, n = (sc / 16.0, -64.0 * sc) if high else (float(sc), -1024.0 * sc)
        return h2pair(hfma(a, c, n), hfma(b, c, n))

    out = np.zeros((16, NTOK))
    for n_tile in range(NTOK // 4):
        acc = [[0.0] * 4 for _ in range(32)]
        for jj in range(4):
            for step_hi in (0, 1):      # sub-block 2 jj (low nibbles), 2 jj + 1 (high)
                for step in range(2):   # k16 steps: elements (0,2),(1,3) then (4,6),(5,7)
                    a, b = {}, {}
                    for lane in range(32):
                        g, t = lane >> 2, lane & 3
                        regs = []
                        for row in (g, g + 8):
                            w = w32(rep[row], 16 + 32 * t + 8 * jj + 4 * step)
                            regs.append((dec(w, row, 2 * jj + step_hi, step_hi),
                                         dec(w >> 8, row, 2 * jj + step_hi, step_hi)))
                        a[lane] = [regs[0][0], regs[1][0], regs[0][1], regs[1][1]]
                        tok = 4 * n_tile + (g >> 1)
                        base = tok * OPW + (g & 1) * 576 + 16 * t + 64 * (2 * jj + step_hi) + 8 * step
                        b[lane] = [w32(opnd, base), w32(opnd, base + 4)]
                    d = mma(a, b, 16, "f16")
                    for lane in range(32):
                        for q in range(4):
                            acc[lane][q] += d[lane][q]
        am, bm = {}, {}
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            mg, m8 = mins_words(rep[g]), mins_words(rep[g + 8])
            am[lane] = [h2pair(mg[2 * t], mg[2 * t + 1]), h2pair(m8[2 * t], m8[2 * t + 1]), 0, 0]
            tok = 4 * n_tile + (g >> 1)
            bm[lane] = [w32(opnd, tok * OPW + 512 + 16 * (g & 1) + 4 * t), 0]
        mt = mma(am, bm, 16, "f16")
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            tok = 4 * n_tile + t
            inv = float(np.frombuffer(bytes(opnd[tok * OPW + 544:tok * OPW + 548]), np.float32)[0])
            for r, row in enumerate((g, g + 8)):
                d_, dm = rep[row][:4].view(np.float16).astype(np.float64)
                out[row, tok] = d_ * inv * (acc[lane][2 * r] + acc[lane][2 * r + 1]) \
                    - 32 * dm * inv * (mt[lane][2 * r] + mt[lane][2 * r + 1])
    ref = wdq @ x.astype(np.float64).T
    for tk in range(NTOK):   # per token: the product of the exact weights with x, to the 22-bit split
        err = np.max(np.abs(out[:, tk] - ref[:, tk])) / np.max(np.abs(ref[:, tk]))
        assert err < 2e-6, (tk, err)


def test_q6w_stage_emulation(tables, oracle):
    rng = np.random.default_rng(18)
    W = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    W[3, :16] *= 40.0   # a sub-block with a large scale: |(q - 32) sc| beyond 2048 (residual MMA)
    blocks = oracle.quantize(W.reshape(-1), oracle.TYPE_Q6_K).reshape(16, 210)
    wdq = oracle.dequant(blocks.reshape(-1), oracle.TYPE_Q6_K, 16 * 256).reshape(16, 256).astype(np.float64)
    Q = np.zeros((16, 192), np.uint8)
    for p, sidx in tables["q6r"].items():
        Q[:, p] = blocks[:, sidx] ^ (0xAA if sidx >= 128 else 0)
    S = blocks[:, 192:208].view(np.int8).astype(int)
    D = blocks[:, 208:210].copy().view(np.float16).astype(np.float64)[:, 0]
    NTOK = 8
    x = (rng.standard_normal((NTOK, 256)) * np.array([1, 1e-3, 50, 1, 1, 1, 1e-5, 3])[:, None]).astype(np.float32)
    opnd, xv = build_wide_operand(tables, x, 6)
    big = 0

    def dec(Wq, Hq, sp, sc):
        nonlocal big
        nib = (Wq if sp < 4 else Wq >> 4) & 0x0F0F0F0F
        f = sp >> 1
        hb = ((Hq << (4 - 2 * f)) if 2 * f <= 4 else (Hq >> (2 * f - 4))) & 0x30303030
        q6 = nib | (hb ^ 0x20202020)
        P, R = [], []
        for sel in (0x4140, 0x4342):
            qa, qb = [h - 1056.0 for h in halves_of(byte_perm(q6, 0x64, sel))]
            p_ = [f16(qa * sc), f16(qb * sc)]
            r_ = [hfma(qa, sc, -p_[0]), hfma(qb, sc, -p_[1])]
            big += sum(1 for v in r_ if v != 0)
            P.append(h2pair(*p_))
            R.append(h2pair(*r_))
        return P, R

    out = np.zeros((16, NTOK))
    for n_tile in range(NTOK // 4):
        acc = [[0.0] * 4 for _ in range(32)]
        for s in range(16):
            h, sp = s >> 3, s & 7
            aP, aR, b, br = {}, {}, {}, {}
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                rg = []
                for row in (g, g + 8):
                    wq = [w32(Q[row], 48 * t + 24 * h + 4 * i) for i in range(6)]
                    rg.append(dec(wq[sp & 3], wq[4 + (sp & 1)], sp, float(S[row, s])))
                aP[lane] = [rg[0][0][0], rg[1][0][0], rg[0][0][1], rg[1][0][1]]
                aR[lane] = [rg[0][1][0], rg[1][1][0], rg[0][1][1], rg[1][1][1]]
                tok = 4 * n_tile + (g >> 1)
                base = tok * OPW + (g & 1) * 576 + 16 * t + 64 * (s >> 1) + 8 * (s & 1)
                b[lane] = [w32(opnd, base), w32(opnd, base + 4)]
                # the R tile: x_hi of token (g / 2) + 4 (g % 2) of the 8-token group
                tokr = 8 * (n_tile >> 1) + (g >> 1) + 4 * (g & 1)
                baser = tokr * OPW + 16 * t + 64 * (s >> 1) + 8 * (s & 1)
                br[lane] = [w32(opnd, baser), w32(opnd, baser + 4)]
            d = mma(aP, b, 16, "f16")
            dr = mma(aR, br, 16, "f16")
            for lane in range(32):
                for q in range(4):
                    acc[lane][q] += d[lane][q]
                # lane t's R columns 2t, 2t+1 are tokens t and t + 4 of the group:
                # this tile's token 4 n + t is column 2t + (n % 2)
                acc[lane][0] += dr[lane][n_tile & 1]
                acc[lane][2] += dr[lane][2 + (n_tile & 1)]
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            tok = 4 * n_tile + t
            inv = float(np.frombuffer(bytes(opnd[tok * OPW + 544:tok * OPW + 548]), np.float32)[0])
            for r, row in enumerate((g, g + 8)):
                out[row, tok] = D[row] * inv * (acc[lane][2 * r] + acc[lane][2 * r + 1])
    assert big > 0   # the residual MMA carried something
    ref = wdq @ x.astype(np.float64).T
    for tk in range(NTOK):
        err = np.max(np.abs(out[:, tk] - ref[:, tk])) / np.max(np.abs(ref[:, tk]))
        assert err < 2e-6, (tk, err)
