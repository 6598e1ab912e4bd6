"""CPU: index arithmetic of the dense GEMVs (moe_dense.cu) emulated in numpy.

stage_rows stores each 256-float chunk of the activations so that lane l's 8
floats sit at 4 l and 128 + 4 l; the gate/up (and lm_head) warps read lane l's
16-byte weight vector i * 32 + l of a row, the down kernel's warp w reads the
vectors w * 32 + l + 256 i.  These tests check that every lane's shared-memory
reads return exactly the 8 activations that match its 8 weights, that a
quarter-warp's 16-byte reads touch distinct banks, that the down kernel's CTAs
cover every hidden row once with at most one row of imbalance, and that the
dense kernels' shared memory fits for DeepSeek's shapes."""
import numpy as np
import pytest


def stage(x):
    """stage_rows: float4 unit q of the source lands at unit
    (q & ~63) | ((q & 1) << 5) | ((q >> 1) & 31)."""
    src = x.reshape(-1, 4)
    dst = np.empty_like(src)
    q = np.arange(src.shape[0])
    dst[(q & ~63) | ((q & 1) << 5) | ((q >> 1) & 31)] = src
    return dst.reshape(-1)


def lane_floats(xs, base):
    """dot8's reads: 4 floats at base and 4 at base + 128."""
    return np.concatenate([xs[base:base + 4], xs[base + 128:base + 132]])


@pytest.mark.parametrize("H", [1024, 7168])
def test_gate_up_lane_reads_match_weights(H):
    x = np.arange(2 * H, dtype=np.float32)          # two tokens
    xs = stage(x)
    nv = H // 256
    for t in range(2):
        for i in range(nv):
            for lane in range(32):
                # weight vector i * 32 + lane holds columns 8 (i * 32 + lane) ...
                want = x[t * H + 8 * (i * 32 + lane): t * H + 8 * (i * 32 + lane) + 8]
                got = lane_floats(xs, t * H + lane * 4 + i * 256)
                assert np.array_equal(got, want), (t, i, lane)


@pytest.mark.parametrize("Id", [2560, 18432])
def test_down_lane_reads_match_weights(Id):
    a = np.arange(Id, dtype=np.float32)
    asm = stage(a)
    nv32 = Id // 8
    for warp in range(8):
        for lane in range(32):
            base = warp * 32 + lane
            cnt = (nv32 - base + 255) // 256 if nv32 > base else 0
            for i in range(cnt):
                v = base + 256 * i
                want = a[8 * v: 8 * v + 8]
                got = lane_floats(asm, warp * 256 + lane * 4 + i * 2048)
                assert np.array_equal(got, want), (warp, lane, i)


def test_quarter_warp_reads_are_conflict_free():
    """A 16-byte shared load is served per quarter warp (8 lanes); the 8 lanes'
    4-word pieces must fall in distinct 4-bank groups."""
    for half in (0, 128):
        for qw in range(4):
            banks = [((lane * 4 + half) % 32) // 4 for lane in range(qw * 8, qw * 8 + 8)]
            assert len(set(banks)) == 8
    # the plain layout (lane l at 8 l) had two lanes per bank group
    plain = [((lane * 8) % 32) // 4 for lane in range(8)]
    assert len(set(plain)) == 4


@pytest.mark.parametrize("H,G", [(7168, 444), (1024, 444), (7168, 148)])
def test_down_rows_split_evenly(H, G):
    G = min(G, H)
    rows = [(H * b // G, H * (b + 1) // G) for b in range(G)]
    assert rows[0][0] == 0 and rows[-1][1] == H
    assert all(rows[b][1] == rows[b + 1][0] for b in range(G - 1))
    sizes = [r1 - r0 for r0, r1 in rows]
    assert max(sizes) - min(sizes) <= 1 and max(sizes) == -(-H // G)


def test_shared_memory_fits_deepseek_shapes():
    H, Id, TT_GU, TT_D, WARPS, RPC_MAX = 7168, 18432, 4, 2, 8, 128
    assert TT_GU * H * 4 <= 227 * 1024                              # gate/up and lm_head
    assert TT_D * Id * 4 + WARPS * RPC_MAX * TT_D * 4 <= 227 * 1024   # down: activations + partial sums
