"""CPU: the weight-byte -> MMA-slot maps and the lossless Q6_K repack used by
the CUDA kernels (moe_common.cuh) are bijections that match the GGUF block
layouts of quant.c, checked on a host build of the same header."""
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
        if f[0] in ("q4k", "q6k"):
            t[f[0]][tuple(map(int, f[1:4]))] = int(f[4])
        elif f[0] in ("q4min", "q6r"):
            t[f[0]][int(f[1])] = int(f[2])
        elif f[0] == "sizes":
            t["sizes"] = tuple(map(int, f[1:]))
        elif f[0] == "f2h":
            t["f2h"][float(f[1])] = int(f[2])
        elif f[0] == "split":
            t["split"] = int(f[1])
    return t


def test_q4k_map_is_bijection(tables):
    ks = sorted(tables["q4k"].values())
    assert ks == list(range(256))


def test_q4k_map_matches_nibble_layout(tables):
    # lane t of MMA step m reads qs bytes [64r+16t, +16), word i = (m/2)%4;
    # slots (0,1) = bytes (0,2) of the word, (2,3) = bytes (1,3); m odd = high
    # nibble.  quant.c:49-58: low nibble of qs byte b (chunk c = b/32) is
    # weight 64c + b%32, the high nibble weight 64c + 32 + b%32.
    for (m, t, j), k in tables["q4k"].items():
        r, i, hi = m // 8, (m // 2) % 4, m % 2
        byte = 64 * r + 16 * t + 4 * i + [0, 2, 1, 3][j]
        c, l = byte // 32, byte % 32
        assert k == 64 * c + 32 * hi + l


def test_q4k_min_subblocks(tables):
    # the four lanes supply the 8 min slots once each
    subs = sorted(s + u for s in tables["q4min"].values() for u in (0, 1))
    assert subs == list(range(8))
    # and lane t owns the scales of those sub-blocks (its nibbles live there)
    for t, s in tables["q4min"].items():
        own = {tables["q4k"][(m, t, 0)] // 32 for m in range(16)}
        assert {s, s + 1} <= own


def test_q6k_map(tables):
    ks = sorted(tables["q6k"].values())
    assert ks == list(range(256))
    for (s, t, j), k in tables["q6k"].items():
        assert k // 16 == s  # one MMA step = one 16-weight sub-block


def test_q6_repack_is_permutation(tables):
    src = sorted(tables["q6r"].values())
    assert src == list(range(192))  # every ql/qh byte exactly once
    n = tables["sizes"]
    assert n[0] == 7168 * 8 * 210   # repacked matrix has the GGUF size


def test_q6_repack_lane_bytes(tables):
    # lane t of block half h reads ql bytes 4t+16w (w<4) and qh bytes 4t+16w'
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
