"""CPU: the sampler's selection (moe_sample.cu) restated step by step in numpy
-- radix selection over the probabilities' bit patterns with 2^40 fixed-point
bucket sums, the tie count, the nucleus mass and the draw -- against the
direct definition (sort descending with ties in index order, running sums,
first crossing), on the edge cases the kernel has to get right: ties, a
uniform row, top_p = 1 with a total mass below 1, probabilities that
underflow to zero, a draw of zero."""
import numpy as np
import pytest

FIX = float(2 ** 40)


def fx(p):
    return (np.asarray(p, np.float32).astype(np.float64) * FIX).astype(np.uint64)


def radix_select(p, target, kmin=None):
    """k_sg_hist / k_sg_pick over keys (all, or those above kmin): (key,
    fixed sum above it, count equal to it)."""
    keys = np.asarray(p, np.float32).view(np.uint32)
    f = fx(p)
    inset = np.ones(keys.size, bool) if kmin is None else keys > np.uint32(kmin)
    pre, msk, above = 0, 0, 0
    last = 0
    for shift in (24, 16, 8, 0):
        sel = inset & ((keys & np.uint32(msk)) == np.uint32(pre))
        d = (keys[sel] >> np.uint32(shift)) & np.uint32(255)
        cnt = np.bincount(d, minlength=256)
        sm = np.zeros(256, np.uint64)
        np.add.at(sm, d, f[sel])
        acc, pick, lowest = above, -1, -1
        for b in range(255, -1, -1):
            if not cnt[b]:
                continue
            lowest = b
            if acc + int(sm[b]) >= target:
                pick = b
                break
            acc += int(sm[b])
        if pick < 0:
            pick = max(lowest, 0)
            acc -= int(sm[pick])
        above = acc
        pre |= pick << shift
        msk |= 255 << shift
        last = int(cnt[pick])
    return pre, above, last


def need(target, above, key, cap):
    f = int(fx(np.uint32(key).view(np.float32)))
    if target <= above:
        return 1
    if not f:
        return cap
    return max(1, min(cap, -(-(target - above) // f)))


def mth_equal(p, key, m):
    idx = np.nonzero(np.asarray(p, np.float32).view(np.uint32) == np.uint32(key))[0]
    return int(idx[m - 1])


def kernel_pick(p, top_p, u):
    """The kernel's token for probabilities p, top_p and the unit draw u."""
    t1 = int(np.float64(np.float32(top_p)) * FIX)
    tau, above1, c1 = radix_select(p, t1)
    j1 = need(t1, above1, tau, c1)
    cum = np.float32((above1 + j1 * int(fx(np.uint32(tau).view(np.float32)))) / FIX)
    r = np.float32(np.float32(u) * cum)
    t2 = int(fx(r))
    if above1 >= t2 and above1 > 0:
        kap, above2, c2 = radix_select(p, t2, kmin=tau)
        return mth_equal(p, kap, need(t2, above2, kap, c2))
    return mth_equal(p, tau, need(t2, above1, tau, j1))


def direct_pick(p, top_p, u):
    """Sort descending (ties by index), exact running sums, first crossings."""
    p = np.asarray(p, np.float32)
    order = np.lexsort((np.arange(p.size), -p.astype(np.float64)))
    c = np.cumsum(fx(p[order]).astype(object))
    t1 = int(np.float64(np.float32(top_p)) * FIX)
    k = next((i for i, v in enumerate(c) if v >= t1), p.size - 1)
    cum = np.float32(c[k] / FIX)
    t2 = int(fx(np.float32(np.float32(u) * cum)))
    j = next((i for i in range(k + 1) if c[i] >= t2), k)
    return int(order[j])


def probs(logits, temp):
    v = (np.asarray(logits, np.float32) * np.float32(1.0 / temp)).astype(np.float32)
    e = np.exp((v - v.max()).astype(np.float32)).astype(np.float32)
    return (e * np.float32(1.0 / e.astype(np.float64).sum())).astype(np.float32)


@pytest.mark.parametrize("case", ["normal", "peaked", "flat", "ties", "uniform", "underflow", "top1"])
def test_selection_matches_direct_definition(case):
    rng = np.random.default_rng(sum(map(ord, case)))
    n, temp, top_p = 3000, 0.7, 0.95
    if case == "normal":
        lg = rng.standard_normal(n) * 2
    elif case == "peaked":
        lg = rng.standard_normal(n) * 8
    elif case == "flat":
        lg = rng.standard_normal(n) * 0.1
    elif case == "ties":
        lg = np.round(rng.standard_normal(n) * 2, 1)     # many equal logits
    elif case == "uniform":
        lg = np.zeros(n)
    elif case == "underflow":
        lg = rng.standard_normal(n) * 3
        temp = 0.02                                      # most probabilities are exactly 0
    else:
        lg = rng.standard_normal(n) * 2
        top_p = 1.0                                      # the mass may never reach 1: all tokens
    p = probs(lg, temp)
    for u in list(rng.random(40)) + [0.0, 1.0 - 2 ** -24]:
        assert kernel_pick(p, top_p, u) == direct_pick(p, top_p, u), (case, u)
