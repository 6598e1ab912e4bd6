"""CPU emulation of the routing warp of k_route_plan (moe_kernels.cu) against
the oracle's route() (infer.m:920-991): the group scores, the top groups
taken by direct rank (instead of repeated argmax), and the slot-order top-K
whose minimum is found by a warp min-reduction over lane-held slots with an
order-preserving integer key.  The oracle is fed logits of -1e30 (sigmoid
exactly 0) and the choice scores as its bias, so both sides rank the same
fp32 values.  The GPU tests check the kernel itself; this pins the algorithm
(slot order included) on random, tied and degenerate inputs."""
import numpy as np
import pytest

F32 = np.float32
NEG = F32(-1e30)
BIG = F32(3.0e38)


def f32_ord(v):
    """The kernel's f32_ord: int32 bits, negative values with the magnitude bits flipped."""
    i = np.asarray(v, F32).view(np.int32).astype(np.int64)
    return np.where(i >= 0, i, i ^ 0x7FFFFFFF)


def group_scores(choice, G, per):
    gs = np.empty(G, F32)
    for g in range(G):
        v = np.sort(choice[g * per:(g + 1) * per])[::-1]
        gs[g] = F32(v[0]) + (F32(v[1]) if per >= 2 else NEG)   # top1 + top2, with multiplicity
    return gs


def top_groups_by_rank(gs, TG):
    G = gs.size
    taken = []
    for g in range(G):
        v = gs[g]
        rank = sum(1 for h in range(G) if gs[h] > v or (gs[h] == v and h < g))
        if v > NEG and rank < TG:
            taken.append(g)
    return taken


def topk_slots(choice, taken, per, K):
    """Lane k < K holds slot k; 32 candidates per batch; the first one above
    the current minimum replaces the first lane holding that minimum."""
    sv = np.array([NEG if k < K else BIG for k in range(32)], F32)
    si = np.zeros(32, np.int64)
    mkey, mk = NEG, 0
    for g in taken:
        for e0 in range(g * per, (g + 1) * per, 32):
            c = np.array([choice[e0 + l] if e0 + l < (g + 1) * per else NEG for l in range(32)], F32)
            rem = np.ones(32, bool)
            while True:
                bal = (c > mkey) & rem
                if not bal.any():
                    break
                f = int(np.argmax(bal))
                sv[mk], si[mk] = c[f], e0 + f
                o = f32_ord(sv)
                mk = int(np.argmax(o == o.min()))
                mkey = sv[mk]
                rem = np.arange(32) > f
    return si[:K]


def emulate(choice, G, TG, K):
    per = choice.size // G
    return topk_slots(choice, top_groups_by_rank(group_scores(choice, G, per), TG), per, K)


def oracle_slots(oracle, choice, G, TG, K):
    idx, _ = oracle.route(np.full(choice.size, -1e30, F32), choice, G, TG, K, 2.5)
    return idx


CASES = [(256, 8, 4, 8), (16, 4, 2, 4), (256, 4, 2, 8), (64, 2, 1, 6), (128, 8, 8, 16)]


@pytest.mark.parametrize("E,G,TG,K", CASES)
def test_routing_warp_matches_oracle_slot_order(oracle, E, G, TG, K):
    rng = np.random.default_rng(E * 131 + G * 17 + TG * 7 + K)
    for trial in range(60):
        kind = trial % 4
        if kind == 0:      # continuous scores
            choice = rng.normal(0.5, 0.2, E).astype(F32)
        elif kind == 1:    # few levels: exact ties inside and across groups
            choice = rng.integers(0, 4, E).astype(F32) * F32(0.25)
        elif kind == 2:    # near ties (1e-7 apart)
            choice = (F32(0.5) + rng.integers(0, 5, E).astype(F32) * F32(1e-7)).astype(F32)
        else:              # one hot group, the rest negative
            choice = rng.normal(-1.0, 0.1, E).astype(F32)
            g = int(rng.integers(0, G))
            choice[g * (E // G):(g + 1) * (E // G)] += F32(2.0)
        got = emulate(choice, G, TG, K)
        want = oracle_slots(oracle, choice, G, TG, K)
        assert np.array_equal(got, want), (trial, kind, got, want)


def test_all_equal_scores(oracle):
    choice = np.full(256, F32(0.3))
    assert np.array_equal(emulate(choice, 8, 4, 8), oracle_slots(oracle, choice, 8, 4, 8))


def test_f32_ord_preserves_order():
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-30, 500), rng.normal(0, 1e30, 500),
                        [1e-45, -1e-45, 3.0e38, -3.0e38, -1e30, 1e30, np.inf, -np.inf, 0.0]]).astype(F32)
    a, b = v[:, None], v[None, :]
    oa, ob = f32_ord(v)[:, None], f32_ord(v)[None, :]
    assert np.array_equal(a < b, oa < ob)
    # the kernel's f32_unord inverts it exactly
    o = f32_ord(v)
    back = np.where(o >= 0, o, o ^ 0x7FFFFFFF).astype(np.int64).astype(np.int32).view(F32)
    assert np.array_equal(back.view(np.int32), v.view(np.int32))
