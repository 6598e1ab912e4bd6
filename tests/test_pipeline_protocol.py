"""The A-stage hand-off of the prefill GEMM (k_prefill_gemm, moe_prefill.cu)
as a protocol model: dequantizing groups write A stages, the MMA issuer
consumes the K atoms in order, across persistent work items.  mbarrier waits
test a phase parity, which is right only when the awaited phase is the
barrier's current one or the one just completed; a waiter a whole phase early
passes on an old phase, one two phases late waits forever.  Random
interleavings check that every wait of the kernel's mapping (group g owns
stage g and takes atoms g, g + 3, ...) stays within one phase, and that the
mapping it replaced (four groups, atom g of every super-block, over three
stages) does not."""
import numpy as np
import pytest


def run(n_atoms, n_items, n_stages, owner, rng):
    """owner(i) -> (group, stage) of atom i of an item.  Producers and the MMA
    derive the awaited phase from the atom's position, as the kernel does: the
    u-th use of stage s (in atom order) waits for phase u - 1 of a_empty[s]
    and completes phase u of a_full[s].  A wait passes when the barrier's
    completed-phase count has the other parity (the hardware test).  Returns
    (violations, deadlocked): a pass before the phase completed, or the MMA
    finding another atom in the stage."""
    total = n_atoms * n_items
    stage = [owner(a % n_atoms)[1] for a in range(total)]
    group = [owner(a % n_atoms)[0] for a in range(total)]
    use = [0] * total
    cnt = [0] * n_stages
    for a in range(total):
        use[a] = cnt[stage[a]]
        cnt[stage[a]] += 1
    seq = {}
    for a in range(total):
        seq.setdefault(group[a], []).append(a)
    pos = {g: 0 for g in seq}
    full = [0] * n_stages
    empty = [0] * n_stages
    data = [None] * n_stages
    mma, bad = 0, 0

    def passes(done, k):    # parity wait for phase k (k = -1: a fresh barrier's "previous" phase)
        return (done & 1) != (k & 1)

    while mma < total:
        moves = [("p", g) for g in seq if pos[g] < len(seq[g])] + [("m", None)]
        rng.shuffle(moves)
        for kind, g in moves:
            if kind == "p":
                a = seq[g][pos[g]]
                s, k = stage[a], use[a] - 1
                if passes(empty[s], k):
                    if empty[s] < k + 1:
                        bad += 1          # passed before the stage was released
                    data[s] = a
                    full[s] += 1
                    pos[g] += 1
                    break
            else:
                a = mma
                s, k = stage[a], use[a]
                if passes(full[s], k):
                    if full[s] < k + 1 or data[s] != a:
                        bad += 1          # passed early, or another atom sits in the stage
                    empty[s] += 1
                    mma += 1
                    break
        else:
            return bad, True              # nobody can move
    return bad, False


@pytest.mark.parametrize("n_atoms", [8, 32, 112])
def test_one_group_per_stage_keeps_every_wait_within_one_phase(n_atoms):
    rng = np.random.default_rng(n_atoms)
    for trial in range(20):
        bad, dead = run(n_atoms, 3, 3, lambda i: (i % 3, i % 3), rng)
        assert not dead and bad == 0, (trial, bad, dead)


def test_four_groups_over_three_stages_breaks_a_parity_wait():
    rng = np.random.default_rng(1)
    bad = 0
    for trial in range(40):
        b, dead = run(32, 2, 3, lambda i: (i % 4, i % 3), rng)
        bad += b > 0 or dead
    assert bad > 0
