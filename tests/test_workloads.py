"""CPU: the synthetic workloads of the bench (flash_deepseek_b200.workloads).
The Zipf(1.1) logit bias is seeded and deterministic, follows its rank
profile, and gives config 3 the expert-load skew the measurements rely on:
at B = 64 about 80 routed experts are hit and the hottest ones get tens of
tokens (routing by the oracle's restatement of route(), infer.m:920-991)."""
import math

import numpy as np

from flash_deepseek_b200 import workloads as W


def test_zipf_bias_is_seeded_and_follows_the_rank_profile():
    a, b = W.zipf_logit_bias(), W.zipf_logit_bias()
    assert np.array_equal(a, b)
    assert not np.array_equal(a, W.zipf_logit_bias(seed=1))
    beta = W.LOGIT_STD * math.sqrt(6.0) / math.pi
    p = np.arange(1, W.E + 1, dtype=np.float64) ** -1.1
    p /= p.sum()
    expect = np.sort(beta * np.log(W.E * p))[::-1]
    assert np.allclose(np.sort(a.astype(np.float64))[::-1], expect, rtol=1e-6, atol=1e-6)


def test_zipf_skew_of_config3(oracle):
    O = oracle
    router = O.normal(0, O.stream(0, 0, O.KIND_ROUTER), W.E * W.H, W.ROUTER_SIGMA).reshape(W.E, W.H)
    bias = O.normal(0, O.stream(0, 0, O.KIND_BIAS), W.E, W.BIAS_SIGMA)
    lb = W.zipf_logit_bias()
    x = W.tokens(64)
    logits = (x.astype(np.float64) @ router.astype(np.float64).T + lb).astype(np.float32)
    counts = np.zeros(W.E, int)
    for t in range(64):
        idx, _ = O.route(logits[t], bias, 8, 4, W.K, 2.5)
        counts[idx] += 1
    hit = int((counts > 0).sum())
    assert 60 <= hit <= 110, hit                          # load still spreads over many experts
    assert counts.max() >= 30, counts.max()               # the hottest expert is a multi-chunk one
    assert np.sort(counts)[::-1][:4].sum() >= 100, np.sort(counts)[::-1][:8]
