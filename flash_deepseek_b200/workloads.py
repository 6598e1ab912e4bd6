"""Synthetic workloads of the reference's headline configurations (configs
1-5: one expert, one layer at batch 1 and 64, the 58-layer stack, a
4096-token prefill) for tests and bench.py: shapes, seeds and the Zipf
expert-load skew.  Weights are random-init N(0, 0.02) quantized to Q4_K
(gate/up) and Q6_K or Q4_K (down); router N(0, 0.006), selection bias
N(0, 0.01); tokens N(0, 1)."""
from __future__ import annotations

import math

import numpy as np

H, I, E, K = 7168, 2048, 256, 8
W_SIGMA, ROUTER_SIGMA, BIAS_SIGMA = 0.02, 0.006, 0.01
# standard deviation of a router logit W_r h with W_r ~ N(0, 0.006), h ~ N(0, 1)
LOGIT_STD = ROUTER_SIGMA * math.sqrt(H)


def zipf_logit_bias(n: int = E, s: float = 1.1, seed: int = 0, beta: float | None = None) -> np.ndarray:
    """Per-expert term added to the router logits so that expert load follows
    a Zipf(s) profile: expert e gets rank pi(e) of a seeded permutation and
    bias beta * log(n * p_pi(e)), p_r proportional to r^-s.  beta defaults to
    the Gumbel scale of the logit noise (LOGIT_STD * sqrt(6) / pi), under which
    a logit offset of log p multiplies the selection odds by about p."""
    if beta is None:
        beta = LOGIT_STD * math.sqrt(6.0) / math.pi
    rng = np.random.default_rng(seed)
    p = np.arange(1, n + 1, dtype=np.float64) ** -s
    p /= p.sum()
    return (beta * np.log(n * p[rng.permutation(n)])).astype(np.float32)


def tokens(batch: int, seed: int = 1234) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((batch, H)).astype(np.float32)


def token_pool(batch: int, n_pool: int = 4, seed: int = 1234) -> list:
    """n_pool batches of N(0, 1) tokens [batch, H] from one generator, in
    order: the inputs of bench.py's GPU steps (step s uses batch s % n_pool)
    and, token by token in the same order, of its CPU reference arm."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((batch, H)).astype(np.float32) for _ in range(n_pool)]
