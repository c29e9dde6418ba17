"""The sampler's host logic against the reference Sampler (compiled in
oracle/_ref): the xorshift* restatement that advances the GPU sampler's
state (src/inference/Utils.h:18-29) reproduces the reference's coins."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.has_ref_engine(), reason="oracle/_ref not built")

SEEDS = [1, 7, 42, 1234, 99991, 0xDEADBEEF, (1 << 40) + 7, (1 << 63) + 12345]


def test_random_f32_is_the_reference_coin():
    """Uniform logits over 2^20 tokens: every probability is exactly 2^-20,
    the reference's multinomial walk is exact, and its token is
    floor(coin * 2^20) — 20 bits of each coin, for a chain of states."""
    n = 1 << 20
    logits = np.zeros(n, np.float32)
    for seed in SEEDS:
        state = seed
        for _ in range(3):
            coin, nxt = oracle.random_f32(state)
            assert oracle.ref_sample(logits, 1.0, 0.0, state) == int(coin * n), (seed, state)
            state = nxt


def test_reference_topp_picks_from_the_top():
    """A sanity pin of the reference call itself: one dominant token with
    topp 0.5 is always chosen."""
    logits = np.full(1000, -5.0, np.float32)
    logits[321] = 10.0
    for seed in SEEDS:
        assert oracle.ref_sample(logits, 1.0, 0.5, seed) == 321
