"""The oracle's restatement of Sampler::sample (generate.cpp:197-252) against
the reference Sampler itself (oracle/_ref), on the CPU.

Sequences of draws from one generator (std::mt19937_64 seeded like the
reference) over varying logits rows: greedy (temperature <= 0, top_k == 1),
top-k only, top-p only, both, full vocabulary.  Logits are distinct values
(the reference's partial_sort leaves the order of equal values unspecified).
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")

CONFIGS = [  # temperature, top_k, top_p
    (0.8, 40, 0.95),     # the reference defaults
    (0.0, 40, 0.95),     # greedy by temperature
    (1.0, 1, 1.0),       # greedy by top_k
    (1.3, 0, 0.9),       # top-p over the full vocabulary
    (0.7, 5, 1.0),       # top-k only
    (2.0, 1000, 0.5),    # wide k, tight p
    (0.5, 0, 1.0),       # full vocabulary, no cut
]


def distinct_logits(n, vocab, seed, scale=4.0):
    rng = np.random.default_rng(seed)
    rows = []
    for _ in range(n):
        # distinct floats: a permutation of k * 2^-12, shifted
        rows.append(rng.permutation(vocab).astype(np.float32) * np.float32(scale * 2.0 ** -12) - np.float32(2.0))
    return np.stack(rows)


@pytest.mark.parametrize("t,k,p", CONFIGS)
def test_sample_seq_matches_reference(t, k, p):
    lg = distinct_logits(24, 5000, seed=int(100 * t) + k)
    for seed in (0, 12345):
        ref = oracle.ref_sample_seq(lg, t, k, p, seed)
        got = oracle.sample_seq(lg, t, k, p, seed)
        np.testing.assert_array_equal(got, ref)


def test_sample_seq_qwen_vocab():
    lg = distinct_logits(6, 151936, seed=7, scale=16.0)
    ref = oracle.ref_sample_seq(lg, 0.8, 40, 0.95, 42)
    np.testing.assert_array_equal(oracle.sample_seq(lg, 0.8, 40, 0.95, 42), ref)
