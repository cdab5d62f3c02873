"""Device sampling (Sampler::sample, generate.cpp:197-252) against the
oracle's restatement, which tests/test_sampler_oracle.py pins to the
reference Sampler.

The host draws from std::mt19937_64(seed) exactly as the reference does (one
uniform double per non-greedy call), so a seeded device sampler must pick the
reference's token sequence.  Configurations cover greedy, top-k only, top-p
only, both, the full 151,936-entry vocabulary (parallel sums on the device),
and a sampled decode loop of the engine.
"""
import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import mini_config
from test_sampler_oracle import CONFIGS, distinct_logits

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("t,k,p", CONFIGS)
def test_device_sampler_matches_oracle(t, k, p):
    lg = distinct_logits(24, 5000, seed=int(100 * t) + k)
    dev = torch.from_numpy(lg).cuda()
    for seed in (0, 12345):
        want = oracle.sample_seq(lg, t, k, p, seed)
        s = vb200.Sampler(t, k, p, seed)
        got = [s.sample(dev[i]) for i in range(len(lg))]
        s.close()
        np.testing.assert_array_equal(np.array(got), want)


@pytest.mark.parametrize("t,k,p", [(0.8, 40, 0.95), (1.2, 0, 0.9), (0.9, 2000, 1.0)])
def test_device_sampler_qwen_vocab(t, k, p):
    lg = distinct_logits(8, 151936, seed=3 + k, scale=16.0)
    dev = torch.from_numpy(lg).cuda()
    want = oracle.sample_seq(lg, t, k, p, 99)
    s = vb200.Sampler(t, k, p, 99)
    got = [s.sample(dev[i]) for i in range(len(lg))]
    s.close()
    np.testing.assert_array_equal(np.array(got), want)


@pytest.mark.parametrize("path", [-1, 1])
def test_engine_decode_sampled_matches_oracle(path):
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=71)
    T, K, P, seed, n = 0.8, 40, 0.95, 2024, 16
    eng = vb200.Engine(cfg).load(w)
    eng.set_path(path)
    eng.reset_cache(n + 8)
    s = vb200.Sampler(T, K, P, seed)
    got = eng.decode_sampled(s, 17, n)
    o = oracle.OracleModel(cfg, w)
    o.reset_cache(n + 8)
    rows, want, tok = [], [], 17
    for _ in range(n):
        rows.append(o.step(tok))
        tok = int(oracle.sample_seq(np.stack(rows), T, K, P, seed)[-1])
        want.append(tok)
    np.testing.assert_array_equal(got, np.array(want))
    # greedy settings take the greedy decode
    eng.reset_cache(n + 8)
    g = vb200.Sampler(0.0, 40, 0.95, seed)
    np.testing.assert_array_equal(eng.decode_sampled(g, 17, 8), eng_greedy(cfg, w, path, 17, 8))
    o.close()
    s.close()
    g.close()
    eng.close()


def eng_greedy(cfg, w, path, first, n):
    e = vb200.Engine(cfg).load(w)
    e.set_path(path)
    e.reset_cache(n + 8)
    toks = e.decode(first, n)
    e.close()
    return toks


def test_device_sampler_ties_at_the_threshold():
    """More than 4096 logits tie with the k-th largest: the selection fallback
    (ties ordered by index, like the oracle)."""
    V = 20000
    rng = np.random.default_rng(5)
    lg = np.full((6, V), 1.0, np.float32)
    for r in lg:
        r[rng.choice(V, 10, replace=False)] = np.float32(2.0) + rng.permutation(10).astype(np.float32)
    dev = torch.from_numpy(lg).cuda()
    want = oracle.sample_seq(lg, 0.9, 40, 0.95, 3)
    s = vb200.Sampler(0.9, 40, 0.95, 3)
    got = [s.sample(dev[i]) for i in range(len(lg))]
    s.close()
    np.testing.assert_array_equal(np.array(got), want)
