"""Opt-in INT8 tied lm_head (no reference counterpart; the reference keeps
the lm_head in f32, model.cpp:313-338) against the oracle with the same
opt-in (the embedding rows through quantize_rows, the product as
matmul_nt_q8): logits within the INT8 bar, greedy tokens identical, on every
step path, for f32 and INT8 projections, and for a batch.
"""
import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import mini_config

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.mark.parametrize("mode,path", [("int8", -1), ("int8", 1), ("f32", -1), ("f32", 1), ("int8", 2)])
def test_engine_lm_int8_matches_oracle(mode, path):
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=81)
    e = vb200.Engine(cfg).load(w)
    o = oracle.OracleModel(cfg, w)
    if mode == "int8":
        e.quantize()
        o.quantize()
    e.quantize_lm_head()
    o.quantize_lm_head()
    e.set_path(path)
    e.reset_cache(32)
    o.reset_cache(32)
    prompt = vbsynth.prompt_ids(6, 9, cfg["vocab_size"])
    for t in prompt:
        lg = e.step(int(t))
        lo = o.step(int(t))
        assert np.max(np.abs(lg - lo)) <= TOL
    first = int(np.argmax(lg))
    assert first == oracle.argmax(lo)
    toks = e.decode(first, 8)
    tok = first
    for i in range(8):
        tok = oracle.argmax(o.step(tok))
        assert tok == int(toks[i]), i
    o.close()
    e.close()


def test_batch_lm_int8_matches_oracle():
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=83)
    e = vb200.Engine(cfg).load(w)
    e.quantize()
    e.quantize_lm_head()
    B, P = 3, 9
    prompts = np.stack([vbsynth.prompt_ids(P, 40 + b, cfg["vocab_size"]) for b in range(B)])
    bt = vb200.Batch(e, B, P + 8)
    nx = bt.prefill(prompts.T.copy())
    lg, _ = bt.step(nx)
    for b in range(B):
        o = oracle.OracleModel(cfg, w)
        o.quantize()
        o.quantize_lm_head()
        o.reset_cache(P + 8)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        assert oracle.argmax(lo) == int(nx[b])
        lo = o.step(int(nx[b]))
        assert np.max(np.abs(lo - lg[b])) <= TOL
        o.close()
    bt.close()
    e.close()
