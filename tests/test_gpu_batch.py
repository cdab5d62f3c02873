"""Batched independent-sequence decode against the oracle, per sequence.

B sequences share one engine's weights; each must produce exactly the
logits / greedy tokens the reference gives that sequence alone.
"""
import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import mini_config

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "int8": 1e-2}


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_batch_matches_per_sequence_oracle(mode):
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=41)
    B, P, G = 5, 7, 12
    prompts = np.stack([vbsynth.prompt_ids(P, 100 + b, cfg["vocab_size"]) for b in range(B)])
    eng = vb200.Engine(cfg).load(w)
    if mode == "int8":
        eng.quantize()
    bt = vb200.Batch(eng, B, P + G + 4)
    # step() API with logits, position by position
    for t in range(P):
        lg, nx = bt.step(prompts[:, t])
    orcs = []
    for b in range(B):
        o = oracle.OracleModel(cfg, w)
        if mode == "int8":
            o.quantize()
        o.reset_cache(P + G + 4)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        assert np.max(np.abs(lo - lg[b])) <= TOL[mode]
        assert oracle.argmax(lo) == int(nx[b])
        orcs.append((o, lo))
    # greedy continuation on the device vs the oracle
    nxt = bt.decode(nx, G)
    for b, (o, lo) in enumerate(orcs):
        tok = oracle.argmax(lo)
        for _ in range(G):
            lo = o.step(tok)
            tok = oracle.argmax(lo)
        assert tok == int(nxt[b]), b
        o.close()
    # prefill API == step API
    bt.reset()
    nx2 = bt.prefill(prompts.T.copy())
    assert np.array_equal(nx2, nx)
    assert bt.cache_len() == P
    # rolled back to P positions, the same continuation comes out again
    bt.decode(nx, 3)
    bt.truncate(P)
    assert bt.cache_len() == P
    assert np.array_equal(bt.decode(nx, G), nxt)
    with pytest.raises(vb200.VBError):
        bt.truncate(P + G + 1)
    bt.close()
    eng.close()


def test_batch64_full_model_two_sequences():
    """Full Qwen3-0.6B INT8, 64 sequences; sequences 0 and 63 checked."""
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=55)
    B, P, G = 64, 24, 6
    prompts = np.stack([vbsynth.prompt_ids(P, 500 + b, cfg["vocab_size"]) for b in range(B)])
    eng = vb200.Engine(cfg).load(w)
    eng.quantize()
    bt = vb200.Batch(eng, B, P + G + 4)
    nx = bt.prefill(prompts.T.copy())
    nxt = bt.decode(nx, G)
    for b in (0, B - 1):
        o = oracle.OracleModel(cfg, w)
        o.quantize()
        o.reset_cache(P + G + 4)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        tok = oracle.argmax(lo)
        assert tok == int(nx[b])
        for _ in range(G):
            tok = oracle.argmax(o.step(tok))
        assert tok == int(nxt[b])
        o.close()
    bt.close()
    eng.close()


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_batch33_matches_oracle(mode):
    """33 sequences (one more than a 32-row tile half): sequences at the ends
    and in the middle give the oracle's logits and greedy tokens."""
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=43)
    B, P, G = 33, 6, 5
    prompts = np.stack([vbsynth.prompt_ids(P, 300 + b, cfg["vocab_size"]) for b in range(B)])
    eng = vb200.Engine(cfg).load(w)
    if mode == "int8":
        eng.quantize()
    bt = vb200.Batch(eng, B, P + G + 4)
    for t in range(P):
        lg, nx = bt.step(prompts[:, t])
    nxt = bt.decode(nx, G)
    for b in (0, 15, 16, 32):
        o = oracle.OracleModel(cfg, w)
        if mode == "int8":
            o.quantize()
        o.reset_cache(P + G + 4)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        assert np.max(np.abs(lo - lg[b])) <= TOL[mode], b
        tok = oracle.argmax(lo)
        assert tok == int(nx[b]), b
        for _ in range(G):
            tok = oracle.argmax(o.step(tok))
        assert tok == int(nxt[b]), b
        o.close()
    bt.close()
    eng.close()


def test_batch_full_model_f32_matches_oracle():
    """Full Qwen3-0.6B with f32 weights (bf16 pair operands, one GEMM CTA per
    SM, the q|k|v splits summed in 4-CTA clusters with the q/k norm), 8
    sequences: sequences 0 and 7 against the oracle's logits and picks."""
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=57)
    B, P, G = 8, 5, 3
    prompts = np.stack([vbsynth.prompt_ids(P, 700 + b, cfg["vocab_size"]) for b in range(B)])
    eng = vb200.Engine(cfg).load(w)
    bt = vb200.Batch(eng, B, P + G + 4)
    for t in range(P):
        lg, nx = bt.step(prompts[:, t])
    nxt = bt.decode(nx, G)
    for b in (0, B - 1):
        o = oracle.OracleModel(cfg, w)
        o.reset_cache(P + G + 4)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        assert np.max(np.abs(lo - lg[b])) <= TOL["f32"], b
        tok = oracle.argmax(lo)
        assert tok == int(nx[b]), b
        for _ in range(G):
            tok = oracle.argmax(o.step(tok))
        assert tok == int(nxt[b]), b
        o.close()
    bt.close()
    eng.close()
