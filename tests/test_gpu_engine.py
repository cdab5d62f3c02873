"""Engine-level parity: the B200 decode loop against the reference.

- The small seeded model of tests/golden/mini_ref.json against logits recorded
  from the reference engine itself (tests/golden/mini_ref.npz).
- The full Qwen3-0.6B shape (28 layers, vocab 151936) against the C oracle
  (bit-exact with the reference, see test_oracle_vs_ref.py) for the
  32-token-prompt + 128-greedy-token f32 run and a 512 + 64 INT8 run.
- decode() (device-side greedy feedback, graph replay) == step() loop.
- KV cache contents, weight_bytes, and the reference's error behaviour.
Bars: f32 logits max-abs <= 1e-3, INT8 logits <= 1e-2, greedy
tokens identical.
"""
import json

import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import GOLDEN, mini_config

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "int8": 1e-2}


def make_engine(cfg, w, mode, max_seq, path=-1):
    """path -1 = the engine's automatic choice; 1 = the per-op CUDA graph."""
    e = vb200.Engine(cfg).load(w)
    if mode == "int8":
        e.quantize()
    e.reset_cache(max_seq)
    e.set_path(path)
    return e


@pytest.fixture(scope="module")
def mini():
    meta = json.loads((GOLDEN / "mini_ref.json").read_text())
    fx = np.load(GOLDEN / "mini_ref.npz")
    w = vbsynth.make_weights(meta["config"], seed=meta["weights_seed"])
    return meta, fx, w


@pytest.mark.parametrize("path", [-1, 1])
@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_mini_model_matches_reference_fixture(mini, mode, path):
    meta, fx, w = mini
    cfg = meta["config"]
    e = make_engine(cfg, w, mode, meta["prompt_len"] + meta["greedy"] + 8, path)
    assert e.weight_bytes() == int(fx[f"weight_bytes_{mode}"])
    steps = [int(t) for t in fx["prompt"]] + [int(t) for t in fx[f"tokens_{mode}"][:-1]]
    for i, t in enumerate(steps):
        lg = e.step(t)
        assert np.max(np.abs(lg - fx[f"logits_{mode}"][i])) <= TOL[mode], (mode, i)
        if i >= meta["prompt_len"] - 1:
            assert int(np.argmax(lg)) == int(fx[f"tokens_{mode}"][i - meta["prompt_len"] + 1])
    e.close()


@pytest.mark.parametrize("path", [-1, 1])
@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_decode_equals_step_loop_and_oracle(mode, path):
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=31)
    prompt = vbsynth.prompt_ids(6, 3, cfg["vocab_size"])
    orc = oracle.OracleModel(cfg, w)
    if mode == "int8":
        orc.quantize()
    orc.reset_cache(64)
    for t in prompt:
        lg = orc.step(int(t))
    ref_toks = []
    for _ in range(40):
        nxt = oracle.argmax(lg)
        ref_toks.append(nxt)
        lg = orc.step(nxt)
    # step() loop
    e = make_engine(cfg, w, mode, 64, path)
    for t in prompt:
        glg = e.step(int(t))
    toks = []
    for i in range(40):
        nxt = int(np.argmax(glg))
        toks.append(nxt)
        glg = e.step(nxt)
    assert toks == ref_toks
    # prefill + decode(): device-side feedback
    e.reset_cache(64)
    plg = e.prefill(prompt, want_logits=True)
    first = int(np.argmax(plg))
    dtoks, dlg = e.decode(first, 40, want_logits=True)
    assert [first] + list(dtoks[:-1]) == ref_toks
    assert np.max(np.abs(dlg - lg)) <= TOL[mode]
    # KV cache rows written by the engine equal the oracle's
    for layer in range(cfg["num_hidden_layers"]):
        for which in (0, 1):
            assert np.max(np.abs(e.read_kv(layer, which) - orc.kv(layer, which))) < 1e-4
    e.close()


def test_errors_match_reference_semantics():
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=32)
    e = vb200.Engine(cfg).load(w)
    with pytest.raises(vb200.VBError, match="call reset_cache"):
        e.step(1)
    e.reset_cache(2)
    e.step(1)
    with pytest.raises(vb200.VBError, match="token id out of range"):
        e.step(cfg["vocab_size"])
    e.step(2)
    with pytest.raises(vb200.VBError, match="kv cache is full"):
        e.step(3)
    assert e.cache_len() == 2
    # positions past the 4096-entry rope table (model.cpp:136-138, nn.cpp:82-84)
    e.reset_cache(4100)
    e.decode(0, 4096)
    with pytest.raises(vb200.VBError, match="outside the rope table"):
        e.step(1)
    e.close()


def _full_run(mode, prompt_len, n_new, seed):
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=seed)
    prompt = vbsynth.prompt_ids(prompt_len, seed + 1, cfg["vocab_size"])
    max_seq = prompt_len + n_new + 8
    orc = oracle.OracleModel(cfg, w)
    if mode == "int8":
        orc.quantize()
    orc.reset_cache(max_seq)
    e = make_engine(cfg, w, mode, max_seq)
    assert e.weight_bytes() == orc.weight_bytes()
    worst = 0.0
    for t in prompt:
        lo = orc.step(int(t))
        lg = e.step(int(t))
        worst = max(worst, float(np.max(np.abs(lo - lg))))
    toks_o, toks_g = [], []
    for _ in range(n_new):
        to, tg = oracle.argmax(lo), int(np.argmax(lg))
        toks_o.append(to)
        toks_g.append(tg)
        lo = orc.step(to)
        lg = e.step(tg)
        worst = max(worst, float(np.max(np.abs(lo - lg))))
    e.close()
    orc.close()
    return worst, toks_o, toks_g


def test_qwen3_full_f32_prompt32_decode128():
    worst, to, tg = _full_run("f32", 32, 128, seed=1234)
    assert tg == to
    assert worst <= TOL["f32"], worst

# The INT8 configuration (512-token prompt) runs over its whole benchmarked
# length, 512 + 512, in test_gpu_parity_full.py.
