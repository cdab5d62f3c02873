"""The persistent clustered decode step (path 2, one launch per token) against
the oracle: f32 and INT8 at full widths with 2 layers and a cache length that
is not a multiple of the 32-position attention chunk, then the full
Qwen3-0.6B shape; and the engine's automatic choice of step path.  Same bars
as the per-op path: f32 logits max-abs <= 1e-3, INT8 <= 1e-2, greedy tokens
identical."""
import numpy as np
import pytest

import oracle
import vb200
import vbsynth

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "int8": 1e-2}


def cfg_wide():
    """Full Qwen3-0.6B widths (hidden 1024, 16/8 heads, ffn 3072), 2 layers,
    small vocab: the shapes the two-barrier clustered step is laid out for."""
    return vbsynth.qwen3_config(num_hidden_layers=2, vocab_size=4096)


def run_pair(cfg, w, mode, prompt, n_new, max_seq, path=2):
    orc = oracle.OracleModel(cfg, w)
    e = vb200.Engine(cfg).load(w)
    if mode == "int8":
        orc.quantize()
        e.quantize()
    orc.reset_cache(max_seq)
    e.reset_cache(max_seq)
    e.set_path(path)
    worst = 0.0
    for t in prompt:
        lo, lg = orc.step(int(t)), e.step(int(t))
        worst = max(worst, float(np.max(np.abs(lo - lg))))
    if path == 2:
        assert e.graph_nodes() == 1, "clustered step did not run"
    to, tg = [], []
    for _ in range(n_new):
        a, b = oracle.argmax(lo), int(np.argmax(lg))
        to.append(a)
        tg.append(b)
        lo, lg = orc.step(a), e.step(b)
        worst = max(worst, float(np.max(np.abs(lo - lg))))
    return e, orc, worst, to, tg


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_two_barrier_step_wide_model(mode):
    """Path 2 on full widths: chunks spread over the cluster (cache length 300
    -> 10 chunks, 2 on some CTAs), KV rows and decode() as well."""
    cfg = cfg_wide()
    w = vbsynth.make_weights(cfg, seed=71)
    prompt = vbsynth.prompt_ids(270, 13, cfg["vocab_size"])
    e, orc, worst, to, tg = run_pair(cfg, w, mode, prompt, 24, 300, path=2)
    assert tg == to and worst <= TOL[mode], worst
    for layer in range(cfg["num_hidden_layers"]):
        for which in (0, 1):
            assert np.max(np.abs(e.read_kv(layer, which) - orc.kv(layer, which))) < 1e-4
    e.reset_cache(300)
    lg = e.prefill(prompt, want_logits=True)
    toks = e.decode(int(np.argmax(lg)), 24)
    assert [int(np.argmax(lg))] + list(toks[:-1]) == to
    # errors keep the reference's wording on this path too
    with pytest.raises(vb200.VBError, match="kv cache is full"):
        e.decode(0, 10)
    e.close()


def test_clustered_full_f32_prompt32_decode128():
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=1234)
    prompt = vbsynth.prompt_ids(32, 1235, cfg["vocab_size"])
    e, orc, worst, to, tg = run_pair(cfg, w, "f32", prompt, 128, 168, path=2)
    assert tg == to and worst <= TOL["f32"], worst
    e.close()


def test_per_op_full_int8_prompt512_decode64():
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=4321)
    prompt = vbsynth.prompt_ids(512, 4322, cfg["vocab_size"])
    e, orc, worst, to, tg = run_pair(cfg, w, "int8", prompt, 64, 584, path=1)
    assert tg == to and worst <= TOL["int8"], worst
    assert e.graph_nodes() > 1
    e.close()


def test_automatic_path_is_the_measured_fastest():
    """set_path(-1) (the default) takes the per-op graph for f32 weights and
    the clustered step for INT8 -- the faster of each on B200 -- and path 0
    (a removed implementation) is refused."""
    cfg = cfg_wide()
    w = vbsynth.make_weights(cfg, seed=3)
    e = vb200.Engine(cfg).load(w)
    e.reset_cache(16)
    assert e.path() == 1
    e.step(1)
    assert e.graph_nodes() > 1
    with pytest.raises(vb200.VBError):
        e.set_path(0)
    e.set_path(2)
    assert e.path() == 2
    e.set_path(-1)
    e.quantize()
    e.reset_cache(16)
    assert e.path() == 2
    e.step(1)
    assert e.graph_nodes() == 1
    e.close()
