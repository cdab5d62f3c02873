"""The oracle's layer-major prefill (or_model_prefill) against its own
token-by-token step and against the reference engine.

The prefill exists so the batched engine's parity tests can afford 2048-token
prompts on the host: it reads each weight row once per block of positions
instead of once per position.  It must compute exactly what feeding the
tokens one at a time through Model::step computes (tools/generate.cpp:75-77),
so every comparison here is bit-for-bit: logits, the KV caches and the logits
of a step after it, in f32 and INT8, with the prompt split over several calls
(later calls attend over cached positions).
"""
import tempfile

import numpy as np
import pytest

import oracle
import vbsynth

CFG = vbsynth.qwen3_config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                           num_key_value_heads=2, intermediate_size=512, vocab_size=1000)


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_prefill_equals_steps_bitwise(mode):
    w = vbsynth.make_weights(CFG, seed=3, normal=oracle.synth_normal)
    toks = vbsynth.prompt_ids(153, 5, CFG["vocab_size"])
    a, b = oracle.OracleModel(CFG, w), oracle.OracleModel(CFG, w)
    if mode == "int8":
        a.quantize()
        b.quantize()
    a.reset_cache(164)
    b.reset_cache(164)
    for t in toks:
        la = a.step(int(t))
    # chunks of 1, 69 (not a multiple of the 32-position block) and the rest
    b.prefill(toks[:1])
    b.prefill(toks[1:70])
    lb = b.prefill(toks[70:])
    assert np.array_equal(_bits(la), _bits(lb))
    assert a.cache_len() == b.cache_len() == len(toks)
    for layer in range(CFG["num_hidden_layers"]):
        for which in (0, 1):
            assert np.array_equal(_bits(a.kv(layer, which)), _bits(b.kv(layer, which)))
    assert np.array_equal(_bits(a.step(7)), _bits(b.step(7)))
    a.close()
    b.close()


def test_prefill_errors_keep_the_reference_wording():
    w = vbsynth.make_weights(CFG, seed=3, normal=oracle.synth_normal)
    o = oracle.OracleModel(CFG, w)
    with pytest.raises(RuntimeError, match="call reset_cache"):
        o.prefill([1, 2])
    o.reset_cache(4)
    with pytest.raises(RuntimeError, match="kv cache is full"):
        o.prefill([1, 2, 3, 4, 5])
    with pytest.raises(RuntimeError, match="out of range"):
        o.prefill([1, CFG["vocab_size"]])
    assert o.cache_len() == 0
    o.close()


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")
@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_prefill_equals_reference_steps_bitwise(mode):
    w = vbsynth.make_weights(CFG, seed=11, normal=oracle.synth_normal)
    toks = vbsynth.prompt_ids(40, 12, CFG["vocab_size"])
    with tempfile.TemporaryDirectory() as td:
        ref = oracle.RefModel(str(vbsynth.write_model_dir(td, CFG, w)))
        o = oracle.OracleModel(CFG, w)
        if mode == "int8":
            ref.quantize()
            o.quantize()
        ref.reset_cache(48)
        o.reset_cache(48)
        for t in toks:
            lr = ref.step(int(t))
        lo = o.prefill(toks)
        assert np.array_equal(_bits(lr), _bits(lo))
        ref.close()
        o.close()
