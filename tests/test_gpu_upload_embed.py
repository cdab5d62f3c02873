"""bf16 weight uploads widened on the device, and Model::embed_text
(model.cpp:191-233) on the device, against the reference.

bf16 -> f32 widening is exact (safetensors.cpp:59-66), so an engine loaded
from bf16 bit patterns holds exactly the weights of one loaded from the
widened f32 arrays: its logits must be bit-identical.  embed_text runs the
prompt's layers through the batched prefill path (tensor-core GEMMs and
attention), so it matches the reference's embed_text to f32 rounding.
"""
import tempfile

import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import mini_config

pytestmark = pytest.mark.gpu


def to_bf16_bits(a):
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def test_bf16_upload_matches_f32_upload():
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=91)
    wb = {k: to_bf16_bits(v) for k, v in w.items()}
    wf = {k: from_bf16_bits(v) for k, v in wb.items()}
    a = vb200.Engine(cfg).load_bf16(wb)
    b = vb200.Engine(cfg).load(wf)
    a.reset_cache(16)
    b.reset_cache(16)
    for t in vbsynth.prompt_ids(5, 3, cfg["vocab_size"]):
        assert np.array_equal(a.step(int(t)), b.step(int(t)))
    a.close()
    b.close()


@pytest.mark.parametrize("n", [1, 7, 70])
def test_embed_text_matches_reference(n):
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built")
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=93)
    ids = vbsynth.prompt_ids(n, 11 + n, cfg["vocab_size"])
    with tempfile.TemporaryDirectory() as td:
        vbsynth.write_model_dir(td, cfg, w)
        ref = oracle.RefModel(td)
        want = ref.embed_text(ids, cfg["hidden_size"])
        ref.close()
    e = vb200.Engine(cfg).load(w)
    got = e.embed_text(ids)
    assert abs(float(np.linalg.norm(got)) - 1.0) < 1e-5
    assert np.max(np.abs(got - want)) < 1e-4
    e.quantize()
    with pytest.raises(vb200.VBError):
        e.embed_text(ids)  # the reference: "embed_text needs the f32 path"
    e.close()


def test_embed_text_rejects_empty():
    cfg = mini_config()
    e = vb200.Engine(cfg).load(vbsynth.make_weights(cfg, seed=95))
    with pytest.raises(vb200.VBError):
        e.embed_text([])
    e.close()
