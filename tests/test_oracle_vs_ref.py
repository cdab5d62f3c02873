"""Pins the C oracle bit-for-bit to the reference engine itself.

oracle/_ref/libverbum_ref.so is the unmodified reference (core/src/*.cpp)
compiled by oracle/Makefile.  Every comparison here is exact equality of the
float32 / int8 bit patterns, so any later change to the oracle that drifts
from the reference's arithmetic fails loudly.  Also checks the committed
fixtures of tests/golden/mini_ref.npz (made from the same library).
"""
import json
import tempfile

import numpy as np
import pytest

import oracle
import vbsynth
from conftest import GOLDEN, mini_config

needs_ref = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")


def rng(seed):
    return np.random.default_rng(seed)


@needs_ref
def test_matmul_nt_bitexact():
    A = rng(1).standard_normal((3, 1024)).astype(np.float32)
    B = (rng(2).standard_normal((257, 1024)) * 0.02).astype(np.float32)
    assert np.array_equal(oracle.matmul_nt(A, B), oracle.ref_matmul_nt(A, B))


@needs_ref
@pytest.mark.parametrize("shape", [(64, 1024), (33, 3072), (7, 100)])
def test_quantize_rows_bitexact(shape):
    W = (rng(3).standard_normal(shape) * 0.02).astype(np.float32)
    W[0, :] = 0.0  # an all-zero row takes the scale = 1 branch
    q0, s0 = oracle.quantize_rows(W)
    q1, s1 = oracle.ref_quantize_rows(W)
    assert np.array_equal(q0, q1)
    assert np.array_equal(s0.view(np.uint32), s1.view(np.uint32))


@needs_ref
def test_quantize_rows_ties_round_half_even():
    # values that land exactly on .5 after scaling: lrintf rounds to even
    row = np.array([[127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 63.5]], np.float32)
    q0, _ = oracle.quantize_rows(row)
    q1, _ = oracle.ref_quantize_rows(row)
    assert np.array_equal(q0, q1)
    assert list(q0[0, 1:7]) == [0, 2, 2, 0, -2, -2]


@needs_ref
def test_matmul_nt_q8_bitexact():
    A = rng(4).standard_normal((2, 3072)).astype(np.float32)
    q, s = oracle.quantize_rows((rng(5).standard_normal((300, 3072)) * 0.02).astype(np.float32))
    assert np.array_equal(oracle.matmul_nt_q8(A, q, s), oracle.ref_matmul_nt_q8(A, q, s))


@needs_ref
def test_rmsnorm_and_rope_table_bitexact():
    x = rng(6).standard_normal((5, 1024)).astype(np.float32)
    w = (1.0 + 0.1 * rng(7).standard_normal(1024)).astype(np.float32)
    assert np.array_equal(oracle.rmsnorm(x, w, 1e-6), oracle.ref_rmsnorm(x, w, 1e-6))
    c0, s0 = oracle.rope_table(128, 4096, 1e6)
    c1, s1 = oracle.ref_rope_table(128, 4096, 1e6)
    assert np.array_equal(c0, c1) and np.array_equal(s0, s1)


def _model_pair(cfg, seed, mode, td):
    w = vbsynth.make_weights(cfg, seed=seed)
    vbsynth.write_model_dir(td, cfg, w)
    ref = oracle.RefModel(td)
    orc = oracle.OracleModel(cfg, w)
    if mode == "int8":
        ref.quantize()
        orc.quantize()
    return ref, orc, w


@needs_ref
@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_model_step_bitexact(mode):
    cfg = mini_config()
    with tempfile.TemporaryDirectory() as td:
        ref, orc, _ = _model_pair(cfg, 21, mode, td)
        ref.reset_cache(12)
        orc.reset_cache(12)
        assert ref.weight_bytes() == orc.weight_bytes()
        tok = 17
        for _ in range(9):
            a = ref.step(tok)
            b = orc.step(tok)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
            tok = oracle.ref_greedy(a)
            assert tok == oracle.argmax(b)
        for layer in range(cfg["num_hidden_layers"]):
            for which in (0, 1):
                assert np.array_equal(ref.kv(layer, which, 12)[:9], orc.kv(layer, which))
        if mode == "int8":
            H, D, hd = cfg["num_attention_heads"], cfg["head_dim"], cfg["hidden_size"]
            q0, s0 = ref.quant_tensor(1, 0, H * D, hd)
            q1, s1 = orc.quant_tensor(1, 0)
            assert np.array_equal(q0, q1) and np.array_equal(s0, s1)


@needs_ref
def test_model_errors_match_reference():
    cfg = mini_config()
    with tempfile.TemporaryDirectory() as td:
        ref, orc, _ = _model_pair(cfg, 22, "f32", td)
        for m in (ref, orc):
            with pytest.raises(RuntimeError, match="call reset_cache"):
                m.step(1)
            m.reset_cache(2)
            m.step(1)
            m.step(2)
            with pytest.raises(RuntimeError, match="kv cache is full"):
                m.step(3)
        orc.reset_cache(4)
        with pytest.raises(RuntimeError, match="token id out of range"):
            orc.step(cfg["vocab_size"])


def test_mini_fixture_reproduced_by_oracle():
    meta = json.loads((GOLDEN / "mini_ref.json").read_text())
    fx = np.load(GOLDEN / "mini_ref.npz")
    cfg = meta["config"]
    w = vbsynth.make_weights(cfg, seed=meta["weights_seed"])
    for mode in ("f32", "int8"):
        m = oracle.OracleModel(cfg, w)
        if mode == "int8":
            m.quantize()
            q, s = m.quant_tensor(0, 1)
            assert np.array_equal(q, fx["l0_k_q"]) and np.array_equal(s, fx["l0_k_s"])
        m.reset_cache(meta["prompt_len"] + meta["greedy"] + 8)
        assert m.weight_bytes() == int(fx[f"weight_bytes_{mode}"])
        steps = [int(t) for t in fx["prompt"]] + [int(t) for t in fx[f"tokens_{mode}"][:-1]]
        for i, t in enumerate(steps):
            lg = m.step(t)
            assert np.array_equal(lg, fx[f"logits_{mode}"][i]), (mode, i)
        assert oracle.argmax(lg) == int(fx[f"tokens_{mode}"][-1])
