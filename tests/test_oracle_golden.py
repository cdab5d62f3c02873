"""Pins the C oracle to the reference's own golden vectors and known answers.

Mirrors the reference's CPU tests case for case:
  tests/test_nn.cpp:104-151        rmsnorm (1e-5) and rope (1e-4) vs reference_nn.json
  tests/test_attention.cpp:57-111  GQA attention with QK-norm + RoPE (1e-5) vs reference_attn.json
  tests/test_block.cpp:41-110      SwiGLU FFN and a full pre-norm layer (1e-5) vs reference_block.json
  tests/test_cache.cpp:30-81       token-by-token KV-cache decode == full attention (1e-5)
  tests/test_quant.cpp:42-141      quantisation known answers and error bounds
  tests/test_cache.cpp:83-93       greedy sampling = argmax
The attention and layer cases are run through the oracle's DECODE path (one
token at a time against a KV cache), which is the path the engine accelerates;
matching the reference's full-sequence golden outputs within 1e-5 is the
structural-equivalence check of test_cache.cpp.
"""
import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.skipif(not oracle.have_oracle(), reason="liboracle.so not built")


def cases(group):
    index = json.loads((GOLDEN / "reference_cases.json").read_text())[group]
    arr = np.load(GOLDEN / "reference_vectors.npz")
    for i, meta in enumerate(index):
        d = dict(meta)
        pre = f"{group}_{i}_"
        for k in arr.files:
            if k.startswith(pre):
                d[k[len(pre):]] = arr[k]
        yield d


def maxdiff(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


@pytest.mark.parametrize("case", list(cases("rmsnorm")), ids=lambda c: f"{c['rows']}x{c['dim']}")
def test_rmsnorm_golden(case):
    x = case["x"].reshape(case["rows"], case["dim"])
    y = oracle.rmsnorm(x, case["w"], case["eps"])
    assert maxdiff(y.ravel(), case["y"]) < 1e-5


@pytest.mark.parametrize("case", list(cases("rope")), ids=lambda c: f"D{c['head_dim']}p{c['pos']}")
def test_rope_golden(case):
    c, s = oracle.rope_table(case["head_dim"], 64, case["theta"])
    x = case["x"].reshape(case["heads"], case["head_dim"])
    y = oracle.apply_rope(x, case["pos"], c, s)
    assert maxdiff(y.ravel(), case["y"]) < 1e-4


def attention_decode_seq(x, wq, wk, wv, wo, qn, kn, H, KVH, D, eps, theta):
    """generate.cpp:24-108 applied token by token with a growing KV cache."""
    seq, hidden = x.shape
    wq, wk, wv = wq.reshape(H * D, hidden), wk.reshape(KVH * D, hidden), wv.reshape(KVH * D, hidden)
    wo = wo.reshape(hidden, H * D)
    cos, sin = oracle.rope_table(D, seq + 8, theta)
    kc = np.zeros((seq, KVH * D), np.float32)
    vc = np.zeros((seq, KVH * D), np.float32)
    out = np.zeros((seq, hidden), np.float32)
    for t in range(seq):
        xt = x[t:t + 1]
        q = oracle.rmsnorm(oracle.matmul_nt(xt, wq).reshape(H, D), qn, eps)
        k = oracle.rmsnorm(oracle.matmul_nt(xt, wk).reshape(KVH, D), kn, eps)
        v = oracle.matmul_nt(xt, wv)
        q = oracle.apply_rope(q, t, cos, sin)
        k = oracle.apply_rope(k, t, cos, sin)
        kc[t] = k.ravel()
        vc[t] = v.ravel()
        ctx = oracle.attention_decode(q, kc, vc, H, KVH, D, t + 1)
        out[t] = oracle.matmul_nt(ctx.reshape(1, -1), wo)[0]
    return out


@pytest.mark.parametrize("case", list(cases("attention")), ids=lambda c: f"KVH{c['KVH']}D{c['D']}")
def test_attention_golden_via_decode(case):
    x = case["x"].reshape(case["seq"], case["hidden"])
    y = attention_decode_seq(x, case["wq"], case["wk"], case["wv"], case["wo"], case["qn"],
                             case["kn"], case["H"], case["KVH"], case["D"], case["eps"],
                             case["theta"])
    assert maxdiff(y.ravel(), case["y"]) < 1e-5


def ffn(x, g, u, d, hidden, F):
    gate = oracle.matmul_nt(x, g.reshape(F, hidden))
    up = oracle.matmul_nt(x, u.reshape(F, hidden))
    return oracle.matmul_nt(oracle.silu_mul(gate, up), d.reshape(hidden, F))


@pytest.mark.parametrize("case", list(cases("ffn")), ids=lambda c: f"h{c['hidden']}")
def test_ffn_golden(case):
    x = case["x"].reshape(case["seq"], case["hidden"])
    y = ffn(x, case["g"], case["u"], case["d"], case["hidden"], case["ffn"])
    assert maxdiff(y.ravel(), case["y"]) < 1e-5


@pytest.mark.parametrize("case", list(cases("layer")), ids=lambda c: f"h{c['hidden']}")
def test_layer_golden_via_decode(case):
    """model.cpp:235-254 (layer_step) run per token."""
    seq, hidden, eps = case["seq"], case["hidden"], case["eps"]
    x = case["x"].reshape(seq, hidden)
    normed = oracle.rmsnorm(x, case["inorm"], eps)
    attn = attention_decode_seq(normed, case["wq"], case["wk"], case["wv"], case["wo"], case["qn"],
                                case["kn"], case["H"], case["KVH"], case["D"], eps, case["theta"])
    h = (x + attn).astype(np.float32)
    out = h + ffn(oracle.rmsnorm(h, case["pnorm"], eps), case["g"], case["u"], case["d"], hidden,
                  case["F"])
    assert maxdiff(out.ravel(), case["y"]) < 1e-5


# ---- tests/test_quant.cpp:42-141 ---------------------------------------------

def rel_rms(ref, got):
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    sr = np.sum(ref * ref)
    return float(np.sqrt(np.sum((ref - got) ** 2) / sr)) if sr > 0 else 0.0


def test_quant_exact_cases():
    q, s = oracle.quantize_rows(np.array([[127.0, -127.0, 0.0]], np.float32))
    assert np.array_equal(oracle.dequantize(q, s), [[127.0, -127.0, 0.0]])
    q, s = oracle.quantize_rows(np.zeros((1, 4), np.float32))
    assert np.all(oracle.dequantize(q, s) == 0.0) and s[0] == 1.0
    big = np.array([[1e6, -1e6, 0, 5, -5], [1, 2, 3, 4, 5]], np.float32)
    q, _ = oracle.quantize_rows(big)
    assert q.min() >= -127 and q.max() <= 127


@pytest.mark.parametrize("cols", [1024, 3072])
def test_quant_roundtrip_error(cols):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((256, cols)) * 0.02).astype(np.float32)
    q, s = oracle.quantize_rows(w)
    assert rel_rms(w, oracle.dequantize(q, s)) < 0.02


@pytest.mark.parametrize("mnk", [(1, 1024, 1024), (1, 3072, 1024), (8, 1024, 1024)])
def test_q8_matmul_error(mnk):
    M, N, K = mnk
    rng = np.random.default_rng(12)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, s = oracle.quantize_rows(B)
    assert rel_rms(oracle.matmul_nt(A, B), oracle.matmul_nt_q8(A, q, s)) < 0.02


def test_quant_per_row_beats_global():
    rng = np.random.default_rng(13)
    w = np.stack([rng.standard_normal(1024) * (0.02 if r % 2 == 0 else 0.0004)
                  for r in range(64)]).astype(np.float32)
    q, s = oracle.quantize_rows(w)
    per_row = rel_rms(w, oracle.dequantize(q, s))
    g = np.float32(np.abs(w).max() / np.float32(127.0))
    glob = np.clip(np.rint(w / g), -127, 127) * g
    assert per_row < rel_rms(w, glob)


def test_quant_memory_ratio():
    # 1000x1000: int8 data + one f32 scale per row vs f32
    assert (1000 * 1000 * 4) / (1000 * 1000 + 1000 * 4) > 3.9


def test_greedy_is_argmax():
    assert oracle.argmax(np.array([1.0, 5.0, 2.0, 3.0], np.float32)) == 1
    # ties: the strict '>' scan keeps the lowest index
    assert oracle.argmax(np.array([0.5, 2.0, 2.0, 1.0], np.float32)) == 1
