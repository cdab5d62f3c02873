"""Prefill of whole prompt chunks (tensor-core GEMMs over all rows + causal
flash attention) against the oracle.

The reference prefills one position at a time through Model::step
(generate.cpp:75-77); the chunked prefill computes the same layers
(model.cpp:240-254, generate.cpp:42-107) for all positions of a chunk at once,
so only the summation order differs.  Checked: the causal attention kernels
(tensor cores for a prompt from position 0, CUDA cores otherwise) against the
oracle's decode attention at every query position, and a batch
prefilled in several chunks against per-sequence oracle decoding (greedy pick
after the prompt, and the logits of the next step within the logits bars).
"""
import numpy as np
import pytest

import oracle
import vb200
import vbsynth
from conftest import mini_config

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = {"f32": 1e-3, "int8": 1e-2}


@pytest.mark.parametrize("B,C,p0", [(3, 40, 9), (2, 1, 0), (1, 64, 0), (2, 33, 100), (2, 200, 0), (1, 130, 0)])
def test_attn_prefill_matches_decode_attention(B, C, p0):
    H, KVH, D = 16, 8, 128
    n = p0 + C
    g = torch.Generator(device="cuda").manual_seed(7 * B + C + p0)
    q = torch.randn(B * C, H * D, device="cuda", generator=g)
    k = torch.randn(B, KVH, n + 3, D, device="cuda", generator=g)
    v = torch.randn(B, KVH, n + 3, D, device="cuda", generator=g)
    out = torch.full((B * C, H * D), float("nan"), device="cuda")
    vb200.attn_prefill(q, k, v, out, B, C, p0, H, KVH, D, KVH * (n + 3) * D, (n + 3) * D)
    torch.cuda.synchronize()
    got, qh = out.cpu().numpy(), q.cpu().numpy()
    kh = k.cpu().numpy().transpose(0, 2, 1, 3).reshape(B, n + 3, KVH * D)
    vh = v.cpu().numpy().transpose(0, 2, 1, 3).reshape(B, n + 3, KVH * D)
    for b in range(B):
        for c in sorted({0, C // 2, C - 1}):
            ref = oracle.attention_decode(qh[b * C + c], kh[b], vh[b], H, KVH, D, p0 + c + 1).ravel()
            assert np.max(np.abs(got[b * C + c] - ref)) < 5e-5, (b, c)


def test_attn_prefill_rejects_bad_shapes():
    t = torch.zeros(64, device="cuda")
    with pytest.raises(vb200.VBError):
        vb200.attn_prefill(t, t, t, t, 1, 1, 0, 16, 4, 128, 128, 128)  # H != 2 * KVH
    with pytest.raises(vb200.VBError):
        vb200.attn_prefill(t, t, t, t, 1, 1, 0, 16, 8, 64, 64, 64)     # D != 128


@pytest.mark.parametrize("mode", ["f32", "int8"])
@pytest.mark.parametrize("rows", ["64", None])
def test_chunked_prefill_matches_oracle(mode, rows, monkeypatch):
    """rows 64: 12 positions per chunk (chunks 12, 12, 6; attention on the CUDA
    cores after the first chunk); default: one chunk, tensor-core attention."""
    cfg = mini_config()
    w = vbsynth.make_weights(cfg, seed=61)
    B, P = 5, 30
    if rows:
        monkeypatch.setenv("VB_PREFILL_ROWS", rows)
    else:
        monkeypatch.delenv("VB_PREFILL_ROWS", raising=False)
    prompts = np.stack([vbsynth.prompt_ids(P, 300 + b, cfg["vocab_size"]) for b in range(B)])
    eng = vb200.Engine(cfg).load(w)
    if mode == "int8":
        eng.quantize()
    bt = vb200.Batch(eng, B, P + 8)
    nx = bt.prefill(prompts.T.copy())
    assert bt.cache_len() == P
    lg, nx2 = bt.step(nx)
    for b in range(B):
        o = oracle.OracleModel(cfg, w)
        if mode == "int8":
            o.quantize()
        o.reset_cache(P + 8)
        for t in range(P):
            lo = o.step(int(prompts[b, t]))
        assert oracle.argmax(lo) == int(nx[b]), b
        lo = o.step(int(nx[b]))
        assert np.max(np.abs(lo - lg[b])) <= TOL[mode], b
        assert oracle.argmax(lo) == int(nx2[b]), b
        o.close()
    bt.close()
    eng.close()
