"""Seeded synthetic Qwen3 models: the weights every benchmark and test uses.

Linear weights and the tied embedding are N(0, 0.02) f32, RMSNorm weights are
1.0, and there is no lm_head.weight (tie_word_embeddings = true).  Each tensor
gets its own stream of the counter-based generator vb_synth_normal, seeded by
(seed, tensor index), so a model is identical wherever it is generated.

write_model_dir() stores a model as config.json + one F32 safetensors file,
the format the reference's Model(dir) reads through its F32 path
(core/src/safetensors.cpp:245-247, core/src/config.cpp:34-63).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

import vb200

QWEN3_0_6B = {
    "architectures": ["Qwen3ForCausalLM"],
    "hidden_size": 1024,
    "num_hidden_layers": 28,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "intermediate_size": 3072,
    "vocab_size": 151936,
    "max_position_embeddings": 40960,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "tie_word_embeddings": True,
}


def qwen3_config(**over) -> dict:
    c = dict(QWEN3_0_6B)
    c.update(over)
    return c


def tensor_specs(cfg: dict):
    """(name, shape, kind) in a fixed order; kind 'linear' or 'norm'."""
    H, KVH = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd, D, F, V = cfg["hidden_size"], cfg["head_dim"], cfg["intermediate_size"], cfg["vocab_size"]
    specs = [("model.embed_tokens.weight", (V, hd), "linear"), ("model.norm.weight", (hd,), "norm")]
    for i in range(cfg["num_hidden_layers"]):
        n = vb200.layer_names(i)
        specs += [
            (n["input_norm"], (hd,), "norm"),
            (n["post_norm"], (hd,), "norm"),
            (n["wq"], (H * D, hd), "linear"),
            (n["wk"], (KVH * D, hd), "linear"),
            (n["wv"], (KVH * D, hd), "linear"),
            (n["wo"], (hd, H * D), "linear"),
            (n["q_norm"], (D,), "norm"),
            (n["k_norm"], (D,), "norm"),
            (n["wg"], (F, hd), "linear"),
            (n["wu"], (F, hd), "linear"),
            (n["wd"], (hd, F), "linear"),
        ]
    return specs


def make_weights(cfg: dict, seed: int = 1234, std: float = 0.02, norm_value: float = 1.0,
                 normal=None) -> dict:
    """normal(n, seed, std) -> f32 array: the generator (default the engine
    library's vb_synth_normal; the oracle's or_synth_normal gives the same
    values for callers that must not load the engine library)."""
    normal = normal or vb200.synth_normal
    out = {}
    for idx, (name, shape, kind) in enumerate(tensor_specs(cfg)):
        n = int(np.prod(shape))
        if kind == "linear":
            a = normal(n, seed * 1000003 + idx, std)
        else:
            a = np.full(n, norm_value, dtype=np.float32)
        out[name] = a.reshape(shape)
    return out


def write_safetensors(path: Path, tensors: dict):
    header = {}
    off = 0
    for name, a in tensors.items():
        nb = a.size * 4
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + nb]}
        off += nb
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for a in tensors.values():
            f.write(memoryview(np.ascontiguousarray(a, dtype=np.float32)).cast("B"))


def write_model_dir(path, cfg: dict, weights: dict):
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(cfg, indent=1))
    write_safetensors(path / "model.safetensors", weights)
    return path


def prompt_ids(n: int, seed: int, vocab: int) -> np.ndarray:
    """Uniform random token ids in [0, vocab) from a fixed seed."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
