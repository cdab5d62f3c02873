"""Python face of the CPU oracle (TEST INFRASTRUCTURE ONLY).

`Oracle*` wrap liboracle.so, the C restatement of the reference's CPU path
(vb_oracle.c).  `Ref*` wrap oracle/_ref/libverbum_ref.so, the unmodified
reference engine compiled from its own sources by oracle/Makefile.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, always as the checker of the CUDA engine, never in its place.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libverbum_ref.so"

_P, _I, _L, _F, _Z = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t


class OrConfig(C.Structure):
    _fields_ = [("hidden", _I), ("layers", _I), ("heads", _I), ("kv_heads", _I),
                ("head_dim", _I), ("ffn", _I), ("vocab", _I), ("rope_positions", _I),
                ("eps", _F), ("theta", _F)]


class OrLayer(C.Structure):
    _fields_ = [(n, _P) for n in ("input_norm", "post_norm", "wq", "wk", "wv", "wo", "q_norm",
                                  "k_norm", "wg", "wu", "wd")]


_OR = None
_REF = None


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def have_oracle() -> bool:
    return ORACLE_SO.exists()


def have_ref() -> bool:
    return REF_SO.exists()


def olib():
    global _OR
    if _OR is None:
        if not ORACLE_SO.exists():
            raise RuntimeError(f"{ORACLE_SO} missing: run make -C oracle")
        L = C.CDLL(str(ORACLE_SO))
        sig = {
            "or_rmsnorm": (None, [_P, _P, _F, _P, _L, _L]),
            "or_build_rope_table": (_I, [_I, _I, _F, _P, _P]),
            "or_apply_rope": (_I, [_P, _L, _I, _I, _I, _P, _P]),
            "or_matmul_nt": (None, [_P, _P, _P, _L, _L, _L]),
            "or_quantize_rows": (None, [_P, _L, _L, _P, _P]),
            "or_matmul_nt_q8": (None, [_P, _P, _P, _P, _L, _L, _L]),
            "or_dequantize": (None, [_P, _P, _L, _L, _P]),
            "or_attention_decode": (None, [_P, _P, _P, _L, _I, _I, _I, _I, _P]),
            "or_silu_mul": (None, [_P, _P, _L]),
            "or_argmax": (_I, [_P, _L]),
            "or_synth_normal": (None, [_P, C.c_uint64, C.c_uint64, _F]),
            "or_sample_seq": (_I, [_F, _I, _F, C.c_uint64, _P, _L, _I, _P]),
            "or_last_error": (C.c_char_p, []),
            "or_model_create": (_P, [C.POINTER(OrConfig), _P, _P, C.POINTER(OrLayer)]),
            "or_model_free": (None, [_P]),
            "or_model_quantize": (_I, [_P]),
            "or_model_quantize_lm_head": (_I, [_P]),
            "or_model_is_quantized": (_I, [_P]),
            "or_model_quant_tensor": (_I, [_P, _I, _I, C.POINTER(C.c_void_p),
                                           C.POINTER(C.c_void_p), C.POINTER(_L), C.POINTER(_L)]),
            "or_model_reset_cache": (_I, [_P, _I]),
            "or_model_step": (_I, [_P, _I, _P]),
            "or_model_prefill": (_I, [_P, _P, _I, _P]),
            "or_model_cache_len": (_I, [_P]),
            "or_model_weight_bytes": (_Z, [_P]),
            "or_model_kv": (_P, [_P, _I, _I]),
            "or_set_threads": (None, [_I]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _OR = L
    return _OR


def rlib():
    global _REF
    if _REF is None:
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} missing: run make -C oracle ref")
        L = C.CDLL(str(REF_SO))
        sig = {
            "ref_last_error": (C.c_char_p, []),
            "ref_model_open": (_P, [C.c_char_p]),
            "ref_model_free": (None, [_P]),
            "ref_model_quantize": (_I, [_P]),
            "ref_model_reset_cache": (_I, [_P, _I]),
            "ref_model_step": (_I, [_P, _I, _P]),
            "ref_model_greedy_steps": (_I, [_P, _I, _I, _P, _P]),
            "ref_model_set_cache_len": (_I, [_P, _I]),
            "ref_model_cache_len": (_I, [_P]),
            "ref_model_weight_bytes": (C.c_ulonglong, [_P]),
            "ref_model_is_quantized": (_I, [_P]),
            "ref_model_quant_tensor": (_I, [_P, _I, _I, _P, _P]),
            "ref_model_kv": (_I, [_P, _I, _I, _P]),
            "ref_quantize_rows": (_I, [_P, _L, _L, _P, _P]),
            "ref_matmul_nt": (_I, [_P, _P, _P, _L, _L, _L]),
            "ref_matmul_nt_q8": (_I, [_P, _P, _P, _P, _L, _L, _L]),
            "ref_rmsnorm": (_I, [_P, _P, _F, _P, _L, _L]),
            "ref_rope_table": (_I, [_I, _I, _F, _P, _P]),
            "ref_apply_rope": (_I, [_P, _L, _I, _I, _I, _F]),
            "ref_greedy": (_I, [_P, _L]),
            "ref_sample_seq": (_I, [_F, _I, _F, C.c_uint64, _P, _L, _I, _P]),
            "ref_model_embed_text": (_I, [_P, _P, _I, _P]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _REF = L
    return _REF


def set_threads(n: int):
    olib().or_set_threads(int(n))


# ---- primitive ops ----------------------------------------------------------

def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rmsnorm(x, w, eps):
    x = f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.empty_like(x2)
    olib().or_rmsnorm(_p(x2), _p(f32(w)), float(eps), _p(out), x2.shape[0], x2.shape[1])
    return out.reshape(x.shape)


def rope_table(head_dim, max_pos, theta):
    c = np.empty((max_pos, head_dim), np.float32)
    s = np.empty((max_pos, head_dim), np.float32)
    assert olib().or_build_rope_table(head_dim, max_pos, float(theta), _p(c), _p(s)) == 0
    return c, s


def apply_rope(x, pos, cos_tab, sin_tab):
    x = f32(x).copy()
    rc = olib().or_apply_rope(_p(x), x.shape[0], x.shape[1], int(pos), cos_tab.shape[0],
                              _p(cos_tab), _p(sin_tab))
    if rc:
        raise RuntimeError(olib().or_last_error().decode())
    return x


def matmul_nt(A, B):
    A, B = f32(A), f32(B)
    out = np.empty((A.shape[0], B.shape[0]), np.float32)
    olib().or_matmul_nt(_p(A), _p(B), _p(out), A.shape[0], B.shape[0], A.shape[1])
    return out


def quantize_rows(W):
    W = f32(W)
    q = np.empty(W.shape, np.int8)
    s = np.empty(W.shape[0], np.float32)
    olib().or_quantize_rows(_p(W), W.shape[0], W.shape[1], _p(q), _p(s))
    return q, s


def matmul_nt_q8(A, q, s):
    A = f32(A)
    q = np.ascontiguousarray(q, dtype=np.int8)
    out = np.empty((A.shape[0], q.shape[0]), np.float32)
    olib().or_matmul_nt_q8(_p(A), _p(q), _p(f32(s)), _p(out), A.shape[0], q.shape[0], A.shape[1])
    return out


def dequantize(q, s):
    out = np.empty(q.shape, np.float32)
    olib().or_dequantize(_p(np.ascontiguousarray(q)), _p(f32(s)), q.shape[0], q.shape[1], _p(out))
    return out


def attention_decode(q, kcache, vcache, H, KVH, D, n):
    """q [H, D]; caches [>=n, KVH*D] (the reference layout)."""
    q, kc, vc = f32(q), f32(kcache), f32(vcache)
    ctx = np.empty((H, D), np.float32)
    olib().or_attention_decode(_p(q), _p(kc), _p(vc), KVH * D, H, KVH, D, int(n), _p(ctx))
    return ctx


def silu_mul(g, u):
    g = f32(g).copy()
    olib().or_silu_mul(_p(g), _p(f32(u)), g.size)
    return g


def argmax(logits):
    logits = f32(logits)
    return int(olib().or_argmax(_p(logits), logits.size))


def synth_normal(n: int, seed: int, std: float = 0.02) -> np.ndarray:
    """The seeded N(0, std) weight generator (same values as the engine
    library's vb_synth_normal), so CPU-only callers need not load it."""
    out = np.empty(int(n), dtype=np.float32)
    olib().or_synth_normal(_p(out), int(n), int(seed) & (2**64 - 1), float(std))
    return out


def sample_seq(logits, temperature, top_k, top_p, seed):
    """generate.cpp:197-252: one Sampler over the rows of logits [n, vocab]."""
    logits = f32(logits)
    n, vocab = logits.shape
    out = np.empty(n, np.int32)
    if olib().or_sample_seq(float(temperature), int(top_k), float(top_p), int(seed), _p(logits), vocab, n,
                            _p(out)) != 0:
        raise MemoryError("or_sample_seq")
    return out


def ref_sample_seq(logits, temperature, top_k, top_p, seed):
    """The reference Sampler itself (oracle/_ref), for pinning sample_seq."""
    logits = f32(logits)
    n, vocab = logits.shape
    out = np.empty(n, np.int32)
    if rlib().ref_sample_seq(float(temperature), int(top_k), float(top_p), int(seed), _p(logits), vocab, n,
                             _p(out)) != 0:
        raise RuntimeError(rlib().ref_last_error().decode())
    return out


# ---- whole model --------------------------------------------------------------

def or_config(cfg: dict) -> OrConfig:
    heads = cfg["num_attention_heads"]
    return OrConfig(hidden=cfg["hidden_size"], layers=cfg["num_hidden_layers"], heads=heads,
                    kv_heads=cfg.get("num_key_value_heads", heads),
                    head_dim=cfg.get("head_dim", cfg["hidden_size"] // heads),
                    ffn=cfg["intermediate_size"], vocab=cfg["vocab_size"],
                    rope_positions=min(cfg.get("max_position_embeddings", 32768), 4096),
                    eps=cfg.get("rms_norm_eps", 1e-6), theta=cfg.get("rope_theta", 10000.0))


class OracleModel:
    """verbum::Model restated in C: step() returns the reference's logits."""

    NAMES = ("input_norm", "post_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "wg", "wu", "wd")

    def __init__(self, cfg: dict, weights: dict):
        from_names = _layer_names
        self.cfg = cfg
        self.c = or_config(cfg)
        self._keep = {k: f32(v) for k, v in weights.items()}
        layers = (OrLayer * self.c.layers)()
        for i in range(self.c.layers):
            nm = from_names(i)
            for f in self.NAMES:
                setattr(layers[i], f, self._keep[nm[f]].ctypes.data)
        self.h = olib().or_model_create(C.byref(self.c), _p(self._keep["model.embed_tokens.weight"]),
                                        _p(self._keep["model.norm.weight"]), layers)
        if not self.h:
            raise RuntimeError("or_model_create failed")

    def quantize(self):
        assert olib().or_model_quantize(self.h) == 0

    def quantize_lm_head(self):
        """Opt-in INT8 tied lm_head (no reference counterpart)."""
        assert olib().or_model_quantize_lm_head(self.h) == 0

    def quant_tensor(self, layer, which):
        q, s = C.c_void_p(), C.c_void_p()
        r, c = C.c_int64(), C.c_int64()
        assert olib().or_model_quant_tensor(self.h, layer, which, C.byref(q), C.byref(s),
                                            C.byref(r), C.byref(c)) == 0
        qa = np.ctypeslib.as_array(C.cast(q, C.POINTER(C.c_int8)), shape=(r.value, c.value)).copy()
        sa = np.ctypeslib.as_array(C.cast(s, C.POINTER(C.c_float)), shape=(r.value,)).copy()
        return qa, sa

    def reset_cache(self, max_seq):
        assert olib().or_model_reset_cache(self.h, int(max_seq)) == 0
        self.max_seq = int(max_seq)

    def step(self, token):
        out = np.empty(self.c.vocab, np.float32)
        rc = olib().or_model_step(self.h, int(token), _p(out))
        if rc:
            raise RuntimeError(olib().or_last_error().decode())
        return out

    def prefill(self, tokens):
        """Feeds the tokens from the current position (layer by layer over
        all of them; bit-identical to one step() per token) and returns the
        last position's logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.c.vocab, np.float32)
        rc = olib().or_model_prefill(self.h, _p(t), int(t.size), _p(out))
        if rc:
            raise RuntimeError(olib().or_last_error().decode())
        return out

    def cache_len(self):
        return olib().or_model_cache_len(self.h)

    def weight_bytes(self):
        return int(olib().or_model_weight_bytes(self.h))

    def kv(self, layer, which):
        p = olib().or_model_kv(self.h, layer, which)
        w = self.c.kv_heads * self.c.head_dim
        a = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(self.max_seq, w))
        return a[: self.cache_len()].copy()

    def close(self):
        if self.h:
            olib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _layer_names(i):
    p = f"model.layers.{i}."
    return {
        "input_norm": p + "input_layernorm.weight",
        "post_norm": p + "post_attention_layernorm.weight",
        "wq": p + "self_attn.q_proj.weight", "wk": p + "self_attn.k_proj.weight",
        "wv": p + "self_attn.v_proj.weight", "wo": p + "self_attn.o_proj.weight",
        "q_norm": p + "self_attn.q_norm.weight", "k_norm": p + "self_attn.k_norm.weight",
        "wg": p + "mlp.gate_proj.weight", "wu": p + "mlp.up_proj.weight",
        "wd": p + "mlp.down_proj.weight",
    }


class RefModel:
    """The reference's own verbum::Model, loaded from a model directory."""

    def __init__(self, model_dir):
        self.h = rlib().ref_model_open(str(model_dir).encode())
        if not self.h:
            raise RuntimeError(rlib().ref_last_error().decode())
        import json
        self.cfg = json.loads((Path(model_dir) / "config.json").read_text())
        self.vocab = self.cfg["vocab_size"]

    def _chk(self, rc):
        if rc:
            raise RuntimeError(rlib().ref_last_error().decode())

    def quantize(self):
        self._chk(rlib().ref_model_quantize(self.h))

    def reset_cache(self, n):
        self._chk(rlib().ref_model_reset_cache(self.h, int(n)))

    def set_cache_len(self, n):
        self._chk(rlib().ref_model_set_cache_len(self.h, int(n)))

    def step(self, token):
        out = np.empty(self.vocab, np.float32)
        self._chk(rlib().ref_model_step(self.h, int(token), _p(out)))
        return out

    def embed_text(self, ids, hidden):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(hidden, np.float32)
        self._chk(rlib().ref_model_embed_text(self.h, _p(ids), int(ids.size), _p(out)))
        return out

    def greedy_steps(self, first_token, n):
        toks = np.empty(n, np.int32)
        secs = np.empty(n, np.float64)
        self._chk(rlib().ref_model_greedy_steps(self.h, int(first_token), int(n), _p(toks), _p(secs)))
        return toks, secs

    def weight_bytes(self):
        return int(rlib().ref_model_weight_bytes(self.h))

    def quant_tensor(self, layer, which, rows, cols):
        q = np.empty((rows, cols), np.int8)
        s = np.empty(rows, np.float32)
        self._chk(rlib().ref_model_quant_tensor(self.h, layer, which, _p(q), _p(s)))
        return q, s

    def kv(self, layer, which, max_seq):
        w = self.cfg["num_key_value_heads"] * self.cfg["head_dim"]
        out = np.empty((max_seq, w), np.float32)
        self._chk(rlib().ref_model_kv(self.h, layer, which, _p(out)))
        return out

    def close(self):
        if self.h:
            rlib().ref_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_quantize_rows(W):
    W = f32(W)
    q = np.empty(W.shape, np.int8)
    s = np.empty(W.shape[0], np.float32)
    assert rlib().ref_quantize_rows(_p(W), W.shape[0], W.shape[1], _p(q), _p(s)) == 0
    return q, s


def ref_matmul_nt(A, B):
    A, B = f32(A), f32(B)
    out = np.empty((A.shape[0], B.shape[0]), np.float32)
    assert rlib().ref_matmul_nt(_p(A), _p(B), _p(out), A.shape[0], B.shape[0], A.shape[1]) == 0
    return out


def ref_matmul_nt_q8(A, q, s):
    A = f32(A)
    out = np.empty((A.shape[0], q.shape[0]), np.float32)
    assert rlib().ref_matmul_nt_q8(_p(A), _p(np.ascontiguousarray(q)), _p(f32(s)), _p(out),
                                   A.shape[0], q.shape[0], A.shape[1]) == 0
    return out


def ref_rmsnorm(x, w, eps):
    x = f32(x)
    out = np.empty_like(x)
    assert rlib().ref_rmsnorm(_p(x), _p(f32(w)), float(eps), _p(out), x.shape[0], x.shape[1]) == 0
    return out


def ref_rope_table(head_dim, max_pos, theta):
    c = np.empty((max_pos, head_dim), np.float32)
    s = np.empty((max_pos, head_dim), np.float32)
    assert rlib().ref_rope_table(head_dim, max_pos, float(theta), _p(c), _p(s)) == 0
    return c, s


def ref_greedy(logits):
    logits = f32(logits)
    return int(rlib().ref_greedy(_p(logits), logits.size))
