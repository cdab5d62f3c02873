"""ctypes binding of libverbum_b200.so (the C ABI in include/verbum_b200.h).

This is the Python face of the drop-in boundary: `Engine` mirrors verbum::Model
(core/include/verbum/model.h:47-116) -- reset_cache / step / quantize /
weight_bytes -- and `Batch` is the batched independent-sequence extension.
The kernel helpers (matmul_nt_f32, attn_decode, ...) take torch CUDA tensors
and the current stream; torch is used only for device memory and streams.

Every call fails loudly: a missing library raises at import of `lib()`, and a
non-zero vb_status raises VBError with the library's message.  There is no
CPU fallback anywhere in this module.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
# VB200_LIB selects another build of the library (e.g. a VB_STEP_TRACE=1
# profiling build); the default is the in-tree one
LIB_PATH = Path(os.environ["VB200_LIB"]) if os.environ.get("VB200_LIB") else PKG / "lib" / "libverbum_b200.so"

VB_OK = 0
ERR_NAMES = {
    -1: "VB_ERR_ARG", -2: "VB_ERR_CUDA", -3: "VB_ERR_NO_CACHE", -4: "VB_ERR_CACHE_FULL",
    -5: "VB_ERR_ROPE", -6: "VB_ERR_TOKEN", -7: "VB_ERR_STATE", -8: "VB_ERR_TIMEOUT",
    -9: "VB_ERR_UNSUPPORTED",
}


class VBError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERR_NAMES.get(code, code)}: {msg}")
        self.code = code
        self.msg = msg


class VBConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn", C.c_int),
                ("vocab", C.c_int), ("rope_positions", C.c_int), ("eps", C.c_float),
                ("theta", C.c_float)]


class VBLayerHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "input_norm", "post_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "wg", "wu", "wd")]


class VBLayerHostQ8(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "input_norm", "post_norm", "q_norm", "k_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd",
        "sq", "sk", "sv", "so", "sg", "su", "sd")]


_LIB = None

# name -> (restype, argtypes)
_P, _I, _Z, _F, _L = C.c_void_p, C.c_int, C.c_size_t, C.c_float, C.c_int64
_SIGS = {
    "vb_last_error": (C.c_char_p, []),
    "vb_version": (C.c_char_p, []),
    "vb_debug_arm_fault": (_I, [_I]),
    "vb_device_count": (_I, []),
    "vb_device_name": (_I, [_I, C.c_char_p, _Z]),
    "vb_free_memory": (_I, [_I, C.POINTER(C.c_size_t)]),
    "vb_alloc": (_I, [C.POINTER(C.c_void_p), _Z]),
    "vb_free": (_I, [_P]),
    "vb_upload": (_I, [_P, _P, _Z, _P]),
    "vb_download": (_I, [_P, _P, _Z, _P]),
    "vb_zero": (_I, [_P, _Z, _P]),
    "vb_sync": (_I, [_P]),
    "vb_matmul_nt_f32": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "vb_matmul_nt_q8": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "vb_matmul_nt_tc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "vb_quantize_rows": (_I, [_P, _L, _L, _P, _P, _P]),
    "vb_rmsnorm": (_I, [_P, _P, _P, _I, _I, _F, _P]),
    "vb_rope": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "vb_silu_mul": (_I, [_P, _P, _I, _P]),
    "vb_add": (_I, [_P, _P, _I, _P]),
    "vb_cache_append": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "vb_attn_decode": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "vb_attn_decode_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "vb_attn_workspace_bytes": (_Z, [_I, _I, _I]),
    "vb_attn_prefill": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _P]),
    "vb_attn_decode_batched": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _L, _L, _L, _P, _P]),
    "vb_argmax_rows": (_I, [_P, _I, _L, _P, _P]),
    "vb_synth_normal": (None, [_P, C.c_uint64, C.c_uint64, _F]),
    "vb_engine_create": (_I, [C.POINTER(VBConfig), _I, C.POINTER(C.c_void_p)]),
    "vb_engine_destroy": (_I, [_P]),
    "vb_engine_set_globals": (_I, [_P, _P, _P]),
    "vb_engine_set_layer": (_I, [_P, _I, C.POINTER(VBLayerHost)]),
    "vb_engine_set_layer_q8": (_I, [_P, _I, C.POINTER(VBLayerHostQ8)]),
    "vb_engine_quantize": (_I, [_P]),
    "vb_engine_is_quantized": (_I, [_P]),
    "vb_engine_weight_bytes": (_Z, [_P]),
    "vb_engine_reset_cache": (_I, [_P, _I]),
    "vb_engine_cache_len": (_I, [_P]),
    "vb_engine_step": (_I, [_P, _I, _P]),
    "vb_engine_decode": (_I, [_P, _I, _I, _P, _P]),
    "vb_engine_read_kv": (_I, [_P, _I, _I, _P]),
    "vb_engine_prefill": (_I, [_P, _P, _I, _P]),
    "vb_engine_graph_nodes": (_I, [_P]),
    "vb_engine_set_path": (_I, [_P, _I]),
    "vb_engine_path": (_I, [_P]),
    "vb_engine_stream": (_P, [_P]),
    "vb_engine_set_trace": (_I, [_P, _I]),
    "vb_engine_read_trace": (_I, [_P, _P, _I]),
    "vb_batch_create": (_I, [_P, _I, _I, C.POINTER(C.c_void_p)]),
    "vb_batch_destroy": (_I, [_P]),
    "vb_batch_step": (_I, [_P, _P, _P, _P]),
    "vb_batch_decode": (_I, [_P, _P, _I, _P]),
    "vb_batch_cache_len": (_I, [_P]),
    "vb_batch_prefill": (_I, [_P, _P, _I, _P]),
    "vb_batch_graph_nodes": (_I, [_P]),
    "vb_batch_reset": (_I, [_P]),
    "vb_sampler_create": (_I, [_F, _I, _F, C.c_uint64, _P]),
    "vb_engine_quantize_lm_head": (_I, [_P]),
    "vb_engine_set_globals_bf16": (_I, [_P, _P, _P]),
    "vb_engine_embed_text": (_I, [_P, _P, _I, _P]),
    "vb_engine_set_layer_bf16": (_I, [_P, _I, _P]),
    "vb_engine_lm_head_int8": (_I, [_P]),
    "vb_sampler_destroy": (_I, [_P]),
    "vb_sampler_sample": (_I, [_P, _P, _L, _P, _P]),
    "vb_engine_decode_sampled": (_I, [_P, _P, _I, _I, _P]),
    "vb_batch_truncate": (_I, [_P, _I]),
}


def lib():
    """Loads the in-tree library (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run python verbum.cpp_b200/build.py")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def exported_symbols():
    return list(_SIGS)


def check(code):
    if code != VB_OK:
        raise VBError(code, lib().vb_last_error().decode())
    return code


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def synth_normal(n: int, seed: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(int(n), dtype=np.float32)
    lib().vb_synth_normal(_ptr(out), int(n), int(seed) & (2**64 - 1), float(std))
    return out


def debug_arm_fault(site: int):
    """Arms the failure-path test hook for one launch (1 = clustered step,
    2 = tensor-core GEMM; 0 disarms)."""
    check(lib().vb_debug_arm_fault(int(site)))


def device_count() -> int:
    return lib().vb_device_count()


def make_config(cfg: dict) -> VBConfig:
    """HF config.json keys -> vb_config (ModelConfig::from_file, config.cpp:34-63)."""
    heads = cfg["num_attention_heads"]
    return VBConfig(
        hidden=cfg["hidden_size"], layers=cfg["num_hidden_layers"], heads=heads,
        kv_heads=cfg.get("num_key_value_heads", heads),
        head_dim=cfg.get("head_dim", cfg["hidden_size"] // heads),
        ffn=cfg["intermediate_size"], vocab=cfg["vocab_size"],
        rope_positions=min(cfg.get("max_position_embeddings", 32768), 4096),
        eps=cfg.get("rms_norm_eps", 1e-6), theta=cfg.get("rope_theta", 10000.0))


def layer_names(i: int) -> dict:
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


class Engine:
    """Device-resident decode engine; the verbum::Model surface."""

    def __init__(self, cfg: dict, device: int = 0):
        self.cfg = dict(cfg)
        self.vcfg = make_config(cfg)
        h = C.c_void_p()
        check(lib().vb_engine_create(C.byref(self.vcfg), int(device), C.byref(h)))
        self.h = h
        self.vocab = self.vcfg.vocab

    # -- weights -------------------------------------------------------------
    def load(self, weights: dict):
        """Uploads a {HF tensor name: float32 array} dict (tied embeddings)."""
        emb = np.ascontiguousarray(weights["model.embed_tokens.weight"], dtype=np.float32)
        fn = np.ascontiguousarray(weights["model.norm.weight"], dtype=np.float32)
        check(lib().vb_engine_set_globals(self.h, _ptr(emb), _ptr(fn)))
        for i in range(self.vcfg.layers):
            names = layer_names(i)
            arrs = {k: np.ascontiguousarray(weights[v], dtype=np.float32) for k, v in names.items()}
            lh = VBLayerHost(**{k: a.ctypes.data for k, a in arrs.items()})
            check(lib().vb_engine_set_layer(self.h, i, C.byref(lh)))
        return self

    def load_quantized(self, weights: dict, qlayers):
        """Uploads the f32 globals and norms from `weights` and, per layer,
        already-quantized projections: qlayers[i] = {name: (int8 [rows][cols],
        f32 scales [rows])} for name in wq wk wv wo wg wu wd (the reference's
        QuantLayer).  The engine then holds exactly these INT8 weights."""
        emb = np.ascontiguousarray(weights["model.embed_tokens.weight"], dtype=np.float32)
        fn = np.ascontiguousarray(weights["model.norm.weight"], dtype=np.float32)
        check(lib().vb_engine_set_globals(self.h, _ptr(emb), _ptr(fn)))
        keep = []
        for i in range(self.vcfg.layers):
            names = layer_names(i)
            f = {k: np.ascontiguousarray(weights[names[k]], dtype=np.float32)
                 for k in ("input_norm", "post_norm", "q_norm", "k_norm")}
            args = {k: a.ctypes.data for k, a in f.items()}
            for k, sk in (("wq", "sq"), ("wk", "sk"), ("wv", "sv"), ("wo", "so"), ("wg", "sg"),
                          ("wu", "su"), ("wd", "sd")):
                q, sc = qlayers[i][k]
                q = np.ascontiguousarray(q, dtype=np.int8)
                sc = np.ascontiguousarray(sc, dtype=np.float32)
                keep += [q, sc]
                args[k], args[sk] = q.ctypes.data, sc.ctypes.data
            keep += list(f.values())
            check(lib().vb_engine_set_layer_q8(self.h, i, C.byref(VBLayerHostQ8(**args))))
        return self

    def load_bf16(self, weights: dict):
        """Uploads a {HF tensor name: uint16 bf16-bit-pattern array} dict, widened on the device."""
        emb = np.ascontiguousarray(weights["model.embed_tokens.weight"], dtype=np.uint16)
        fn = np.ascontiguousarray(weights["model.norm.weight"], dtype=np.uint16)
        check(lib().vb_engine_set_globals_bf16(self.h, _ptr(emb), _ptr(fn)))
        for i in range(self.vcfg.layers):
            names = layer_names(i)
            arrs = {k: np.ascontiguousarray(weights[v], dtype=np.uint16) for k, v in names.items()}
            lh = VBLayerHost(**{k: a.ctypes.data for k, a in arrs.items()})  # same field order
            check(lib().vb_engine_set_layer_bf16(self.h, i, C.byref(lh)))
        return self

    def quantize(self):
        check(lib().vb_engine_quantize(self.h))

    def is_quantized(self) -> bool:
        return bool(lib().vb_engine_is_quantized(self.h))

    def weight_bytes(self) -> int:
        return int(lib().vb_engine_weight_bytes(self.h))

    # -- decode --------------------------------------------------------------
    def reset_cache(self, max_seq: int):
        check(lib().vb_engine_reset_cache(self.h, int(max_seq)))

    def cache_len(self) -> int:
        return lib().vb_engine_cache_len(self.h)

    def step(self, token: int, out: np.ndarray | None = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.vocab, dtype=np.float32)
        check(lib().vb_engine_step(self.h, int(token), _ptr(out)))
        return out

    def embed_text(self, ids) -> np.ndarray:
        """Model::embed_text: mean-pooled, L2-normalised final hidden states."""
        t = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.vcfg.hidden, dtype=np.float32)
        check(lib().vb_engine_embed_text(self.h, _ptr(t), int(t.size), _ptr(out)))
        return out

    def quantize_lm_head(self):
        """Opt-in INT8 tied lm_head (not reference-identical; see the C header)."""
        check(lib().vb_engine_quantize_lm_head(self.h))
        return self

    def decode_sampled(self, sampler: "Sampler", first_token: int, n: int) -> np.ndarray:
        """n decode steps, each next token drawn by `sampler` on the device."""
        toks = np.empty(int(n), dtype=np.int32)
        check(lib().vb_engine_decode_sampled(self.h, sampler.h, int(first_token), int(n), _ptr(toks)))
        return toks

    def decode(self, first_token: int, n: int, want_logits=False):
        toks = np.empty(int(n), dtype=np.int32)
        lg = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        check(lib().vb_engine_decode(self.h, int(first_token), int(n), _ptr(toks),
                                     _ptr(lg) if lg is not None else None))
        return (toks, lg) if want_logits else toks

    def prefill(self, tokens, want_logits=False):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        check(lib().vb_engine_prefill(self.h, _ptr(t), int(t.size),
                                      _ptr(lg) if lg is not None else None))
        return lg

    def graph_nodes(self) -> int:
        return lib().vb_engine_graph_nodes(self.h)

    def read_kv(self, layer: int, which: int) -> np.ndarray:
        n = self.cache_len()
        out = np.empty((n, self.vcfg.kv_heads * self.vcfg.head_dim), dtype=np.float32)
        check(lib().vb_engine_read_kv(self.h, int(layer), int(which), _ptr(out)))
        return out

    def set_path(self, path: int):
        """1 = per-op CUDA graph, 2 = clustered persistent step, -1 = automatic."""
        check(lib().vb_engine_set_path(self.h, int(path)))
        return self

    def path(self) -> int:
        """The step path the next step runs (the automatic choice if not fixed)."""
        return lib().vb_engine_path(self.h)

    def set_trace(self, on: bool):
        check(lib().vb_engine_set_trace(self.h, int(bool(on))))

    def read_trace(self) -> np.ndarray:
        out = np.zeros(148 * 1024 * 2, dtype=np.uint64)
        n = lib().vb_engine_read_trace(self.h, _ptr(out), out.size)
        return out[:n]

    def stream(self) -> int:
        return lib().vb_engine_stream(self.h) or 0

    def close(self):
        if getattr(self, "h", None):
            # a batch refers to its engine: close the engine's live batches
            # first (finalizers of a collected cycle run in any order)
            for b in list(getattr(self, "_batches", ())):
                b.close()
            lib().vb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """B independent sequences sharing one engine's weights."""

    def __init__(self, engine: Engine, batch: int, max_seq: int):
        self.engine = engine
        self.B = int(batch)
        h = C.c_void_p()
        check(lib().vb_batch_create(engine.h, self.B, int(max_seq), C.byref(h)))
        self.h = h
        if not hasattr(engine, "_batches"):
            engine._batches = weakref.WeakSet()
        engine._batches.add(self)

    def step(self, tokens, want_logits=True, want_next=True):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        assert t.shape == (self.B,)
        lg = np.empty((self.B, self.engine.vocab), dtype=np.float32) if want_logits else None
        nx = np.empty(self.B, dtype=np.int32) if want_next else None
        check(lib().vb_batch_step(self.h, _ptr(t), _ptr(lg) if lg is not None else None,
                                  _ptr(nx) if nx is not None else None))
        return lg, nx

    def decode(self, tokens, n: int):
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        nx = np.empty(self.B, dtype=np.int32)
        check(lib().vb_batch_decode(self.h, _ptr(t) if t is not None else None, int(n), _ptr(nx)))
        return nx

    def prefill(self, tokens_pb):
        """tokens_pb: [P, B] position-major prompt ids; returns next ids [B]."""
        t = np.ascontiguousarray(tokens_pb, dtype=np.int32)
        assert t.ndim == 2 and t.shape[1] == self.B
        nx = np.empty(self.B, dtype=np.int32)
        check(lib().vb_batch_prefill(self.h, _ptr(t), int(t.shape[0]), _ptr(nx)))
        return nx

    def graph_nodes(self) -> int:
        return lib().vb_batch_graph_nodes(self.h)

    def cache_len(self) -> int:
        return lib().vb_batch_cache_len(self.h)

    def reset(self):
        check(lib().vb_batch_reset(self.h))

    def truncate(self, length: int):
        check(lib().vb_batch_truncate(self.h, int(length)))

    def close(self):
        if getattr(self, "h", None):
            lib().vb_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# -- kernel entry points on torch CUDA tensors (tests / microbenchmarks) -----

def _tp(t):
    return C.c_void_p(t.data_ptr())


def _stream(stream=None):
    if stream is not None:
        return C.c_void_p(int(stream))
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def matmul_nt_f32(A, W, C_out, stream=None):
    M, K = A.shape
    N = W.shape[0]
    check(lib().vb_matmul_nt_f32(_tp(A), _tp(W), _tp(C_out), M, N, K, _stream(stream)))


def matmul_nt_q8(A, Wq, scales, C_out, stream=None):
    M, K = A.shape
    N = Wq.shape[0]
    check(lib().vb_matmul_nt_q8(_tp(A), _tp(Wq), _tp(scales), _tp(C_out), M, N, K, _stream(stream)))


def matmul_nt_tc(A, W, C_out, scales=None, stream=None):
    """C = A . W^T on the tensor cores; W f32, or int8 with per-row scales."""
    M, K = A.shape
    N = W.shape[0]
    q8 = scales is not None
    check(lib().vb_matmul_nt_tc(_tp(A), _tp(W), _tp(scales) if q8 else None, _tp(C_out), M, N, K, int(q8),
                                _stream(stream)))


def quantize_rows(W, q, scales, stream=None):
    rows, cols = W.shape
    check(lib().vb_quantize_rows(_tp(W), rows, cols, _tp(q), _tp(scales), _stream(stream)))


def rmsnorm(x, w, out, eps, stream=None):
    rows, dim = x.shape
    check(lib().vb_rmsnorm(_tp(x), _tp(w), _tp(out), rows, dim, float(eps), _stream(stream)))


def rope(x, cos_tab, sin_tab, pos, stream=None):
    heads, D = x.shape
    check(lib().vb_rope(_tp(x), _tp(cos_tab), _tp(sin_tab), int(pos), heads, D, _stream(stream)))


def silu_mul(gate, up, stream=None):
    check(lib().vb_silu_mul(_tp(gate), _tp(up), gate.numel(), _stream(stream)))


def add(a, b, stream=None):
    check(lib().vb_add(_tp(a), _tp(b), a.numel(), _stream(stream)))


def cache_append(kc, vc, kn, vn, pos, stream=None):
    check(lib().vb_cache_append(_tp(kc), _tp(vc), _tp(kn), _tp(vn), int(pos), kn.numel(),
                                _stream(stream)))


def attn_decode(q, kc, vc, out, H, KVH, D, n, stream=None):
    check(lib().vb_attn_decode(_tp(q), _tp(kc), _tp(vc), _tp(out), H, KVH, D, int(n),
                               _stream(stream)))


def attn_decode_noalloc(q, kc, vc, out, H, KVH, D, n, stream=None):
    """vb_attn_decode without any device allocation (static scratch)."""
    check(lib().vb_attn_decode_noalloc(_tp(q), _tp(kc), _tp(vc), _tp(out), H, KVH, D, int(n),
                                       _stream(stream)))


def attn_workspace_bytes(B, H, n_max):
    return int(lib().vb_attn_workspace_bytes(B, H, n_max))


def attn_decode_batched(q, k, v, out, lens, B, H, KVH, D, n_max, stride_b, stride_pos,
                        stride_h, workspace, stream=None):
    check(lib().vb_attn_decode_batched(_tp(q), _tp(k), _tp(v), _tp(out), _tp(lens), B, H, KVH, D,
                                       n_max, stride_b, stride_pos, stride_h, _tp(workspace),
                                       _stream(stream)))


def attn_prefill(q, k, v, out, B, C, p0, H, KVH, D, stride_b, stride_h, stream=None):
    """Causal attention of a prompt chunk: q / out [B*C, H*D]; caches [B, KVH, n, D]."""
    check(lib().vb_attn_prefill(_tp(q), _tp(k), _tp(v), _tp(out), B, C, p0, H, KVH, D, stride_b,
                                stride_h, _stream(stream)))


class Sampler:
    """Sampler / SamplerConfig (generate.h:49-67): temperature, top_k (0
    disables), top_p (1 disables), seed of the host std::mt19937_64."""

    def __init__(self, temperature=0.8, top_k=40, top_p=0.95, seed=0):
        h = C.c_void_p()
        check(lib().vb_sampler_create(float(temperature), int(top_k), float(top_p), int(seed), C.byref(h)))
        self.h = h

    def sample(self, logits, stream=None) -> int:
        """One Sampler::sample of a device logits row."""
        tok = C.c_int()
        check(lib().vb_sampler_sample(self.h, _tp(logits), int(logits.numel()), _stream(stream), C.byref(tok)))
        return tok.value

    def close(self):
        if getattr(self, "h", None):
            lib().vb_sampler_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def argmax_rows(logits, out_idx, stream=None):
    rows, n = logits.shape
    check(lib().vb_argmax_rows(_tp(logits), rows, n, _tp(out_idx), _stream(stream)))
