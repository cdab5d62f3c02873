"""The C++20 host: the reference's own verbum::Model over libverbum_b200.so.

verbum.cpp_b200/dropin builds two libraries from the reference's sources
(read in place by its Makefile, never copied):
  seam   -- the unmodified core/src/*.cpp with VERBUM_CUDA, linked against
            this library's implementation of the reference's launcher API
            (cuda_backend.h:7-43): Model::to_cuda / step_cuda (model.cpp:
            367-497) run the reference's own per-op step on the B200 kernels;
  engine -- model.h / model.cpp patched (VERBUM_B200) so to_cuda uploads the
            weights -- f32, or the reference's own quantized layers -- to the
            engine and step runs the engine's step.
Both carry dropin/model_shim.cpp, an extern "C" face for these tests.

CPU tests: both libraries load (their undefined symbols resolve against
libverbum_b200.so) and to_cuda() without a device throws the reference's
"no CUDA device found".  GPU tests: Model(dir) -> [quantize()] -> reset_cache
-> to_cuda -> step x N -> Sampler, against the oracle at the parity bars
(f32 logits <= 1e-3, INT8 <= 1e-2, greedy tokens identical), and the
reference's own Sampler picking from both.
"""
import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import oracle
import vb200
import vbsynth

ROOT = Path(__file__).resolve().parents[1]
DROPIN = ROOT / "verbum.cpp_b200" / "dropin" / "_build"
LIBS = {"seam": DROPIN / "libverbum_model_seam.so", "engine": DROPIN / "libverbum_model_engine.so"}
TOL = {"f32": 1e-3, "int8": 1e-2}


class Model:
    """ctypes wrapper of dropin/model_shim.cpp (verbum::Model)."""

    _libs = {}

    @classmethod
    def lib(cls, kind):
        if kind not in cls._libs:
            L = C.CDLL(str(LIBS[kind]))
            P, I = C.c_void_p, C.c_int
            for name, res, args in (
                ("vbm_last_error", C.c_char_p, []), ("vbm_create", P, [C.c_char_p]), ("vbm_free", None, [P]),
                ("vbm_quantize", I, [P]), ("vbm_reset_cache", I, [P, I]), ("vbm_to_cuda", I, [P]),
                ("vbm_is_cuda", I, [P]), ("vbm_is_quantized", I, [P]), ("vbm_weight_bytes", C.c_size_t, [P]),
                ("vbm_vocab", I, [P]), ("vbm_step", I, [P, I, P]),
                ("vbm_sampler_create", P, [C.c_float, I, C.c_float, C.c_uint64]),
                ("vbm_sampler_sample", I, [P, P, C.c_int64]), ("vbm_sampler_free", None, [P])):
                f = getattr(L, name)
                f.restype, f.argtypes = res, args
            cls._libs[kind] = L
        return cls._libs[kind]

    def __init__(self, kind, model_dir):
        self.L = self.lib(kind)
        self.h = self.L.vbm_create(str(model_dir).encode())
        if not self.h:
            raise RuntimeError(self.L.vbm_last_error().decode())
        self.vocab = self.L.vbm_vocab(self.h)

    def _ok(self, rc):
        if rc:
            raise RuntimeError(self.L.vbm_last_error().decode())

    def quantize(self):
        self._ok(self.L.vbm_quantize(self.h))

    def reset_cache(self, n):
        self._ok(self.L.vbm_reset_cache(self.h, int(n)))

    def to_cuda(self):
        self._ok(self.L.vbm_to_cuda(self.h))

    def is_cuda(self):
        return bool(self.L.vbm_is_cuda(self.h))

    def weight_bytes(self):
        return int(self.L.vbm_weight_bytes(self.h))

    def step(self, tok):
        out = np.empty(self.vocab, np.float32)
        self._ok(self.L.vbm_step(self.h, int(tok), out.ctypes.data))
        return out

    def sampler(self, temperature, top_k, top_p, seed):
        s = self.L.vbm_sampler_create(temperature, top_k, top_p, seed)
        return lambda lg: self.L.vbm_sampler_sample(
            s, np.ascontiguousarray(lg, np.float32).ctypes.data, lg.size)

    def close(self):
        if self.h:
            self.L.vbm_free(self.h)
            self.h = None


needs_build = pytest.mark.skipif(not all(p.exists() for p in LIBS.values()),
                                 reason="drop-in libraries not built (make -C verbum.cpp_b200/dropin)")

SMALL = vbsynth.qwen3_config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                             num_key_value_heads=2, intermediate_size=512, vocab_size=1000)


@pytest.fixture(scope="module")
def small_dir():
    w = vbsynth.make_weights(SMALL, seed=21, normal=oracle.synth_normal)
    with tempfile.TemporaryDirectory() as td:
        yield vbsynth.write_model_dir(Path(td) / "m", SMALL, w), w


@needs_build
@pytest.mark.parametrize("kind", ["seam", "engine"])
def test_dropin_loads_and_keeps_the_reference_api(kind, small_dir):
    d, w = small_dir
    m = Model(kind, d)
    assert m.vocab == SMALL["vocab_size"]
    o = oracle.OracleModel(SMALL, w)
    assert m.weight_bytes() == o.weight_bytes()
    m.quantize()
    o.quantize()
    assert m.weight_bytes() == o.weight_bytes()
    m.close()
    o.close()


@needs_build
@pytest.mark.skipif(vb200.device_count() > 0, reason="checks the no-device error")
@pytest.mark.parametrize("kind", ["seam", "engine"])
def test_to_cuda_without_a_device_throws_the_reference_error(kind, small_dir):
    m = Model(kind, small_dir[0])
    m.reset_cache(8)
    with pytest.raises(RuntimeError, match="no CUDA device found"):
        m.to_cuda()
    assert not m.is_cuda()
    m.close()


def _run_against_oracle(kind, cfg, w, model_dir, mode, prompt, n_new, sample=None):
    """Model(dir) -> [quantize] -> reset_cache -> to_cuda -> step loop, fed
    the same tokens as the oracle; returns the worst max|diff| of logits and
    checks greedy (or sampled, with the reference's Sampler on both logits
    streams) picks."""
    m = Model(kind, model_dir)
    o = oracle.OracleModel(cfg, w)
    if mode == "int8":
        m.quantize()
        o.quantize()
    n = len(prompt) + n_new + 4
    m.reset_cache(n)
    o.reset_cache(n)
    m.to_cuda()
    assert m.is_cuda()
    pick_m = pick_o = None
    if sample:
        pick_m, pick_o = m.sampler(*sample), m.sampler(*sample)
    worst = 0.0
    for t in prompt:
        lm, lo = m.step(int(t)), o.step(int(t))
        worst = max(worst, float(np.max(np.abs(lm - lo))))
    for i in range(n_new):
        if sample:
            tm, to = pick_m(lm), pick_o(lo)
        else:
            tm, to = int(np.argmax(lm)), oracle.argmax(lo)
        assert tm == to, (kind, mode, i)
        lm, lo = m.step(tm), o.step(to)
        worst = max(worst, float(np.max(np.abs(lm - lo))))
    m.close()
    o.close()
    return worst


@needs_build
@pytest.mark.gpu
def test_seam_reference_step_loop_on_b200_kernels(small_dir):
    d, w = small_dir
    prompt = vbsynth.prompt_ids(9, 4, SMALL["vocab_size"])
    worst = _run_against_oracle("seam", SMALL, w, d, "f32", prompt, 24)
    assert worst <= TOL["f32"], worst


@needs_build
@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_engine_model_small(mode, small_dir):
    d, w = small_dir
    prompt = vbsynth.prompt_ids(9, 4, SMALL["vocab_size"])
    worst = _run_against_oracle("engine", SMALL, w, d, mode, prompt, 24)
    assert worst <= TOL[mode], worst
    # the reference's default sampler (T 0.8, top-k 40, top-p 0.95) on both streams
    worst = _run_against_oracle("engine", SMALL, w, d, mode, prompt, 24, sample=(0.8, 40, 0.95, 7))
    assert worst <= TOL[mode], worst


@needs_build
@pytest.mark.gpu
@pytest.mark.parametrize("mode,kind", [("int8", "engine"), ("f32", "engine"), ("f32", "seam")])
def test_full_qwen3_through_the_reference_model(mode, kind):
    cfg = vbsynth.qwen3_config()
    w = vbsynth.make_weights(cfg, seed=99)
    prompt = vbsynth.prompt_ids(16, 98, cfg["vocab_size"])
    with tempfile.TemporaryDirectory() as td:
        d = vbsynth.write_model_dir(Path(td) / "m", cfg, w)
        worst = _run_against_oracle(kind, cfg, w, d, mode, prompt, 16)
    assert worst <= TOL[mode], worst
