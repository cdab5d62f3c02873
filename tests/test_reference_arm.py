"""The benchmark's reference arm must run the reference's own code only.

bench.py --impl reference times oracle/_ref (the reference engine compiled
from its sources) on weights drawn by the oracle's copy of the synthetic
generator, so the process never maps the engine library.  These tests check
that the two generators give bit-identical weights (so both arms decode the
same model) and, in a fresh process, that producing the reference arm's
weights maps no libverbum_b200.so.
"""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
import vb200

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("n,seed", [(1, 5), (7, 2**63 + 5), (1_000_003, 1234 * 1000003 + 7)])
def test_oracle_generator_equals_engine_generator(n, seed):
    a = vb200.synth_normal(n, seed, 0.02)
    b = oracle.synth_normal(n, seed, 0.02)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_reference_arm_weights_do_not_load_the_engine_library():
    code = (
        "import sys; sys.path[:0] = [%r, %r, %r]\n"
        "import bench, vbsynth\n"
        "cfg = vbsynth.qwen3_config(hidden_size=256, num_hidden_layers=1, num_attention_heads=4,"
        " num_key_value_heads=2, intermediate_size=512, vocab_size=1000)\n"
        "w = bench.reference_weights(cfg)\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('ENGINE' if 'libverbum_b200' in maps else 'CLEAN', len(w))\n"
    ) % (str(ROOT), str(ROOT / "verbum.cpp_b200"), str(ROOT / "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split()[0] == "CLEAN", r.stdout
