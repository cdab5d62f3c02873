"""The C-ABI library loads and exports exactly what include/verbum_b200.h
declares (no compute calls: these run on machines without a GPU)."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import vb200

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "verbum_b200.h"


def declared():
    txt = HEADER.read_text()
    return set(re.findall(r"^VB_API [^()]*?\b(vb_\w+)\(", txt, flags=re.M))


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(vb200.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T vb_" in ln}


def test_library_loads():
    L = vb200.lib()
    assert b"sm_100a" in L.vb_version()


def test_every_declared_symbol_is_exported():
    d = declared()
    assert len(d) >= 40
    missing = d - exported()
    assert not missing, missing


def test_binding_covers_header():
    assert declared() == set(vb200.exported_symbols())


def test_library_targets_sm100a():
    # the fatbin carries sm_100a code (cuobjdump's ELF listing only, no disassembly)
    out = subprocess.run(["cuobjdump", "--list-elf", str(vb200.LIB_PATH)], capture_output=True,
                         text=True).stdout
    assert "sm_100a" in out


def test_no_device_means_clean_errors():
    if vb200.device_count() > 0:
        pytest.skip("a GPU is present")
    cfg = {"hidden_size": 256, "num_hidden_layers": 1, "num_attention_heads": 4,
           "num_key_value_heads": 2, "head_dim": 128, "intermediate_size": 512, "vocab_size": 100}
    with pytest.raises(vb200.VBError) as ei:
        vb200.Engine(cfg)
    assert ei.value.code == -2 and "no CUDA device" in ei.value.msg


def test_engine_config_validation_before_device():
    cfg = {"hidden_size": 256, "num_hidden_layers": 1, "num_attention_heads": 4,
           "num_key_value_heads": 2, "head_dim": 64, "intermediate_size": 512, "vocab_size": 100}
    with pytest.raises(vb200.VBError) as ei:
        vb200.Engine(cfg)
    assert ei.value.code == -9


def test_synth_normal_deterministic_and_sliceable():
    a = vb200.synth_normal(100001, seed=9)
    b = vb200.synth_normal(100001, seed=9)
    assert np.array_equal(a, b)
    assert abs(float(a.std()) - 0.02) < 0.001 and abs(float(a.mean())) < 0.001
    assert not np.array_equal(a, vb200.synth_normal(100001, seed=10))
