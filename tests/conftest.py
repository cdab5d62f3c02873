import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "verbum.cpp_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def mini_config(**over):
    """A small Qwen3-shaped model: real head_dim / GQA ratio, few layers."""
    import vbsynth
    c = vbsynth.qwen3_config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                             num_key_value_heads=2, intermediate_size=512, vocab_size=1000)
    c.update(over)
    return c
