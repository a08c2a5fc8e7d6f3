import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "index-tts-rs_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _ensure_built():
    pkg = ROOT / "index-tts-rs_b200"
    need = [pkg / "libitts_gpt.so", pkg / "libitts_synth.so", ROOT / "oracle" / "libitts_oracle.so"]
    if not all(p.exists() for p in need):
        import __graft_entry__
        __graft_entry__.build()


_ensure_built()


@pytest.fixture(scope="session")
def small_cfg():
    from itts_gpt.synth import SMALL
    return SMALL


@pytest.fixture(scope="session")
def small_weights(small_cfg):
    from itts_gpt.synth import make_weights
    return make_weights(small_cfg, seed=7, ln_beta_std=0.02)
