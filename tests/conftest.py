import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "wasm-chord_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_DIR = os.environ.get("WCB_MODEL_DIR", os.path.join("/tmp", "wcb_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes)")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_dir():
    os.makedirs(MODEL_DIR, exist_ok=True)
    return MODEL_DIR


@pytest.fixture(scope="session")
def tiny_gguf(model_dir):
    from wcb import synth
    return synth.cached_model("tiny", model_dir)


@pytest.fixture(scope="session")
def tiny_mix_gguf(model_dir):
    from wcb import synth
    return synth.cached_model("tiny_mix", model_dir)


@pytest.fixture(scope="session")
def gpu():
    if not cuda_available():
        pytest.fail("this test needs a CUDA GPU")
    return True
