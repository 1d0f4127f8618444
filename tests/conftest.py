import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

FIXTURE_DIR = os.environ.get("QASR_FIXTURE_DIR", "/tmp/qasr_fixtures")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libqwen_asr.so")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def model_dir(preset: str, seed: int = 0) -> str:
    """Seeded synthetic checkpoint in the reference layout (generated once per machine)."""
    from qwen_asr_b200 import synth
    d = os.path.join(FIXTURE_DIR, f"{preset}-s{seed}")
    dev = "cuda" if (preset != "tiny" and _has_gpu()) else "cpu"
    synth.write_model(d, preset, seed, device=dev)
    return d


@pytest.fixture(scope="session")
def tiny_dir():
    return model_dir("tiny", 0)


@pytest.fixture(scope="session")
def m06_dir():
    return model_dir("0.6b", 0)


@pytest.fixture(scope="session")
def m17_dir():
    return model_dir("1.7b", 1)


@pytest.fixture(scope="session")
def m17l4_dir():
    return model_dir("1.7b-l4", 1)
