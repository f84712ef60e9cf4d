import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size model cases (minutes on the CPU oracle)")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("MGB_MODEL_DIR") or str(tmp_path_factory.mktemp("models"))
    os.makedirs(d, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def model(model_dir):
    """model(name, preset, seed=0) -> GGUF path (generated once per session)."""
    from malaga_b200 import models

    def get(name, preset, seed=0):
        return models.model_path(name, preset, seed, model_dir)

    return get


@pytest.fixture(scope="session")
def gpu():
    if not gpu_available():
        pytest.skip("no CUDA device")
    from malaga_b200 import _lib

    _lib.load()  # fails loudly if the engine library is missing
    return 0
