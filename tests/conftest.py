import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("rf-detr.cpp_b200", "oracle", "tests"):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


_MODELS = {}


@pytest.fixture(scope="session")
def make_model(model_dir):
    """Write (and cache) a synthetic GGUF: make_model(variant, dtype, seed)."""
    from rfdetr_b200 import synth

    def _make(variant, dtype="f32", seed=0):
        key = (variant, dtype, seed)
        if key not in _MODELS:
            path = str(model_dir / f"{variant}-{dtype}-{seed}.gguf")
            synth.write_model(path, variant, dtype, seed)
            _MODELS[key] = path
        return _MODELS[key]

    return _make
