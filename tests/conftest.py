import hashlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

TINY_MODELS = ("tiny_f16", "tiny_q8", "tiny_q4")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def golden_model(name: str) -> str:
    return os.path.join(GOLDEN, name + ".gguf")


def file_sha256(path: str) -> bytes:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.digest()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def smollm_models(model_dir):
    """135M-shaped GGUFs regenerated from their seeds, checked against the fixture sha256."""
    from laicompute_b200 import synth
    out = {}
    for name, arch in (("smollm135m_f16", synth.SMOL_135M_F16), ("smollm135m_q8", synth.SMOL_135M_Q8)):
        g = golden(name)
        path = os.path.join(model_dir, name + ".gguf")
        synth.write_model(path, arch, seed=int(g["seed"][0]))
        assert file_sha256(path) == g["sha256"].tobytes(), f"{name}: regenerated GGUF differs from the fixture's"
        out[name] = path
    return out
