import importlib
import json
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden" / "quant_golden.json"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; runs the CUDA kernels")


@pytest.fixture(scope="session")
def clq():
    return importlib.import_module("cl-inference_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("cl-inference_b200.synth")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    return o


def load_golden():
    doc = json.loads(GOLDEN.read_text())
    out = {}
    for name, f in doc["fixtures"].items():
        out[name] = {
            "bytes": np.frombuffer(bytes.fromhex(f["bytes_hex"]), np.uint8).copy(),
            "values": np.frombuffer(bytes.fromhex(f["value_bits_hex"]), "<f4").astype(np.float32),
            "elements": f["elements"],
            "block_bytes": f["block_bytes"],
            "ggml_type": f["ggml_type"],
            "bad_offsets": f["nonfinite_scale_offsets"],
        }
    return out


@pytest.fixture(scope="session")
def golden():
    return load_golden()


@pytest.fixture(scope="session")
def cuda():
    """A usable CUDA device; a gpu-marked test without one fails rather than skips."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch
