import importlib
import pathlib
import sys

import numpy as np
import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
PKG_NAME = "mlsys26-flashinfer-ai-kernel-generation-contest_b200"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    return importlib.import_module(PKG_NAME)


def load_golden(name: str):
    """Load a tests/golden/*.npz fixture -> (tensors, meta)."""
    z = np.load(GOLDEN / f"{name}.npz")
    tensors, meta = {}, {}
    for key in z.files:
        if key.startswith("meta__"):
            meta[key[6:]] = z[key].item()
        elif not key.endswith("__dtype"):
            dt = str(z[key + "__dtype"])
            t = torch.from_numpy(z[key].copy())
            if dt == "bfloat16":
                t = t.view(torch.bfloat16)
            tensors[key] = t
    return tensors, meta


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
