import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "komp_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


class Golden:
    """Reference outputs recorded by tests/golden/make_golden.py (COMP under TRITON_INTERPRET=1)."""

    def __init__(self, path):
        self.z = np.load(path)
        self.manifest = json.loads(bytes(self.z["manifest"]).decode())

    def __getitem__(self, k):
        return self.z[k]

    def cases(self):
        return self.manifest["gemv"]

    def case(self, cid):
        return {k.split("/")[-1]: self.z[k] for k in self.z.files if k.startswith(f"gemv/{cid}/")}


@pytest.fixture(scope="session")
def golden():
    return Golden(GOLDEN)


def golden_case_ids():
    return [c["id"] for c in json.loads(bytes(np.load(GOLDEN)["manifest"]).decode())["gemv"]]


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comp_b200 import _lib

    _lib.load()  # the product path must load the in-tree CUDA library; a missing build fails here
    return torch.device("cuda:0")
