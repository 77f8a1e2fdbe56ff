import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA device) and the built CUDA library")


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False)


def cases(z, key="names"):
    return [str(n) for n in z[key]]


def cdict(z, prefix, w=None):
    d = {k: z[f"{prefix}{k}"] for k in ("m8", "e4", "rp", "er", "ec", "ev")}
    d["base"] = int(z[f"{prefix}base"])
    d["N"], d["K"] = d["m8"].shape
    d["CH"] = 256
    return d


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
