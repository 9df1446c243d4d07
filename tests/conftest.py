"""Shared fixtures for the libkernelsmith (B200) tests.

Markers:
  gpu -- needs a CUDA device (B200); run with `pytest -m gpu`.
Everything unmarked runs on a CPU-only host.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT / "oracle", ROOT / "ulir-kernels_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def ks():
    """The ctypes-bound libkernelsmith (B200)."""
    import kernelsmith_b200 as K

    K.lib()
    return K


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    return O.Oracle()


@pytest.fixture(scope="session")
def smoke_bundles():
    return json.loads((GOLDEN / "reference_smoke.json").read_text())


@pytest.fixture(scope="session")
def seeded():
    meta = json.loads((GOLDEN / "ref_seeded.json").read_text())
    arrays = dict(np.load(GOLDEN / "ref_seeded.npz"))
    return meta, arrays


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def bundle_array(bundle: dict, name: str) -> np.ndarray:
    t = bundle["tensors"][name]
    return np.asarray(t["data"], dtype=t["dtype"]).reshape(t["shape"])
