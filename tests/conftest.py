"""Shared test helpers. GPU tests are marked `gpu` and need a CUDA device plus the built library."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


PARITY = {}   # measured distances, by section and case: written to $MOTEOPT_PARITY_RECORD at the end of the session


def record(section: str, case: str, values: dict) -> None:
    """Keep a test's measured distances (relative Frobenius and the like) for the session's parity record."""
    PARITY.setdefault(section, {})[case] = {k: float(v) for k, v in values.items()}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libmoteopt.so")


def pytest_sessionfinish(session, exitstatus):
    import json
    path = os.environ.get("MOTEOPT_PARITY_RECORD")
    if path and PARITY:
        with open(path, "w") as f:
            json.dump(PARITY, f, indent=1, sort_keys=True)


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
