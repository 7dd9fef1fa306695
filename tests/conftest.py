"""Test configuration: the ``gpu`` marker, repository import path, shared fixtures.

``-m "not gpu"`` runs on any machine (oracle pins, host logic, the C ABI's exports and planner).
``-m gpu`` needs an sm_100 GPU: it exercises the CUDA kernels through the C ABI and compares them with the
oracle and the golden fixtures produced by the reference's own CPU programs.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built native library")


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def gpu() -> None:
    """Skip-free guard: GPU tests fail loudly (not skip) when the device or library is missing."""
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, f"GPU tests need sm_100 (B200), found {torch.cuda.get_device_name(0)}"
    from chroma_b200.build import build

    build()
