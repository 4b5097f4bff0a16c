"""Test configuration: import paths, the `gpu` marker and shared helpers.

Tests marked ``gpu`` need a CUDA device (a B200 for the tensor-core paths) and
call the library through its C ABI (``cuda_operator_lab.bindings``); all
other tests run on CPU.  ``oracle`` is the CPU restatement of the reference's
math and is used only as the checker.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "cuda-operator-lab_b200"
for p in (str(PACKAGE_DIR), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device; calls the sm_100a library")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def seeded(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


@pytest.fixture(scope="session")
def golden() -> list[dict]:
    data = torch.load(ROOT / "tests" / "golden" / "reference_cases.pt", weights_only=True)
    return data["cases"]
