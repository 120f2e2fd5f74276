"""Shared fixtures and markers.

Tests marked ``gpu`` need a CUDA device (a B200: the kernels are built for sm_100a only) and
are skipped elsewhere. Everything else runs on CPU: the oracle against the reference's golden
vectors, host-side logic, and the C ABI surface of the kernel library (symbols and host-only
entry points; no kernel launches).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    skip_gpu = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords and not HAS_CUDA:
            item.add_marker(skip_gpu)


@pytest.fixture(scope="session")
def device() -> torch.device:
    if not HAS_CUDA:
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


@pytest.fixture(autouse=True)
def _reset_counters():  # type: ignore[no-untyped-def]
    from tokenforge_b200.metrics import FALLBACKS, KERNEL_CALLS

    KERNEL_CALLS.reset()
    FALLBACKS.reset()
    yield
