"""Shared test setup: import paths, the gpu marker, device fixtures.

-m "not gpu" runs here without a GPU: the oracle against the reference's golden vectors, host logic (GGUF reader,
argument checks, the page scheduler), and that libocrcuda.so loads and exports every declared symbol.
-m gpu runs on a B200: the CUDA path through the C ABI against the oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "historic-htr-ocr_b200", ROOT / "oracle", ROOT / "tests", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")


@pytest.fixture(scope="session")
def ocr():
    import ocr_b200

    ocr_b200.lib()  # loud if the library is not built
    return ocr_b200


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ctx(ocr):
    c = ocr.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    return torch
