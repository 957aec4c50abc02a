"""Shared pytest setup: the `gpu` marker, the package under test and the oracle.

The package directory is ``nari-qwen3-tts_b200`` (not an identifier), so it is
imported with importlib.  GPU tests are marked ``gpu`` and run only on a
machine with a CUDA device; everything else runs on the CPU.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libnqt.so")


def load_package():
    return importlib.import_module("nari-qwen3-tts_b200")


@pytest.fixture(scope="session")
def nqt():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    def load(name: str):
        return torch.load(GOLDEN / name, weights_only=False)

    return load


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)
