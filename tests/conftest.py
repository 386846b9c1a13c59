"""Test setup: the repository root on sys.path, the `gpu` marker, and the package handle.

Tests marked `gpu` need a B200 and the built libq38.so; the rest run on CPU.
"""

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libq38.so")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("qwen38-27b-aws_b200")
