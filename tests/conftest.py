"""Shared pytest setup.

Markers:
  gpu  — needs a CUDA device (B200); run with `-m gpu` on the GPU box.
Everything unmarked runs on CPU only.
"""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "rknn-matmul-parallel_b200")
for p in (REPO, os.path.join(PKG, "python"), PKG, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(REPO, "tests", "golden")


@pytest.fixture(scope="session")
def model_cache(tmp_path_factory):
    """Directory for seeded synthetic models shared by the whole session."""
    root = os.environ.get("B2_MODEL_CACHE")
    if root:
        os.makedirs(root, exist_ok=True)
        return root
    return str(tmp_path_factory.mktemp("models"))
