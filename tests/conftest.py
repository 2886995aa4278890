"""Shared pytest configuration.

``-m gpu`` tests need a B200 and the in-tree ``libpbgb200.so``; every other
test runs on CPU.  The package directory and the oracle are put on
``sys.path`` here so tests import them the same way on every machine.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("ai-game-learning_b200", "oracle"):
    path = os.path.join(ROOT, sub)
    if path not in sys.path:
        sys.path.insert(0, path)
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built library")


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def gold():
    cache: dict = {}

    def get(name):
        if name not in cache:
            cache[name] = golden(name)
        return cache[name]

    return get
