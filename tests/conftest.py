"""Shared test setup.

Tests marked `gpu` need an sm_100 device and the built library (adai_b200/libadai_b200.so); the
rest run on any host. The CPU oracles (oracle/) are the checkers in both.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_outputs.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")


def tol_ok(got, want, rel=1e-4, abs_=1e-5):
    """The parity bound of the decode path: |got - want| <= abs + rel * |want| elementwise."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return bool(np.all(np.abs(got - want) <= abs_ + rel * np.abs(want)))


def tol_ratio(got, want, rel=1e-4, abs_=1e-5):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want) / (abs_ + rel * np.abs(want))))


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def port():
    from oracle.pyoracle import Port
    return Port()


@pytest.fixture(scope="session")
def ctx():
    from adai_b200 import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    return torch
