"""Shared pytest configuration: the ``gpu`` marker, package import, golden data."""

from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_NAME = "deepseek-v4-experimental-platform-on-dgx-spark_b200"
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def import_pkg():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def pkg():
    return import_pkg()


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


def rel_fro(out_bits: np.ndarray, ref_bits: np.ndarray) -> float:
    from oracle import blockscaled as ob
    o = ob.bf16_to_f32(out_bits).astype(np.float64)
    r = ob.bf16_to_f32(ref_bits).astype(np.float64)
    return float(np.linalg.norm(o - r) / max(np.linalg.norm(r), 1e-30))


def max_abs(out_bits: np.ndarray, ref_bits: np.ndarray) -> float:
    from oracle import blockscaled as ob
    o = ob.bf16_to_f32(out_bits).astype(np.float64)
    r = ob.bf16_to_f32(ref_bits).astype(np.float64)
    return float(np.abs(o - r).max()) if o.size else 0.0
