"""Shared fixtures.

* ``qmv``       the product package (my-inference-engine_b200/), loaded by path.
* ``workloads`` the seeded workload generator of that package.
* ``oracle``    the C restatement of the reference's scalar path (checker only).
* ``ref``       the reference's own sources compiled into oracle/_ref (checker
                only; skipped when neither the built library nor the reference
                sources are available).

Tests that need a B200 are marked ``gpu``; everything else runs on CPU.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "my-inference-engine_b200")


def _load(name: str, path: str):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_package():
    return _load("my_inference_engine_b200", os.path.join(PKG_DIR, "__init__.py"))


def load_workloads():
    return _load("qmv_workloads", os.path.join(PKG_DIR, "workloads.py"))


def load_oracle_binding():
    return _load("qmv_oracle_binding", os.path.join(REPO, "oracle", "binding.py"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


@pytest.fixture(scope="session")
def qmv():
    mod = load_package()
    if not os.path.exists(mod.LIB_PATH):
        _load("qmv_build", os.path.join(PKG_DIR, "build.py")).build_library()
    mod.load_library()
    return mod


@pytest.fixture(scope="session")
def workloads():
    return load_workloads()


@pytest.fixture(scope="session")
def oracle():
    b = load_oracle_binding()
    if not os.path.exists(b.ORACLE_SO):
        b.build(reference=False)
    return b.Oracle()


@pytest.fixture(scope="session")
def ref():
    b = load_oracle_binding()
    if not os.path.exists(b.REF_SCALAR_SO):
        if not os.path.isdir(os.path.join(b.REFERENCE_SRC, "src")):
            pytest.skip("reference library not built and reference sources absent")
        b.build(reference=True)
    return b.Reference(b.REF_SCALAR_SO)


@pytest.fixture(scope="session")
def cuda():
    """torch with a usable CUDA device, or skip (gpu tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def lcg_bytes(n: int, state: int = 0x12345678):
    """The reference tests' LCG (rng = rng * 1664525 + 1013904223, byte = rng >> 24),
    e.g. tests/q8_0_reference_test.cpp:112-118.  Returns (bytes, final state)."""
    out = np.empty(n, dtype=np.uint8)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = state >> 24
    return out, state


def tolerance_ok(y, y_ref, s, rel=1e-4):
    """|y - y_ref| <= rel * sum|w x| per row (the parity bound), vectorised."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    err = np.abs(y - y_ref)
    bound = rel * np.asarray(s, dtype=np.float64)
    bad = np.nonzero(err > bound)[0]
    return bad, err, bound
