"""Shared test setup: the `gpu` marker, import paths and common fixtures.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's
known-answer patterns and golden fixtures, the engine's host-side
bookkeeping (a host-only engine, device=-1) and the C-ABI exports.  GPU tests
(`-m gpu`) are the parity tests: the CUDA path through the C ABI against the
oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "higgs-audio.cpp_b200"
for p in (str(REPO), str(PKG), str(REPO / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def oracle():
    import cpu_oracle
    cpu_oracle.build()
    return cpu_oracle


@pytest.fixture(scope="session")
def hkv_lib():
    import hkv_build
    hkv_build.build()
    import hkv
    return hkv.load_library()


@pytest.fixture(scope="session")
def rope_tables(oracle):
    return oracle.rope_table(32768, 128, 1e6)
