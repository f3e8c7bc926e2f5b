"""The C++ pipeline shim (include/hkv_pipeline.hpp) compiled and run on CPU
against a host-only engine: the reference's slot names, RAII release and
exception types (std::runtime_error, std::out_of_range)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def test_shim_compiles_and_behaves(hkv_lib, tmp_path):
    gxx = shutil.which("g++", path="/usr/bin:/bin")
    if gxx is None:
        pytest.skip("no system g++")
    lib_dir = REPO / "higgs-audio.cpp_b200" / "lib"
    exe = tmp_path / "shim_test"
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{REPO / 'include'}",
                    str(REPO / "tests" / "cpp" / "shim_test.cpp"), f"-L{lib_dir}", "-lhkv",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "shim ok" in res.stdout
