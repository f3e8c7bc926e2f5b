"""The step-level scheduler (include/hkv_scheduler.hpp) compiled and run on a
GPU: several requests batched per step through the Q4_K backbone, one of
them queued until a slot frees, each retired with its frames and its slot
released, with the same greedy frames as when the requests run one at a
time."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


def test_scheduler_batches_and_retires_requests(hkv_lib, tmp_path):
    gxx = shutil.which("g++", path="/usr/bin:/bin")
    if gxx is None:
        pytest.skip("no system g++")
    lib_dir = REPO / "higgs-audio.cpp_b200" / "lib"
    exe = tmp_path / "scheduler_test"
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{REPO / 'include'}",
                    f"-I{CUDA / 'include'}", str(REPO / "tests" / "cpp" / "scheduler_test.cpp"),
                    f"-L{lib_dir}", "-lhkv", f"-L{CUDA / 'lib64'}", "-lcudart",
                    f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)],
                   check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "scheduler ok" in res.stdout
