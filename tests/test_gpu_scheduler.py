"""The step-level scheduler (include/hkv_scheduler.hpp) compiled and run on a
GPU: several requests batched per step through the Q4_K backbone, one of
them queued until a slot frees, each retired with its frames and its slot
released, with the same greedy frames as when the requests run one at a
time; and its host-time counters, read by tests/cpp/scheduler_timing.cpp."""
from __future__ import annotations

import json
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


def compile_program(name, tmp_path):
    gxx = shutil.which("g++", path="/usr/bin:/bin")
    if gxx is None:
        pytest.skip("no system g++")
    lib_dir = REPO / "higgs-audio.cpp_b200" / "lib"
    exe = tmp_path / name
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{REPO / 'include'}",
                    f"-I{CUDA / 'include'}", str(REPO / "tests" / "cpp" / f"{name}.cpp"),
                    f"-L{lib_dir}", "-lhkv", f"-L{CUDA / 'lib64'}", "-lcudart",
                    f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)],
                   check=True)
    return exe


def test_scheduler_batches_and_retires_requests(hkv_lib, tmp_path):
    exe = compile_program("scheduler_test", tmp_path)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "scheduler ok" in res.stdout


def test_scheduler_step_times(hkv_lib, tmp_path):
    """2 layers, 8 timed generation steps at batch 1 and 4: every timed step
    is counted, and host + wait time add up to the step's wall time."""
    exe = compile_program("scheduler_timing", tmp_path)
    res = subprocess.run([str(exe), "2", "8", "1", "4"], capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    lines = [json.loads(x) for x in res.stdout.splitlines() if x.startswith("{")]
    assert [x["batch"] for x in lines] == [1, 4]
    for x in lines:
        assert x["counted_steps"] == 8
        assert x["device_ms_per_step"] > 0 and x["host_us_per_step"] > 0
        assert x["wait_us_per_step"] >= 0
        split_ms = (x["host_us_per_step"] + x["wait_us_per_step"]) / 1e3
        assert split_ms <= x["wall_ms_per_step"] * 1.001 + 1e-3
        assert split_ms >= x["wall_ms_per_step"] * 0.9
