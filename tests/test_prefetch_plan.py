"""The DWDP engine's prefetch planning (owner interleaving, per-expert slices, coalesced
runs of an owner's contiguous experts) as a host-only C++ unit test: compiled with g++
from the engine's own header and run on the CPU."""
import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
CSRC = ROOT / "dwdp-triton-moe-inference-engine_b200" / "csrc"


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_prefetch_plan(tmp_path):
    exe = tmp_path / "test_prefetch_plan"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", f"-I{CSRC}", str(ROOT / "tests" / "cpp" / "test_prefetch_plan.cpp"),
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    assert "all checks passed" in res.stdout
