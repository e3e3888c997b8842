"""Builds and runs the C++ host mirror test (tests/cpp/mirror_test.cpp)."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "kernix_b200"


def _build(tmp_path) -> Path:
    exe = tmp_path / "mirror_test"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-I", str(ROOT / "include"), str(ROOT / "tests/cpp/mirror_test.cpp"),
           "-L", str(LIBDIR), "-lkernix_b200", f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)]
    subprocess.run(cmd, check=True)
    return exe


def test_cpp_mirror_host(tmp_path):
    out = subprocess.run([str(_build(tmp_path)), "--host"], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "mirror_test ok" in out.stdout


@pytest.mark.gpu
def test_cpp_mirror_gpu(tmp_path):
    out = subprocess.run([str(_build(tmp_path)), "--gpu"], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "host+gpu" in out.stdout
