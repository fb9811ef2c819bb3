"""The C++ drop-in API, compiled and run as a program (tests/cxx/test_dropin.cpp): the reference's
own test binary (tests/test_main.cpp:14-177) rewritten against include/varblockspmm/vbsr.hpp, with
the engine's libvbsr_b200_cxx.so and the oracle's cpu_reference, plus a scalar CSR matrix
through from_csr and the VBSR file. The build is checked on any
machine; running it needs the GPU."""
import os
import subprocess

import pytest

import varblockspmm_b200 as vb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(out_dir):
    exe = os.path.join(str(out_dir), "test_dropin")
    libdir = os.path.dirname(vb.LIB_PATH)
    oracle_dir = os.path.join(ROOT, "oracle", "_build")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-I" + os.path.join(ROOT, "include"),
           "-I" + CUDA + "/include", os.path.join(ROOT, "tests", "cxx", "test_dropin.cpp"),
           "-o", exe, "-L" + libdir, "-lvbsr_b200_cxx", "-lvbsr_b200",
           "-L" + oracle_dir, "-l:libvbsr_oracle.so", "-L" + CUDA + "/lib64", "-lcudart",
           "-Wl,-rpath," + libdir, "-Wl,-rpath," + oracle_dir, "-Wl,-rpath," + CUDA + "/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cxx_dropin_program_builds(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_cxx_dropin_program_runs(cuda, tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout
