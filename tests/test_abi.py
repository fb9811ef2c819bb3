"""The C-ABI library loads and exports every symbol the public headers declare (no GPU calls)."""
import ctypes
import os
import re
import subprocess

import varblockspmm_b200 as vb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "vbsr_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vbsr_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(vb.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_cxx_dropin_library_links():
    path = os.path.join(os.path.dirname(vb.LIB_PATH), "libvbsr_b200_cxx.so")
    assert os.path.exists(path)
    ctypes.CDLL(path)
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", path], capture_output=True,
                         text=True).stdout
    for name in ("vbsr::Plan::execute", "vbsr::Matrix::Matrix", "vbsr::HostMatrix::validate",
                 "vbsr::generate", "vbsr::launch_row_owned", "vbsr::launch_row_owned_scalar",
                 "vbsr::MultiPlan::MultiPlan", "vbsr::MultiPlan::replicate_B",
                 "vbsr::MultiPlan::execute", "vbsr::MultiPlan::gather_C",
                 "vbsr::ScalarCsrPlan::execute", "vbsr::GroupedGemmPlan::execute",
                 "vbsr::GroupedGemmPlan::launch_count"):
        assert name in out, name


def test_errors_are_thread_local_and_cleared():
    v = vb.HostMatrix()
    try:
        v.validate()
    except vb.InvalidArgument as e:
        assert "positive block dimensions" in str(e)
    m = vb.generate(vb.GeneratorOptions(4, 4, 2))
    m.validate()
    assert vb.last_error() == ""
