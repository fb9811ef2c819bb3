"""oracle — TEST INFRASTRUCTURE ONLY (the parity checker; never the thing measured or shipped).

Python bindings for
  * _build/libvbsr_oracle.so: vbsr_oracle.c, the CPU restatement of the reference's
    double-accumulating cpu_reference (src/format/vbsr.cpp:167-201), bit-identical to it, plus the
    per-element bound S = sum |a||b|;
  * _ref/libvbsr_ref.so (when present): the reference's own src/format/{vbsr,generator}.cpp
    compiled unchanged by oracle/Makefile, with the C shim ref_shim.cpp;
  * _ref/libvbsr_ref_gpu.so (when present): the reference's own GPU path (Matrix, Plan and the
    row-owned CUDA kernels) compiled unchanged for sm_100a, with the C shim ref_gpu_shim.cpp.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(_HERE, "_build", "libvbsr_oracle.so")
REF_LIB = os.path.join(_HERE, "_ref", "libvbsr_ref.so")
REF_GPU_LIB = os.path.join(_HERE, "_ref", "libvbsr_ref_gpu.so")


def build(ref_dir: str | None = None) -> None:
    """Builds the oracle (and the reference, when its checkout is given by `ref_dir` or the
    environment variable VBSR_REFERENCE_DIR) with oracle/Makefile."""
    ref_dir = ref_dir or os.environ.get("VBSR_REFERENCE_DIR", "")
    subprocess.run(["make", "-s", "-C", _HERE, "REF=" + ref_dir], check=True)


if not os.path.exists(ORACLE_LIB):
    build()
_olib = C.CDLL(ORACLE_LIB)
_olib.vbsr_oracle_spmm.restype = C.c_int
_olib.vbsr_oracle_spmm.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int32, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_int]
_olib.vbsr_oracle_compare.restype = C.c_int
_olib.vbsr_oracle_compare.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int32, C.c_int32,
                                      C.c_void_p, C.c_int, C.POINTER(C.c_double),
                                      C.POINTER(C.c_double), C.POINTER(C.c_int64)]

_rlib = None
if os.path.exists(REF_LIB):
    _rlib = C.CDLL(REF_LIB)
    _rlib.ref_last_error.restype = C.c_char_p
    _rlib.ref_generate.restype = C.c_void_p
    _rlib.ref_generate.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64]
    _rlib.ref_free.argtypes = [C.c_void_p]
    _rlib.ref_arrays.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    _ref_args = [C.c_void_p] * 10
    _rlib.ref_validate.argtypes = _ref_args
    _rlib.ref_validate.restype = C.c_int
    _rlib.ref_cpu_reference_rows.argtypes = _ref_args + [C.c_void_p, C.c_int, C.c_int, C.c_int,
                                                         C.c_void_p, C.c_int]
    _rlib.ref_cpu_reference_rows.restype = C.c_int


def ref_available() -> bool:
    return _rlib is not None


_glib = None


def ref_gpu_available() -> bool:
    """True when the reference's GPU library is built (loaded lazily: it needs a CUDA driver)."""
    return os.path.exists(REF_GPU_LIB)


def _ref_gpu_lib():
    global _glib
    if _glib is None:
        _glib = C.CDLL(REF_GPU_LIB)
        _glib.ref_gpu_last_error.restype = C.c_char_p
        _glib.ref_gpu_create.restype = C.c_void_p
        _glib.ref_gpu_create.argtypes = [C.c_void_p] * 10 + [C.c_int]
        _glib.ref_gpu_execute.restype = C.c_int
        _glib.ref_gpu_execute.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        _glib.ref_gpu_launch_count.restype = C.c_int
        _glib.ref_gpu_launch_count.argtypes = [C.c_void_p]
        _glib.ref_gpu_destroy.argtypes = [C.c_void_p]
    return _glib


class RefGpuPlan:
    """The reference's own Matrix + Plan (row-owned kernels) on the current CUDA device, for
    tests that run the reference's GPU path next to the engine's. execute() takes device
    pointers (ints) and a raw stream handle (0 = the legacy default stream)."""

    def __init__(self, host, rhs: int):
        lib = _ref_gpu_lib()
        args, keep = _ref_view_args(host)
        self._h = lib.ref_gpu_create(*args, rhs)
        del keep
        if not self._h:
            raise RuntimeError("reference Matrix/Plan: " + lib.ref_gpu_last_error().decode())

    def execute(self, B_ptr: int, C_ptr: int, stream: int = 0):
        lib = _ref_gpu_lib()
        if lib.ref_gpu_execute(self._h, B_ptr, C_ptr, stream or None) != 0:
            raise RuntimeError("reference Plan::execute: " + lib.ref_gpu_last_error().decode())

    def launch_count(self) -> int:
        return _ref_gpu_lib().ref_gpu_launch_count(self._h)

    def close(self):
        if self._h:
            _ref_gpu_lib().ref_gpu_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _threads(t):
    return t if t and t > 0 else (os.cpu_count() or 1)


def spmm(host, B, rhs: int, r0: int = 0, r1: int | None = None, threads: int = 0,
         bound: bool = False):
    """Oracle C (and S if bound) for block rows [r0, r1), column-major flattened, ld = rows of the
    range. `host` is a varblockspmm_b200.HostMatrix in the reference layout."""
    r1 = host.block_rows if r1 is None else r1
    B = _f32(B)
    v = host.view()
    rows = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    Cm = np.empty(rows * rhs, dtype=np.float32)
    S = np.empty(rows * rhs, dtype=np.float64) if bound else None
    rc = _olib.vbsr_oracle_spmm(C.addressof(v), B.ctypes.data, rhs, r0, r1, Cm.ctypes.data,
                                S.ctypes.data if bound else None, _threads(threads))
    if rc != 0:
        raise ValueError("oracle rejected its arguments")
    return (Cm, S) if bound else Cm


def compare(host, B, rhs: int, Ctest, r0: int = 0, r1: int | None = None, threads: int = 0):
    """(max error/limit ratio, max abs error, violations) of Ctest against the oracle under
    |C - C_ref| <= 1e-5 * sum|a||b| per element."""
    r1 = host.block_rows if r1 is None else r1
    B = _f32(B)
    Ct = _f32(Ctest)
    v = host.view()
    mr, ma, nb = C.c_double(), C.c_double(), C.c_int64()
    rc = _olib.vbsr_oracle_compare(C.addressof(v), B.ctypes.data, rhs, r0, r1, Ct.ctypes.data,
                                   _threads(threads), C.byref(mr), C.byref(ma), C.byref(nb))
    if rc != 0:
        raise ValueError("oracle rejected its arguments")
    return mr.value, ma.value, nb.value


# ---- the reference itself -------------------------------------------------------------------------

def _ref_view_args(host):
    v = host.view()  # normalises dtypes and keeps arrays alive on `host`
    dims = np.array([host.block_rows, host.block_cols], dtype=np.int32)
    lens = np.array([host.row_ptr.size, host.block_col.size, host.row_size.size,
                     host.col_size.size, host.row_scalar_off.size, host.col_scalar_off.size,
                     host.value_off.size, host.values.size], dtype=np.int64)
    args = [dims.ctypes.data, host.row_ptr.ctypes.data, host.block_col.ctypes.data,
            host.row_size.ctypes.data, host.col_size.ctypes.data,
            host.row_scalar_off.ctypes.data, host.col_scalar_off.ctypes.data,
            host.value_off.ctypes.data, host.values.ctypes.data, lens.ctypes.data]
    return args, (dims, lens, v)


def ref_generate(rows, cols, degree, distribution, local, seed):
    """The reference's generate() -> dict of numpy arrays."""
    h = _rlib.ref_generate(rows, cols, degree, int(distribution), int(bool(local)), seed)
    if not h:
        raise ValueError(_rlib.ref_last_error().decode())
    try:
        dims = np.zeros(2, dtype=np.int32)
        ptrs = (C.c_void_p * 8)()
        lens = np.zeros(8, dtype=np.int64)
        _rlib.ref_arrays(h, dims.ctypes.data, C.addressof(ptrs), lens.ctypes.data)
        names = ["row_ptr", "block_col", "row_size", "col_size", "row_scalar_off",
                 "col_scalar_off", "value_off", "values"]
        types = [C.c_int32] * 4 + [C.c_int64] * 3 + [C.c_float]
        out = {"block_rows": int(dims[0]), "block_cols": int(dims[1])}
        for i, (n, t) in enumerate(zip(names, types)):
            if lens[i] == 0:
                out[n] = np.zeros(0, dtype=np.ctypeslib.as_ctypes_type(t) and t)
                continue
            arr = np.ctypeslib.as_array(C.cast(ptrs[i], C.POINTER(t)), shape=(int(lens[i]),))
            out[n] = arr.copy()
        return out
    finally:
        _rlib.ref_free(h)


def ref_validate(host):
    """(code, message): 0 valid, 1 std::invalid_argument, 2 other."""
    args, keep = _ref_view_args(host)
    rc = _rlib.ref_validate(*args)
    return rc, (_rlib.ref_last_error().decode() if rc else "")


def ref_cpu_reference(host, B, rhs: int, r0: int = 0, r1: int | None = None, threads: int = 1):
    """The reference's own cpu_reference over block rows [r0, r1), run as `threads` independent
    calls on row slices."""
    r1 = host.block_rows if r1 is None else r1
    B = _f32(B)
    args, keep = _ref_view_args(host)
    rows = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    Cm = np.empty(rows * rhs, dtype=np.float32)
    rc = _rlib.ref_cpu_reference_rows(*args, B.ctypes.data, rhs, r0, r1, Cm.ctypes.data, threads)
    if rc != 0:
        raise ValueError(_rlib.ref_last_error().decode())
    return Cm
