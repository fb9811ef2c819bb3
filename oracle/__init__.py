"""oracle — TEST INFRASTRUCTURE ONLY (the parity checker; never the thing measured or shipped).

Python bindings for
  * _build/libvbsr_oracle.so: vbsr_oracle.c, the CPU restatement of the reference's
    double-accumulating cpu_reference (src/format/vbsr.cpp:167-201), bit-identical to it, plus the
    per-element bound S = sum |a||b|;
  * _ref/libvbsr_ref.so (when present): the reference's own src/format/{vbsr,generator}.cpp
    compiled unchanged by oracle/Makefile, with the C shim ref_shim.cpp;
  * _ref/libvbsr_ref_gpu.so (when present): the reference's own GPU path (Matrix, Plan and the
    row-owned CUDA kernels) compiled unchanged for sm_100a, with the C shim ref_gpu_shim.cpp.
  * workload.cpp (in _build/libvbsr_oracle.so): the benchmark workloads' block structure and
    counter-based values, generated without the engine library (WorkloadMatrix), so that the
    benchmark's reference arm never loads the product.
This package does not import the engine package; any object with the HostMatrix fields (numpy
arrays row_ptr, block_col, ... values) is accepted where a matrix is expected.
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
_olib.oracle_fill_uniform.restype = C.c_int
_olib.oracle_fill_uniform.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p,
                                      C.c_int]
_olib.oracle_spec_structure.restype = C.c_int
_olib.oracle_spec_structure.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                        C.c_void_p, C.c_void_p, C.c_void_p]
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
    _rlib.ref_prepare.argtypes = _ref_args + [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
    _rlib.ref_prepare.restype = C.c_void_p
    _rlib.ref_run.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_double)]
    _rlib.ref_run.restype = C.c_int
    _rlib.ref_release.argtypes = [C.c_void_p]


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


_p32, _p64, _pf = C.POINTER(C.c_int32), C.POINTER(C.c_int64), C.POINTER(C.c_float)


class _View(C.Structure):
    """vbsr_host_matrix_view (include/vbsr_b200.h): the HostMatrix fields as pointers + lengths."""
    _fields_ = [("block_rows", C.c_int32), ("block_cols", C.c_int32),
                ("row_ptr", _p32), ("row_ptr_len", C.c_size_t),
                ("block_col", _p32), ("block_col_len", C.c_size_t),
                ("row_size", _p32), ("row_size_len", C.c_size_t),
                ("col_size", _p32), ("col_size_len", C.c_size_t),
                ("row_scalar_off", _p64), ("row_scalar_off_len", C.c_size_t),
                ("col_scalar_off", _p64), ("col_scalar_off_len", C.c_size_t),
                ("value_off", _p64), ("value_off_len", C.c_size_t),
                ("values", _pf), ("values_len", C.c_size_t)]


_F32 = ("row_ptr", "block_col", "row_size", "col_size")
_F64 = ("row_scalar_off", "col_scalar_off", "value_off")


def _view(host):
    """View struct over `host`'s arrays; returns (view, arrays kept alive)."""
    keep = {}
    for f in _F32:
        keep[f] = np.ascontiguousarray(getattr(host, f), dtype=np.int32)
    for f in _F64:
        keep[f] = np.ascontiguousarray(getattr(host, f), dtype=np.int64)
    keep["values"] = np.ascontiguousarray(host.values, dtype=np.float32)
    v = _View()
    v.block_rows = int(host.block_rows)
    v.block_cols = int(host.block_cols)
    for f in _F32:
        setattr(v, f, keep[f].ctypes.data_as(_p32))
        setattr(v, f + "_len", keep[f].size)
    for f in _F64:
        setattr(v, f, keep[f].ctypes.data_as(_p64))
        setattr(v, f + "_len", keep[f].size)
    v.values = keep["values"].ctypes.data_as(_pf) if keep["values"].size else None
    v.values_len = keep["values"].size
    return v, keep


STREAM_VALUES = 0xA11CE
STREAM_DENSE = 0xB0B


def fill_uniform(seed: int, stream: int, first: int, count: int, threads: int = 0):
    """The benchmark inputs' counter-based U[-1,1) values first .. first+count-1 (workload.cpp)."""
    out = np.empty(int(count), dtype=np.float32)
    if count:
        _olib.oracle_fill_uniform(seed, stream, first, count, out.ctypes.data, _threads(threads))
    return out


class WorkloadMatrix:
    """A benchmark-specification matrix built by the oracle library alone (no engine): the block
    structure of oracle_spec_structure, values from fill_uniform(seed, STREAM_VALUES) at their
    packed positions (only when asked for, or per row slice)."""

    def __init__(self, rows, cols, degree, distribution, local, seed, with_values=False):
        rs = np.empty(rows, dtype=np.int32)
        cs = np.empty(cols, dtype=np.int32)
        bc = np.empty(rows * degree, dtype=np.int32)
        if _olib.oracle_spec_structure(rows, cols, degree, int(distribution), int(bool(local)),
                                       seed, rs.ctypes.data, cs.ctypes.data, bc.ctypes.data):
            raise ValueError("invalid generator dimensions")
        self.block_rows, self.block_cols, self.seed = rows, cols, seed
        self.row_size, self.col_size, self.block_col = rs, cs, bc
        self.row_ptr = (np.arange(rows + 1, dtype=np.int64) * degree).astype(np.int32)
        self.row_scalar_off = np.concatenate([[0], np.cumsum(rs, dtype=np.int64)])
        self.col_scalar_off = np.concatenate([[0], np.cumsum(cs, dtype=np.int64)])
        sizes = np.repeat(rs.astype(np.int64), degree) * cs[bc].astype(np.int64)
        self.value_off = np.concatenate([[0], np.cumsum(sizes)])
        self.values = (fill_uniform(seed, STREAM_VALUES, 0, int(self.value_off[-1]))
                       if with_values else np.zeros(0, dtype=np.float32))

    @property
    def nnzb(self) -> int:
        return int(self.block_col.size)

    def scalar_rows(self) -> int:
        return int(self.row_scalar_off[-1])

    def scalar_cols(self) -> int:
        return int(self.col_scalar_off[-1])

    def row_slice(self, r0: int, r1: int) -> "WorkloadMatrix":
        """Block rows [r0, r1) with their values (full column structure)."""
        s = object.__new__(WorkloadMatrix)
        b0, b1 = int(self.row_ptr[r0]), int(self.row_ptr[r1])
        v0, v1 = int(self.value_off[b0]), int(self.value_off[b1])
        s.block_rows, s.block_cols, s.seed = r1 - r0, self.block_cols, self.seed
        s.row_ptr = self.row_ptr[r0:r1 + 1] - b0
        s.block_col = self.block_col[b0:b1].copy()
        s.row_size = self.row_size[r0:r1].copy()
        s.col_size = self.col_size
        s.row_scalar_off = self.row_scalar_off[r0:r1 + 1] - self.row_scalar_off[r0]
        s.col_scalar_off = self.col_scalar_off
        s.value_off = self.value_off[b0:b1 + 1] - v0
        s.values = (self.values[v0:v1].copy() if self.values.size
                    else fill_uniform(self.seed, STREAM_VALUES, v0, v1 - v0))
        return s

    def flops(self, rhs: int, r0: int = 0, r1: int | None = None) -> float:
        r1 = self.block_rows if r1 is None else r1
        b0, b1 = int(self.row_ptr[r0]), int(self.row_ptr[r1])
        return 2.0 * float(self.value_off[b1] - self.value_off[b0]) * rhs


class RefTimer:
    """The reference's own cpu_reference on `host` (all rows) with B, prepared once (per-thread
    row-slice HostMatrix parts and the std::vector copy of B built here, outside any timing);
    run() executes only the cpu_reference calls and returns their wall time in seconds."""

    def __init__(self, host, B, rhs: int, threads: int = 0):
        self.threads = _threads(threads)
        self.rhs = rhs
        self._B = _f32(B)
        args, self._keep = _ref_view_args(host)
        self._h = _rlib.ref_prepare(*args, self._B.ctypes.data, rhs, 0, host.block_rows,
                                    self.threads)
        if not self._h:
            raise ValueError(_rlib.ref_last_error().decode())
        self.rows = int(host.row_scalar_off[host.block_rows] - host.row_scalar_off[0])

    def run(self, C_out=None) -> float:
        sec = C.c_double()
        rc = _rlib.ref_run(self._h, C_out.ctypes.data if C_out is not None else None,
                           C.byref(sec))
        if rc != 0:
            raise ValueError(_rlib.ref_last_error().decode())
        return sec.value

    def close(self):
        if self._h:
            _rlib.ref_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def host_threads() -> int:
    """Host threads this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _threads(t):
    return t if t and t > 0 else host_threads()


def spmm(host, B, rhs: int, r0: int = 0, r1: int | None = None, threads: int = 0,
         bound: bool = False):
    """Oracle C (and S if bound) for block rows [r0, r1), column-major flattened, ld = rows of the
    range. `host` is a varblockspmm_b200.HostMatrix in the reference layout."""
    r1 = host.block_rows if r1 is None else r1
    B = _f32(B)
    v, keep = _view(host)
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
    v, keep = _view(host)
    mr, ma, nb = C.c_double(), C.c_double(), C.c_int64()
    rc = _olib.vbsr_oracle_compare(C.addressof(v), B.ctypes.data, rhs, r0, r1, Ct.ctypes.data,
                                   _threads(threads), C.byref(mr), C.byref(ma), C.byref(nb))
    if rc != 0:
        raise ValueError("oracle rejected its arguments")
    return mr.value, ma.value, nb.value


# ---- the reference itself -------------------------------------------------------------------------

def _ref_view_args(host):
    v, keep = _view(host)  # normalised dtypes, kept alive by the returned tuple
    dims = np.array([host.block_rows, host.block_cols], dtype=np.int32)
    names = list(_F32) + list(_F64) + ["values"]
    lens = np.array([keep[n].size for n in names], dtype=np.int64)
    args = [dims.ctypes.data] + [keep[n].ctypes.data for n in names] + [lens.ctypes.data]
    return args, (dims, lens, v, keep)


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
