"""varblockspmm_b200 — Python binding of the B200-native VBSR SpMM engine.

Mirrors the host API of King-Clawthorne/VarBlockSpMM (include/varblockspmm/vbsr.hpp) over the
engine's C ABI (include/vbsr_b200.h, libvbsr_b200.so): HostMatrix, Matrix, Plan, PlanOptions,
Kernel, Distribution, GeneratorOptions, generate, launch_row_owned, launch_row_owned_scalar, and
the multi-GPU MultiPlan (no reference counterpart).
Errors follow the reference's exception types: malformed input raises InvalidArgument (a
ValueError, the analogue of std::invalid_argument), CUDA failures raise CudaError (a
RuntimeError, the analogue of std::runtime_error).

Device buffers (B, C) may be torch CUDA tensors (float32, contiguous) or raw device pointers
(int). Streams may be torch.cuda.Stream objects, raw cudaStream_t integers, or None (the legacy
default stream). There is no CPU execution path: if the compiled library is missing, importing
this package raises.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# VBSR_B200_LIB overrides the library path (for A/B comparisons of alternative builds).
LIB_PATH = os.environ.get("VBSR_B200_LIB") or os.path.join(_HERE, "libvbsr_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        "libvbsr_b200.so is not built; run `python varblockspmm_b200/build.py` "
        "(or __graft_entry__.build()) first")
_lib = C.CDLL(LIB_PATH)

# ---- status and errors -------------------------------------------------------------------------

OK, INVALID_ARGUMENT, CUDA_ERROR, TIMEOUT, BOUNDS_VIOLATION, OUT_OF_MEMORY = range(6)


class VbsrError(RuntimeError):
    status = -1


class InvalidArgument(ValueError):
    """std::invalid_argument of the reference."""
    status = INVALID_ARGUMENT


class CudaError(VbsrError):
    status = CUDA_ERROR


class TimeoutError_(VbsrError):
    status = TIMEOUT


class BoundsViolation(VbsrError):
    status = BOUNDS_VIOLATION


_lib.vbsr_get_last_error.restype = C.c_char_p


def last_error() -> str:
    return _lib.vbsr_get_last_error().decode()


def _check(status: int):
    if status == OK:
        return
    msg = last_error()
    if status == INVALID_ARGUMENT:
        raise InvalidArgument(msg)
    if status == TIMEOUT:
        raise TimeoutError_(msg)
    if status == BOUNDS_VIOLATION:
        raise BoundsViolation(msg)
    if status == OUT_OF_MEMORY:
        raise MemoryError(msg)
    raise CudaError(msg)


# ---- C structs ---------------------------------------------------------------------------------

_p32 = C.POINTER(C.c_int32)
_p64 = C.POINTER(C.c_int64)
_pf = C.POINTER(C.c_float)


class HostView(C.Structure):
    _fields_ = [("block_rows", C.c_int32), ("block_cols", C.c_int32),
                ("row_ptr", _p32), ("row_ptr_len", C.c_size_t),
                ("block_col", _p32), ("block_col_len", C.c_size_t),
                ("row_size", _p32), ("row_size_len", C.c_size_t),
                ("col_size", _p32), ("col_size_len", C.c_size_t),
                ("row_scalar_off", _p64), ("row_scalar_off_len", C.c_size_t),
                ("col_scalar_off", _p64), ("col_scalar_off_len", C.c_size_t),
                ("value_off", _p64), ("value_off_len", C.c_size_t),
                ("values", _pf), ("values_len", C.c_size_t)]


class DeviceMatrix(C.Structure):
    """Non-owning device view (DeviceMatrix, reference vbsr.hpp:32-38)."""
    _fields_ = [("block_rows", C.c_int32), ("block_cols", C.c_int32), ("nnzb", C.c_int32),
                ("scalar_rows", C.c_int64), ("scalar_cols", C.c_int64),
                ("row_ptr", C.c_void_p), ("block_col", C.c_void_p), ("row_size", C.c_void_p),
                ("col_size", C.c_void_p), ("row_scalar_off", C.c_void_p),
                ("col_scalar_off", C.c_void_p), ("value_off", C.c_void_p), ("values", C.c_void_p)]


class MatrixInfo(C.Structure):
    _fields_ = [("block_rows", C.c_int32), ("block_cols", C.c_int32), ("nnzb", C.c_int64),
                ("scalar_rows", C.c_int64), ("scalar_cols", C.c_int64),
                ("value_count", C.c_int64), ("device_bytes", C.c_int64), ("device", C.c_int32),
                ("row_begin", C.c_int32), ("row_end", C.c_int32)]


class GenOpts(C.Structure):
    _fields_ = [("block_rows", C.c_int32), ("block_cols", C.c_int32), ("degree", C.c_int32),
                ("rhs_width", C.c_int32), ("distribution", C.c_int32),
                ("local_columns", C.c_int32), ("seed", C.c_uint64), ("profile", C.c_int32),
                ("with_values", C.c_int32), ("threads", C.c_int32)]


_vp = C.c_void_p
class MultiShard(C.Structure):
    _fields_ = [("device", C.c_int32), ("row_begin", C.c_int32), ("row_end", C.c_int32),
                ("c_row0", C.c_int64), ("c_rows", C.c_int64), ("B", _vp), ("C", _vp),
                ("plan", _vp), ("stream", _vp)]


_sig = {
    "vbsr_host_validate": [C.POINTER(HostView)],
    "vbsr_matrix_create": [C.POINTER(HostView), C.c_int, C.POINTER(_vp)],
    "vbsr_matrix_create_rows": [C.POINTER(HostView), C.c_int32, C.c_int32, C.c_int, C.POINTER(_vp)],
    "vbsr_matrix_create_rows_generated": [C.POINTER(HostView), C.c_int32, C.c_int32, C.c_uint64,
                                          C.c_int, C.POINTER(_vp)],
    "vbsr_matrix_destroy": [_vp],
    "vbsr_matrix_info_get": [_vp, C.POINTER(MatrixInfo)],
    "vbsr_matrix_device_view": [_vp, C.POINTER(DeviceMatrix)],
    "vbsr_plan_create": [_vp, C.c_int, C.c_int, C.POINTER(_vp)],
    "vbsr_plan_create_ex": [_vp, C.c_int, C.c_int, C.c_uint32, C.POINTER(_vp)],
    "vbsr_plan_destroy": [_vp],
    "vbsr_plan_execute": [_vp, _vp, _vp, _vp],
    "vbsr_plan_launch_count": [_vp, C.POINTER(C.c_int)],
    "vbsr_plan_execute_noalloc": [_vp, _vp, _vp, _vp, C.POINTER(C.c_uint64), C.c_int],
    "vbsr_plan_check_status": [_vp, _vp],
    "vbsr_plan_describe": [_vp, C.c_char_p, C.c_size_t],
    "vbsr_plan_set_debug": [_vp, C.c_int, C.c_int64],
    "vbsr_plan_cta_timing": [_vp, C.c_int, C.POINTER(C.c_uint64), C.c_int, _vp],
    "vbsr_plan_num_tasks": [_vp, C.POINTER(C.c_int)],
    "vbsr_plan_work_info": [_vp, C.c_void_p],
    "vbsr_plan_task_stats": [_vp, C.POINTER(C.c_int32), C.POINTER(C.c_double), C.c_int],
    "vbsr_launch_row_owned": [C.POINTER(DeviceMatrix), _vp, C.c_int, C.c_int, _vp, _vp, C.c_int, _vp],
    "vbsr_launch_row_owned_scalar": [C.POINTER(DeviceMatrix), _vp, _vp, C.c_int, _vp],
    "vbsr_generate": [C.POINTER(GenOpts), C.POINTER(_vp)],
    "vbsr_host_matrix_view_get": [_vp, C.POINTER(HostView)],
    "vbsr_host_matrix_free": [_vp],
    "vbsr_fill_uniform": [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, _pf, C.c_int],
    "vbsr_fill_uniform_device": [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, _vp, _vp],
    "vbsr_fill_mt19937": [C.c_uint32, C.c_uint64, _pf],
    "vbsr_host_matrix_from_csr": [C.c_int64, C.c_int64, _vp, _vp, _vp, C.c_int32, _vp, C.c_int32,
                                  _vp, C.POINTER(_vp)],
    "vbsr_host_matrix_save": [C.POINTER(HostView), C.c_char_p],
    "vbsr_host_matrix_load": [C.c_char_p, C.POINTER(_vp)],
    "vbsr_partition_rows": [C.POINTER(HostView), C.c_int, C.c_int, _p32],
    "vbsr_compulsory_bytes": [C.POINTER(HostView), C.c_int32, C.c_int32, C.c_int,
                              C.POINTER(C.c_double), C.POINTER(C.c_double)],
    "vbsr_multi_plan_create": [C.POINTER(HostView), C.c_int, _p32, C.c_int, C.c_int, C.c_uint32,
                               C.POINTER(_vp)],
    "vbsr_multi_plan_create_generated": [C.POINTER(HostView), C.c_int, _p32, C.c_int, C.c_int,
                                         C.c_uint32, C.c_uint64, C.POINTER(_vp)],
    "vbsr_multi_plan_destroy": [_vp],
    "vbsr_multi_plan_count": [_vp, C.POINTER(C.c_int)],
    "vbsr_multi_plan_shard": [_vp, C.c_int, C.POINTER(MultiShard)],
    "vbsr_multi_plan_replicate_B": [_vp, _vp, C.c_int],
    "vbsr_multi_plan_execute": [_vp],
    "vbsr_multi_plan_synchronize": [_vp, C.POINTER(C.c_float)],
    "vbsr_multi_plan_gather_C": [_vp, _vp, C.c_int],
}
for _name, _args in _sig.items():
    _f = getattr(_lib, _name)
    _f.argtypes = _args
    _f.restype = C.c_int

STREAM_VALUES = 0xA11CE
STREAM_DENSE = 0xB0B
PLAN_BOUNDS_CHECK = 1
PLAN_NO_SPLIT = 2
PLAN_STACKS_RAW = 8        # RHS 64: force raw-B operand stacks (same results)
PLAN_STACKS_PRESPLIT = 16  # RHS 64: force pre-split operand stacks (same results)
PLAN_B_DIRECT = 32         # RHS 64: raw-B stack rows read straight from B, no pre-pass
PLAN_CUDA_CORE_ROWS = 64  # RHS <= 32: short block rows on the CUDA cores in the pre-pass launch
PLAN_FUSED_PREPASS = 128  # B stacks formed by the SpMM's CTAs (one launch; slower, off by default)
PLAN_DIAG_SKIP_COPIES = 1 << 8  # diagnostics only: C is wrong
PLAN_DIAG_SKIP_MATH = 1 << 9    # diagnostics only: C is wrong
PLAN_DIAG_SKIP_PREPASS = 1 << 10  # timing only: reuses the previous execute's B stacks


class Distribution(enum.IntEnum):
    Uniform = 0
    LowVariance = 1
    HighVariance = 2
    Bimodal = 3


class Profile(enum.IntEnum):
    Reference = 0
    Spec = 1


class Kernel(enum.IntEnum):
    Auto = 0
    RowOwned = 1
    SplitRow = 2


# ---- host matrix -------------------------------------------------------------------------------

_FIELDS32 = ("row_ptr", "block_col", "row_size", "col_size")
_FIELDS64 = ("row_scalar_off", "col_scalar_off", "value_off")


def _ptr(a, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


class HostMatrix:
    """Host VBSR matrix (HostMatrix, reference vbsr.hpp:16-29), arrays held as numpy arrays."""

    def __init__(self, block_rows=0, block_cols=0, row_ptr=(), block_col=(), row_size=(),
                 col_size=(), row_scalar_off=(), col_scalar_off=(), value_off=(), values=()):
        self.block_rows = int(block_rows)
        self.block_cols = int(block_cols)
        self.row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int32)
        self.block_col = np.ascontiguousarray(block_col, dtype=np.int32)
        self.row_size = np.ascontiguousarray(row_size, dtype=np.int32)
        self.col_size = np.ascontiguousarray(col_size, dtype=np.int32)
        self.row_scalar_off = np.ascontiguousarray(row_scalar_off, dtype=np.int64)
        self.col_scalar_off = np.ascontiguousarray(col_scalar_off, dtype=np.int64)
        self.value_off = np.ascontiguousarray(value_off, dtype=np.int64)
        self.values = np.ascontiguousarray(values, dtype=np.float32)

    def scalar_rows(self) -> int:
        return int(self.row_scalar_off[-1]) if len(self.row_scalar_off) else 0

    def scalar_cols(self) -> int:
        return int(self.col_scalar_off[-1]) if len(self.col_scalar_off) else 0

    @property
    def nnzb(self) -> int:
        return len(self.block_col)

    def view(self) -> HostView:
        for f in _FIELDS32:
            setattr(self, f, np.ascontiguousarray(getattr(self, f), dtype=np.int32))
        for f in _FIELDS64:
            setattr(self, f, np.ascontiguousarray(getattr(self, f), dtype=np.int64))
        self.values = np.ascontiguousarray(self.values, dtype=np.float32)
        v = HostView()
        v.block_rows = self.block_rows
        v.block_cols = self.block_cols
        for f in _FIELDS32:
            a = getattr(self, f)
            setattr(v, f, _ptr(a, C.c_int32))
            setattr(v, f + "_len", a.size)
        for f in _FIELDS64:
            a = getattr(self, f)
            setattr(v, f, _ptr(a, C.c_int64))
            setattr(v, f + "_len", a.size)
        v.values = _ptr(self.values, C.c_float) if self.values.size else None
        v.values_len = self.values.size
        return v

    def save(self, path: str) -> None:
        """Writes the matrix to a binary VBSR file (see vbsr_host_matrix_save)."""
        v = self.view()
        _check(_lib.vbsr_host_matrix_save(C.byref(v), os.fsencode(path)))

    def validate(self):
        """HostMatrix::validate (reference src/format/vbsr.cpp:29-82)."""
        v = self.view()
        _check(_lib.vbsr_host_validate(C.byref(v)))

    def row_slice(self, r0: int, r1: int, values_seed: int | None = None) -> "HostMatrix":
        """Block rows [r0, r1) as a standalone matrix (full column structure). Values come from
        this matrix, or, for a structure-only spec-profile matrix, are regenerated from the
        counter-based stream of `values_seed` at their packed positions in the full matrix."""
        b0, b1 = int(self.row_ptr[r0]), int(self.row_ptr[r1])
        v0, v1 = int(self.value_off[b0]), int(self.value_off[b1])
        if self.values.size:
            vals = self.values[v0:v1].copy()
        elif values_seed is not None:
            vals = fill_uniform(values_seed, STREAM_VALUES, v0, v1 - v0)
        else:
            raise InvalidArgument("matrix has no values and no values_seed was given")
        return HostMatrix(r1 - r0, self.block_cols, self.row_ptr[r0:r1 + 1] - b0,
                          self.block_col[b0:b1].copy(), self.row_size[r0:r1].copy(),
                          self.col_size.copy(),
                          self.row_scalar_off[r0:r1 + 1] - self.row_scalar_off[r0],
                          self.col_scalar_off.copy(), self.value_off[b0:b1 + 1] - v0, vals)

    def copy(self) -> "HostMatrix":
        return HostMatrix(self.block_rows, self.block_cols, self.row_ptr.copy(),
                          self.block_col.copy(), self.row_size.copy(), self.col_size.copy(),
                          self.row_scalar_off.copy(), self.col_scalar_off.copy(),
                          self.value_off.copy(), self.values.copy())


@dataclass
class GeneratorOptions:
    """GeneratorOptions (reference vbsr.hpp:70-76) plus `profile`."""
    block_rows: int = 1024
    block_cols: int = 1024
    degree: int = 4
    rhs_width: int = 32
    distribution: Distribution = Distribution.HighVariance
    local_columns: bool = True
    seed: int = 1
    profile: Profile = Profile.Reference


def generate(opts: GeneratorOptions, with_values: bool = True, threads: int = 0) -> HostMatrix:
    """generate() (reference src/format/generator.cpp:7-88); see vbsr_b200.h for the profiles."""
    o = GenOpts(opts.block_rows, opts.block_cols, opts.degree, opts.rhs_width,
                int(opts.distribution), int(bool(opts.local_columns)), int(opts.seed),
                int(opts.profile), int(bool(with_values)), int(threads))
    h = _vp()
    _check(_lib.vbsr_generate(C.byref(o), C.byref(h)))
    return _take_host(h)


def _take_host(h) -> "HostMatrix":
    """Copies a library-owned host matrix into a HostMatrix and frees it."""
    try:
        v = HostView()
        _check(_lib.vbsr_host_matrix_view_get(h, C.byref(v)))

        def arr(p, n, dt):
            if n == 0:
                return np.zeros(0, dtype=dt)
            return np.ctypeslib.as_array(p, shape=(n,)).astype(dt, copy=True)

        m = HostMatrix(v.block_rows, v.block_cols,
                       arr(v.row_ptr, v.row_ptr_len, np.int32),
                       arr(v.block_col, v.block_col_len, np.int32),
                       arr(v.row_size, v.row_size_len, np.int32),
                       arr(v.col_size, v.col_size_len, np.int32),
                       arr(v.row_scalar_off, v.row_scalar_off_len, np.int64),
                       arr(v.col_scalar_off, v.col_scalar_off_len, np.int64),
                       arr(v.value_off, v.value_off_len, np.int64),
                       arr(v.values, v.values_len, np.float32))
    finally:
        _lib.vbsr_host_matrix_free(h)
    return m


def load_matrix(path: str) -> HostMatrix:
    """Reads a binary VBSR file written by HostMatrix.save (validated on load)."""
    h = _vp()
    _check(_lib.vbsr_host_matrix_load(os.fsencode(path), C.byref(h)))
    return _take_host(h)


def block_sizes(n: int, size: int = 32) -> np.ndarray:
    """A block partition of n scalars (n a multiple of 8): blocks of `size` (a multiple of 8 in
    [8, 64]) and a last block of the remainder."""
    if n <= 0 or n % 8 or size % 8 or not 8 <= size <= 64:
        raise InvalidArgument("n must be a positive multiple of 8, size a multiple of 8 in [8, 64]")
    sizes = [size] * (n // size)
    if n % size:
        sizes.append(n % size)
    return np.asarray(sizes, dtype=np.int32)


def from_csr(shape, indptr, indices, data, row_sizes, col_sizes) -> HostMatrix:
    """A scalar CSR matrix as a VBSR host matrix for the given block partition (every block that
    holds a nonzero becomes a dense block; see vbsr_host_matrix_from_csr)."""
    rows, cols = int(shape[0]), int(shape[1])
    ip = np.ascontiguousarray(indptr, dtype=np.int64)
    ix = np.ascontiguousarray(indices, dtype=np.int64)
    dv = np.ascontiguousarray(data, dtype=np.float32)
    rs = np.ascontiguousarray(row_sizes, dtype=np.int32)
    cs = np.ascontiguousarray(col_sizes, dtype=np.int32)
    h = _vp()
    _check(_lib.vbsr_host_matrix_from_csr(rows, cols, ip.ctypes.data, ix.ctypes.data,
                                          dv.ctypes.data, rs.size, rs.ctypes.data, cs.size,
                                          cs.ctypes.data, C.byref(h)))
    return _take_host(h)


def load_matrix_market(path: str, row_block: int = 32, col_block: int = 32):
    """Reads a Matrix Market file (scipy.io.mmread) into a VBSR host matrix: the scalar dimensions
    are padded with zero rows / columns up to multiples of 8, then cut into blocks of row_block x
    col_block (a smaller last block). Returns (HostMatrix, (rows, cols) of the file)."""
    import scipy.io
    import scipy.sparse
    a = scipy.sparse.csr_matrix(scipy.io.mmread(path), dtype=np.float32)
    a.sum_duplicates()
    rows, cols = a.shape
    pr, pc = -(-rows // 8) * 8, -(-cols // 8) * 8
    indptr = np.concatenate([a.indptr, np.full(pr - rows, a.indptr[-1], dtype=a.indptr.dtype)])
    m = from_csr((pr, pc), indptr, a.indices, a.data, block_sizes(pr, row_block),
                 block_sizes(pc, col_block))
    return m, (rows, cols)


def fill_uniform(seed: int, stream: int, first: int, count: int, threads: int = 0) -> np.ndarray:
    """Counter-based U[-1,1) values: out[i] = u(seed, stream, first + i)."""
    out = np.empty(count, dtype=np.float32)
    _check(_lib.vbsr_fill_uniform(seed, stream, first, count, _ptr(out, C.c_float), threads))
    return out


def fill_mt19937(seed: int, count: int) -> np.ndarray:
    """std::mt19937(seed) U[-1,1] floats, the reference tests' dense input (test_main.cpp:42-51)."""
    out = np.empty(count, dtype=np.float32)
    _check(_lib.vbsr_fill_mt19937(seed, count, _ptr(out, C.c_float)))
    return out


def partition_rows(host: HostMatrix, parts: int, rhs: int) -> np.ndarray:
    """Balanced contiguous block-row ranges for a multi-GPU split (bounds[0..parts])."""
    v = host.view()
    b = np.zeros(parts + 1, dtype=np.int32)
    _check(_lib.vbsr_partition_rows(C.byref(v), parts, rhs, _ptr(b, C.c_int32)))
    return b


def compulsory_bytes(host: HostMatrix, rhs: int, r0: int = 0, r1: int | None = None):
    """(bytes, flops) of the roofline byte model for block rows [r0, r1)."""
    v = host.view()
    r1 = host.block_rows if r1 is None else r1
    by, fl = C.c_double(), C.c_double()
    _check(_lib.vbsr_compulsory_bytes(C.byref(v), r0, r1, rhs, C.byref(by), C.byref(fl)))
    return by.value, fl.value


# ---- device objects ----------------------------------------------------------------------------

def _dev_ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_cuda:
            raise InvalidArgument("expected a CUDA tensor")
        if x.dtype.__repr__() != "torch.float32":
            raise InvalidArgument("expected a float32 tensor")
        if not x.is_contiguous():
            raise InvalidArgument("expected a contiguous tensor")
        return x.data_ptr()
    raise InvalidArgument("expected a device pointer or CUDA tensor")


def _stream_ptr(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    if hasattr(s, "cuda_stream"):
        return s.cuda_stream
    raise InvalidArgument("expected a CUDA stream")


class Matrix:
    """Owning device matrix (Matrix, reference vbsr.hpp:41-64).

    Matrix(host) copies all of `host` to the current device. Matrix(host, rows=(r0, r1)) holds
    block rows [r0, r1) only (a multi-GPU shard). generated_seed=s builds the values on the device
    with the counter-based generator instead of copying host values (host.values may be empty).
    """

    def __init__(self, host: HostMatrix, device: int = -1, rows=None, generated_seed=None):
        self._h = _vp()
        v = host.view()
        r0, r1 = (0, host.block_rows) if rows is None else rows
        if generated_seed is not None:
            _check(_lib.vbsr_matrix_create_rows_generated(C.byref(v), r0, r1, generated_seed,
                                                          device, C.byref(self._h)))
        elif rows is None:
            _check(_lib.vbsr_matrix_create(C.byref(v), device, C.byref(self._h)))
        else:
            _check(_lib.vbsr_matrix_create_rows(C.byref(v), r0, r1, device, C.byref(self._h)))
        inf = self.info()
        self._rows, self._cols = inf.scalar_rows, inf.scalar_cols

    def info(self) -> MatrixInfo:
        inf = MatrixInfo()
        _check(_lib.vbsr_matrix_info_get(self._h, C.byref(inf)))
        return inf

    def scalar_rows(self) -> int:
        return self._rows

    def scalar_cols(self) -> int:
        return self._cols

    def device_view(self) -> DeviceMatrix:
        d = DeviceMatrix()
        _check(_lib.vbsr_matrix_device_view(self._h, C.byref(d)))
        return d

    def close(self):
        if self._h:
            _lib.vbsr_matrix_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class PlanOptions:
    """PlanOptions (reference vbsr.hpp:94-97)."""
    rhs_width: int = 32
    kernel: Kernel = Kernel.Auto


class Plan:
    """Execution plan (Plan, reference vbsr.hpp:104-119). The Matrix must outlive the plan."""

    def __init__(self, matrix: Matrix, options: PlanOptions | int = PlanOptions(), flags: int = 0):
        if isinstance(options, int):
            options = PlanOptions(options)
        self.options = options
        self._matrix = matrix  # keep the matrix alive
        self._h = _vp()
        _check(_lib.vbsr_plan_create_ex(matrix._h, int(options.rhs_width), int(options.kernel),
                                        flags, C.byref(self._h)))

    def execute(self, B, C_out, stream=None):
        """Enqueues C = A * B on `stream` (asynchronous, allocation-free)."""
        _check(_lib.vbsr_plan_execute(self._h, _dev_ptr(B), _dev_ptr(C_out), _stream_ptr(stream)))

    def execute_noalloc(self, B, C_out, stream=None, report: bool = False):
        """Like execute, but allocates nothing: status words and CTA timestamps live in a fixed
        array inside the library (see vbsr_plan_execute_noalloc). With report=False the call is
        asynchronous and reports no kernel-side error. With report=True, waits for the launch,
        raises on a recorded timeout or bounds violation, and returns the (start, end) timestamps
        per CTA (zeros when B or C is not 16-byte aligned: that path records none)."""
        if not report:
            _check(_lib.vbsr_plan_execute_noalloc(self._h, _dev_ptr(B), _dev_ptr(C_out),
                                                  _stream_ptr(stream), None, 0))
            return None
        n = self.num_tasks()
        out = np.zeros(2 * n, dtype=np.uint64)
        _check(_lib.vbsr_plan_execute_noalloc(self._h, _dev_ptr(B), _dev_ptr(C_out),
                                              _stream_ptr(stream),
                                              out.ctypes.data_as(C.POINTER(C.c_uint64)), 2 * n))
        return out.reshape(n, 2)

    def launch_count(self) -> int:
        n = C.c_int()
        _check(_lib.vbsr_plan_launch_count(self._h, C.byref(n)))
        return n.value

    def check_status(self, stream=None):
        """Synchronises `stream` and raises if a kernel recorded a timeout or bounds violation."""
        _check(_lib.vbsr_plan_check_status(self._h, _stream_ptr(stream)))

    def describe(self) -> str:
        buf = C.create_string_buffer(1024)
        _check(_lib.vbsr_plan_describe(self._h, buf, 1024))
        return buf.value.decode()

    def set_debug(self, drop_stage: int = -1, wait_limit_cycles: int = 0):
        _check(_lib.vbsr_plan_set_debug(self._h, drop_stage, wait_limit_cycles))

    def work_info(self) -> dict:
        """How the plan divides the work: tensor-core items/rows (split_rows cut into row parts)
        and CUDA-core rows, with their A value counts."""
        w = (C.c_int64 * 7)()
        _check(_lib.vbsr_plan_work_info(self._h, C.addressof(w)))
        return dict(zip(("tc_items", "tc_rows", "split_rows", "tc_values", "cc_rows",
                         "cc_values", "cc_scalar_rows"), list(w)))

    def num_tasks(self) -> int:
        n = C.c_int()
        _check(_lib.vbsr_plan_num_tasks(self._h, C.byref(n)))
        return n.value

    def task_stats(self):
        """(team_warps, model_cost) per task of the schedule."""
        n = self.num_tasks()
        tw = np.zeros(n, dtype=np.int32)
        mc = np.zeros(n, dtype=np.float64)
        _check(_lib.vbsr_plan_task_stats(self._h, tw.ctypes.data_as(C.POINTER(C.c_int32)),
                                         mc.ctypes.data_as(C.POINTER(C.c_double)), n))
        return tw, mc

    def enable_cta_timing(self, enable: bool = True):
        _check(_lib.vbsr_plan_cta_timing(self._h, int(enable), None, 0, None))

    def cta_timing(self, stream=None) -> np.ndarray:
        """(start, end) global-timer ns per CTA of the last timed execution, shape (tasks, 2)."""
        n = self.num_tasks()
        out = np.zeros(2 * n, dtype=np.uint64)
        _check(_lib.vbsr_plan_cta_timing(self._h, 1, out.ctypes.data_as(C.POINTER(C.c_uint64)),
                                         2 * n, _stream_ptr(stream)))
        return out.reshape(n, 2)

    def close(self):
        if self._h:
            _lib.vbsr_plan_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MultiPlan:
    """Multi-GPU plan: the block rows of `host` split into len(devices) balanced shards, one per
    entry of `devices` (entries may repeat), each with its own plan, B replica, C block and
    stream (vbsr_multi_plan_*). No reference counterpart: the reference is single-GPU.

        mp = MultiPlan(host, [0, 1, 2, 3], PlanOptions(64))
        mp.replicate_B(B)          # host numpy array or CUDA tensor; peer-to-peer doubling tree
        mp.execute()               # every shard on its own stream
        ms = mp.synchronize()      # max over shards of the device time of that execute
        C = mp.gather_C()          # M x rhs column-major result (host numpy array)
    """

    def __init__(self, host: HostMatrix, devices, options: PlanOptions | int = PlanOptions(),
                 flags: int = 0, generated_seed=None):
        if isinstance(options, int):
            options = PlanOptions(options)
        self.options = options
        self.rhs = int(options.rhs_width)
        devs = np.ascontiguousarray(np.asarray(devices, dtype=np.int32))
        self._h = _vp()
        v = host.view()
        if generated_seed is None:
            _check(_lib.vbsr_multi_plan_create(C.byref(v), len(devs), _ptr(devs, C.c_int32),
                                               self.rhs, int(options.kernel), flags,
                                               C.byref(self._h)))
        else:
            _check(_lib.vbsr_multi_plan_create_generated(C.byref(v), len(devs),
                                                         _ptr(devs, C.c_int32), self.rhs,
                                                         int(options.kernel), flags,
                                                         generated_seed, C.byref(self._h)))
        self.M = int(host.scalar_rows())
        self.K = int(host.scalar_cols())

    def __len__(self) -> int:
        n = C.c_int()
        _check(_lib.vbsr_multi_plan_count(self._h, C.byref(n)))
        return n.value

    def shard(self, rank: int) -> MultiShard:
        sh = MultiShard()
        _check(_lib.vbsr_multi_plan_shard(self._h, rank, C.byref(sh)))
        return sh

    def replicate_B(self, B, src_device: int | None = None):
        """Copies B (K x rhs, column-major) into every shard's replica. B is a host numpy float32
        array, or a CUDA tensor / device pointer on src_device."""
        if isinstance(B, np.ndarray):
            if B.dtype != np.float32 or B.size != self.K * self.rhs:
                raise InvalidArgument("B must be float32 with K * rhs elements")
            Bc = np.ascontiguousarray(B)
            _check(_lib.vbsr_multi_plan_replicate_B(self._h, Bc.ctypes.data, -1))
            self.synchronize()  # the host buffer may be released after the call
            return
        dev = src_device if src_device is not None else B.device.index
        if hasattr(B, "device"):
            import torch
            torch.cuda.synchronize(B.device)  # the copies run on the shards' streams
        _check(_lib.vbsr_multi_plan_replicate_B(self._h, _dev_ptr(B), int(dev)))

    def execute(self):
        _check(_lib.vbsr_multi_plan_execute(self._h))

    def synchronize(self) -> float:
        ms = C.c_float()
        _check(_lib.vbsr_multi_plan_synchronize(self._h, C.byref(ms)))
        return ms.value

    def gather_C(self, out=None, dst_device: int | None = None):
        """The M x rhs column-major result: into a new host array (default), a given host array,
        or a CUDA tensor on dst_device."""
        if out is None:
            out = np.empty(self.M * self.rhs, dtype=np.float32)
        if isinstance(out, np.ndarray):
            if out.dtype != np.float32 or out.size != self.M * self.rhs:
                raise InvalidArgument("out must be float32 with M * rhs elements")
            _check(_lib.vbsr_multi_plan_gather_C(self._h, out.ctypes.data, -1))
            return out
        dev = dst_device if dst_device is not None else out.device.index
        _check(_lib.vbsr_multi_plan_gather_C(self._h, _dev_ptr(out), int(dev)))
        return out

    def close(self):
        if self._h:
            _lib.vbsr_multi_plan_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def launch_row_owned(a: DeviceMatrix, B, C_out, rhs: int, stream=None):
    """launch_row_owned (reference row_owned.cu:397-423) on a device view."""
    _check(_lib.vbsr_launch_row_owned(C.byref(a), None, 0, 0, _dev_ptr(B), _dev_ptr(C_out), rhs,
                                      _stream_ptr(stream)))


def launch_row_owned_scalar(a: DeviceMatrix, B, C_out, rhs: int, stream=None):
    """launch_row_owned_scalar (reference row_owned.cu:376-395) on a device view."""
    _check(_lib.vbsr_launch_row_owned_scalar(C.byref(a), _dev_ptr(B), _dev_ptr(C_out), rhs,
                                             _stream_ptr(stream)))


def fill_uniform_device(seed: int, stream: int, first: int, count: int, out, cuda_stream=None):
    _check(_lib.vbsr_fill_uniform_device(seed, stream, first, count, _dev_ptr(out),
                                         _stream_ptr(cuda_stream)))


__all__ = [
    "HostMatrix", "DeviceMatrix", "Matrix", "Distribution", "Profile", "GeneratorOptions",
    "generate", "Kernel", "PlanOptions", "Plan", "launch_row_owned", "launch_row_owned_scalar",
    "partition_rows", "compulsory_bytes", "fill_uniform", "fill_uniform_device", "fill_mt19937",
    "from_csr", "load_matrix_market", "load_matrix", "block_sizes",
    "InvalidArgument", "CudaError", "VbsrError", "TimeoutError_", "BoundsViolation", "last_error",
    "STREAM_VALUES", "STREAM_DENSE", "PLAN_BOUNDS_CHECK", "PLAN_NO_SPLIT", "LIB_PATH",
]
