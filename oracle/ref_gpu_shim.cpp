// ref_gpu_shim.cpp — TEST INFRASTRUCTURE ONLY. A C-callable shim over the reference's own GPU
// path (King-Clawthorne/VarBlockSpMM: Matrix, Plan and the row-owned CUDA kernels of
// src/format/vbsr.cpp, src/plan/plan.cpp and src/kernels/row_owned.cu), compiled unchanged from
// the reference checkout by oracle/Makefile into oracle/_ref/libvbsr_ref_gpu.so. Tests use it to
// run the reference's kernels on the same GPU and inputs as the engine: their results against
// the oracle, and their device time next to the engine's.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "varblockspmm/vbsr.hpp"

namespace {
thread_local std::string g_err;

struct RefGpu {
  vbsr::Matrix matrix;
  vbsr::Plan plan;
  RefGpu(const vbsr::HostMatrix& h, int rhs)
      : matrix(h), plan(matrix, vbsr::PlanOptions{rhs, vbsr::Kernel::Auto}) {}
};
}  // namespace

extern "C" {

const char* ref_gpu_last_error() { return g_err.c_str(); }

// vbsr::Matrix (on the current device) and vbsr::Plan for `rhs` from the given arrays (the
// fields of HostMatrix; lens as in ref_shim.cpp). Returns NULL on failure.
void* ref_gpu_create(const int32_t* dims, const int32_t* row_ptr, const int32_t* block_col,
                     const int32_t* row_size, const int32_t* col_size, const int64_t* row_off,
                     const int64_t* col_off, const int64_t* value_off, const float* values,
                     const int64_t* lens, int rhs) {
  try {
    vbsr::HostMatrix m;
    m.block_rows = dims[0];
    m.block_cols = dims[1];
    m.row_ptr.assign(row_ptr, row_ptr + lens[0]);
    m.block_col.assign(block_col, block_col + lens[1]);
    m.row_size.assign(row_size, row_size + lens[2]);
    m.col_size.assign(col_size, col_size + lens[3]);
    m.row_scalar_off.assign(row_off, row_off + lens[4]);
    m.col_scalar_off.assign(col_off, col_off + lens[5]);
    m.value_off.assign(value_off, value_off + lens[6]);
    m.values.assign(values, values + lens[7]);
    return new RefGpu(m, rhs);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

// Plan::execute on `stream`; 0 on success.
int ref_gpu_execute(void* h, const float* B, float* C, void* stream) {
  try {
    static_cast<RefGpu*>(h)->plan.execute(B, C, static_cast<cudaStream_t>(stream));
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

int ref_gpu_launch_count(void* h) { return static_cast<RefGpu*>(h)->plan.launch_count(); }

void ref_gpu_destroy(void* h) { delete static_cast<RefGpu*>(h); }

}  // extern "C"
