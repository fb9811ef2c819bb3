// vbsr_comparators.cpp — the library comparator plans of the C++ drop-in API: ScalarCsrPlan
// (cuSPARSE SpMM on the matrix expanded to scalar CSR) and GroupedGemmPlan (grouped cuBLAS SGEMM
// over the blocks). They are the reference's baselines (include/varblockspmm/vbsr.hpp:121-155,
// src/baseline/cusparse_baseline.cu:139-181, src/baseline/slot_split.cu:59-145), kept so that code
// written against the reference's header finds them here, and so that the engine can be compared
// with the vendor libraries on the same B200. Same constructors, methods, error types and results;
// written for this library:
//   * ScalarCsrPlan uses 64-bit CSR indices when the expanded matrix has 2^31 or more nonzeros (the
//     reference's 32-bit indices overflow at that size), and builds the CSR arrays pre-sized;
//   * GroupedGemmPlan keeps the reference's slot order (slot k = the k-th block of every block row
//     that has one; slot 0 overwrites C, later slots accumulate), so its launch_count() is the
//     maximum block-row degree, as in the reference.
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusparse.h>

#include <algorithm>
#include <map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "varblockspmm/vbsr.hpp"

namespace vbsr {
namespace {

void cuda_ok(cudaError_t e) {
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}
void sparse_ok(cusparseStatus_t e) {
  if (e != CUSPARSE_STATUS_SUCCESS)
    throw std::runtime_error(std::string("cuSPARSE failure: ") + cusparseGetErrorString(e));
}
void blas_ok(cublasStatus_t e) {
  if (e != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("cuBLAS failure: " + std::to_string(int(e)));
}
void check_rhs(int rhs) {
  if (rhs != 8 && rhs != 16 && rhs != 32 && rhs != 64) throw std::invalid_argument("invalid rhs width");
}

template <class T>
T* to_device(const std::vector<T>& v) {
  T* d = nullptr;
  if (v.empty()) return d;
  cuda_ok(cudaMalloc(&d, v.size() * sizeof(T)));
  cuda_ok(cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}

}  // namespace

// ---- ScalarCsrPlan ---------------------------------------------------------------------------

struct ScalarCsrPlan::Impl {
  int rhs = 0;
  int64_t M = 0, K = 0, nnz = 0;
  void* row_off = nullptr;
  void* col_idx = nullptr;
  float* val = nullptr;
  void* work = nullptr;
  size_t work_bytes = 0;
  cusparseHandle_t h = nullptr;
  cusparseSpMatDescr_t A = nullptr;
  cusparseDnMatDescr_t Bd = nullptr, Cd = nullptr;
  ~Impl() {
    if (Bd) cusparseDestroyDnMat(Bd);
    if (Cd) cusparseDestroyDnMat(Cd);
    if (A) cusparseDestroySpMat(A);
    if (h) cusparseDestroy(h);
    cudaFree(work);
    cudaFree(row_off);
    cudaFree(col_idx);
    cudaFree(val);
  }
};

namespace {
// Scalar CSR of a VBSR matrix: row i of block row r holds, block after block, the block's row.
template <class I>
void expand_csr(const HostMatrix& m, std::vector<I>& offs, std::vector<I>& cols,
                std::vector<float>& vals) {
  const int64_t M = m.scalar_rows();
  offs.assign(size_t(M) + 1, I(0));
  int64_t nnz = 0;
  for (int r = 0; r < m.block_rows; ++r) {
    int64_t width = 0;
    for (int b = m.row_ptr[r]; b < m.row_ptr[r + 1]; ++b) width += m.col_size[m.block_col[b]];
    nnz += width * m.row_size[r];
  }
  cols.resize(size_t(nnz));
  vals.resize(size_t(nnz));
  int64_t at = 0;
  for (int r = 0; r < m.block_rows; ++r) {
    const int h = m.row_size[r];
    for (int i = 0; i < h; ++i) {
      offs[size_t(m.row_scalar_off[r] + i)] = I(at);
      for (int b = m.row_ptr[r]; b < m.row_ptr[r + 1]; ++b) {
        const int c = m.block_col[b];
        const int w = m.col_size[c];
        const float* blk = m.values.data() + m.value_off[b];
        for (int k = 0; k < w; ++k) {
          cols[size_t(at)] = I(m.col_scalar_off[c] + k);
          vals[size_t(at)] = blk[i + int64_t(k) * h];
          ++at;
        }
      }
    }
  }
  offs[size_t(M)] = I(at);
}
}  // namespace

ScalarCsrPlan::ScalarCsrPlan(const HostMatrix& m, int rhs) : impl_(new Impl) {
  m.validate();
  check_rhs(rhs);
  Impl& d = *impl_;
  d.rhs = rhs;
  d.M = m.scalar_rows();
  d.K = m.scalar_cols();
  std::vector<float> vals;
  const int64_t total = int64_t(m.values.size());  // one CSR nonzero per stored value
  const bool wide = total >= (int64_t(1) << 31) || d.K >= (int64_t(1) << 31);
  cusparseIndexType_t it;
  if (wide) {
    std::vector<int64_t> offs, cols;
    expand_csr(m, offs, cols, vals);
    d.row_off = to_device(offs);
    d.col_idx = to_device(cols);
    it = CUSPARSE_INDEX_64I;
  } else {
    std::vector<int32_t> offs, cols;
    expand_csr(m, offs, cols, vals);
    d.row_off = to_device(offs);
    d.col_idx = to_device(cols);
    it = CUSPARSE_INDEX_32I;
  }
  d.nnz = int64_t(vals.size());
  d.val = to_device(vals);
  sparse_ok(cusparseCreate(&d.h));
  sparse_ok(cusparseCreateCsr(&d.A, d.M, d.K, d.nnz, d.row_off, d.col_idx, d.val, it, it,
                              CUSPARSE_INDEX_BASE_ZERO, CUDA_R_32F));
}

ScalarCsrPlan::~ScalarCsrPlan() = default;

size_t ScalarCsrPlan::workspace_bytes() const { return impl_->work_bytes; }

void ScalarCsrPlan::execute(const float* B, float* C, cudaStream_t stream) {
  Impl& d = *impl_;
  const float one = 1.0f, zero = 0.0f;
  sparse_ok(cusparseSetStream(d.h, stream));
  if (d.Bd == nullptr) {  // first call: dense descriptors and the persistent workspace
    sparse_ok(cusparseCreateDnMat(&d.Bd, d.K, d.rhs, d.K, const_cast<float*>(B), CUDA_R_32F,
                                  CUSPARSE_ORDER_COL));
    sparse_ok(cusparseCreateDnMat(&d.Cd, d.M, d.rhs, d.M, C, CUDA_R_32F, CUSPARSE_ORDER_COL));
    sparse_ok(cusparseSpMM_bufferSize(d.h, CUSPARSE_OPERATION_NON_TRANSPOSE,
                                      CUSPARSE_OPERATION_NON_TRANSPOSE, &one, d.A, d.Bd, &zero,
                                      d.Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &d.work_bytes));
    if (d.work_bytes > 0) cuda_ok(cudaMalloc(&d.work, d.work_bytes));
  } else {
    sparse_ok(cusparseDnMatSetValues(d.Bd, const_cast<float*>(B)));
    sparse_ok(cusparseDnMatSetValues(d.Cd, C));
  }
  sparse_ok(cusparseSpMM(d.h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE,
                         &one, d.A, d.Bd, &zero, d.Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT,
                         d.work));
}

// ---- GroupedGemmPlan -------------------------------------------------------------------------

struct GroupedGemmPlan::Impl {
  struct Slot {
    // one GEMM group per (h, w) shape: C_i (h x rhs) += A_i (h x w) * B_i (w x rhs)
    std::vector<cublasOperation_t> op;
    std::vector<int> m, n, k, lda, ldb, ldc, count;
    std::vector<float> alpha, beta;
    std::vector<int64_t> b_off, c_off;  // per problem: B row offset, C row offset
    const float** dA = nullptr;
    const float** dB = nullptr;
    float** dC = nullptr;
    std::vector<const float*> hB;
    std::vector<float*> hC;
  };
  int rhs = 0;
  int64_t M = 0, K = 0;
  float* values = nullptr;
  cublasHandle_t h = nullptr;
  std::vector<Slot> slots;
  ~Impl() {
    for (Slot& s : slots) {
      cudaFree(s.dA);
      cudaFree(s.dB);
      cudaFree(s.dC);
    }
    if (h) cublasDestroy(h);
    cudaFree(values);
  }
};

GroupedGemmPlan::GroupedGemmPlan(const HostMatrix& m, int rhs) : impl_(new Impl) {
  m.validate();
  check_rhs(rhs);
  Impl& d = *impl_;
  d.rhs = rhs;
  d.M = m.scalar_rows();
  d.K = m.scalar_cols();
  d.values = to_device(m.values);
  blas_ok(cublasCreate(&d.h));
  int depth = 0;
  for (int r = 0; r < m.block_rows; ++r) depth = std::max(depth, m.row_ptr[r + 1] - m.row_ptr[r]);
  d.slots.resize(size_t(depth));
  for (int k = 0; k < depth; ++k) {
    std::map<std::pair<int, int>, std::vector<int>> by_shape;  // (h, w) -> block indices
    for (int r = 0; r < m.block_rows; ++r) {
      const int b = m.row_ptr[r] + k;
      if (b < m.row_ptr[r + 1]) by_shape[{m.row_size[r], m.col_size[m.block_col[b]]}].push_back(b);
    }
    Impl::Slot& s = d.slots[size_t(k)];
    std::vector<const float*> a_ptrs;
    // block -> its block row (row_ptr is monotone): found once per block below
    for (const auto& [shape, blocks] : by_shape) {
      s.op.push_back(CUBLAS_OP_N);
      s.m.push_back(shape.first);
      s.n.push_back(rhs);
      s.k.push_back(shape.second);
      s.lda.push_back(shape.first);
      s.ldb.push_back(int(d.K));
      s.ldc.push_back(int(d.M));
      s.alpha.push_back(1.0f);
      s.beta.push_back(k == 0 ? 0.0f : 1.0f);
      s.count.push_back(int(blocks.size()));
      for (int b : blocks) {
        const int r = int(std::upper_bound(m.row_ptr.begin(), m.row_ptr.end(), b) -
                          m.row_ptr.begin()) - 1;
        a_ptrs.push_back(d.values + m.value_off[b]);
        s.b_off.push_back(m.col_scalar_off[m.block_col[b]]);
        s.c_off.push_back(m.row_scalar_off[r]);
      }
    }
    const size_t bytes = a_ptrs.size() * sizeof(float*);
    cuda_ok(cudaMalloc(reinterpret_cast<void**>(&s.dA), bytes));
    cuda_ok(cudaMalloc(reinterpret_cast<void**>(&s.dB), bytes));
    cuda_ok(cudaMalloc(reinterpret_cast<void**>(&s.dC), bytes));
    cuda_ok(cudaMemcpy(s.dA, a_ptrs.data(), bytes, cudaMemcpyHostToDevice));
    s.hB.resize(a_ptrs.size());
    s.hC.resize(a_ptrs.size());
  }
}

GroupedGemmPlan::~GroupedGemmPlan() = default;

int GroupedGemmPlan::launch_count() const { return int(impl_->slots.size()); }

void GroupedGemmPlan::execute(const float* B, float* C, cudaStream_t stream) {
  Impl& d = *impl_;
  blas_ok(cublasSetStream(d.h, stream));
  // rows of C that no slot writes (block rows without blocks) must read as 0
  cuda_ok(cudaMemsetAsync(C, 0, size_t(d.M) * size_t(d.rhs) * sizeof(float), stream));
  for (Impl::Slot& s : d.slots) {
    for (size_t i = 0; i < s.hB.size(); ++i) {
      s.hB[i] = B + s.b_off[i];
      s.hC[i] = C + s.c_off[i];
    }
    const size_t bytes = s.hB.size() * sizeof(float*);
    cuda_ok(cudaMemcpyAsync(s.dB, s.hB.data(), bytes, cudaMemcpyHostToDevice, stream));
    cuda_ok(cudaMemcpyAsync(s.dC, s.hC.data(), bytes, cudaMemcpyHostToDevice, stream));
    blas_ok(cublasSgemmGroupedBatched(d.h, s.op.data(), s.op.data(), s.m.data(), s.n.data(),
                                      s.k.data(), s.alpha.data(), s.dA, s.lda.data(), s.dB,
                                      s.ldb.data(), s.beta.data(), s.dC, s.ldc.data(),
                                      int(s.count.size()), s.count.data()));
  }
  // (copies from pageable host memory are staged before cudaMemcpyAsync returns, so the host
  // pointer arrays may be rewritten by the next call)
}

}  // namespace vbsr
