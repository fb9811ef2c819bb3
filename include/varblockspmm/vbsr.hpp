// varblockspmm/vbsr.hpp — C++ drop-in for the host API of King-Clawthorne/VarBlockSpMM
// (include/varblockspmm/vbsr.hpp of the reference), implemented over the engine's C ABI
// (vbsr_b200.h) by libvbsr_b200_cxx.so.
//
// Same names, members, signatures, exception types and stream semantics as the reference:
//   HostMatrix (ref vbsr.hpp:16-29), DeviceMatrix (:32-38), Matrix (:41-64), Distribution (:67),
//   GeneratorOptions (:70-76), generate (:80), cpu_reference (:87), Kernel (:91),
//   PlanOptions (:94-97), Plan (:104-119), ScalarCsrPlan (:121-137), GroupedGemmPlan (:139-155),
//   launch_row_owned (:158-159),
//   launch_row_owned_scalar (:161).
// Differences a user can see:
//   * GeneratorOptions has one more member, `profile` (default Profile::Reference reproduces the
//     reference's generate() bit for bit; Profile::Spec gives the benchmark specification's
//     block-size distributions).
//   * Plan owns its device-side schedule (built once in the constructor); copies share it.
//   * DeviceMatrix::values points at the engine's re-laid-out value array (8-column groups), so a
//     DeviceMatrix is only meaningful to this library's launchers.
//   * cpu_reference is the CPU oracle: it is defined in the test-infrastructure library
//     oracle/_build/libvbsr_oracle.so, not in the engine library.
//   * The library comparators ScalarCsrPlan / GroupedGemmPlan (ref vbsr.hpp:121-155) are this
//     library's own cuSPARSE / grouped-cuBLAS plans (vbsr_comparators.cpp); ScalarCsrPlan switches
//     to 64-bit CSR indices when the expanded matrix has 2^31 or more nonzeros.
#pragma once
#include <cuda_runtime_api.h>

#include <cstdint>
#include <memory>
#include <vector>

#include "vbsr_b200.h"

namespace vbsr {

/** Host-side variable-block sparse-row matrix (column-major blocks packed in row order). */
struct HostMatrix {
  int block_rows{}, block_cols{};
  std::vector<int32_t> row_ptr, block_col, row_size, col_size;
  std::vector<int64_t> row_scalar_off, col_scalar_off, value_off;
  std::vector<float> values;
  int64_t scalar_rows() const { return row_scalar_off.empty() ? 0 : row_scalar_off.back(); }
  int64_t scalar_cols() const { return col_scalar_off.empty() ? 0 : col_scalar_off.back(); }
  /** Throws std::invalid_argument if metadata or packed values are inconsistent. */
  void validate() const;
};

/** Non-owning device view. */
struct DeviceMatrix {
  int block_rows{}, block_cols{}, nnzb{};
  int64_t scalar_rows{}, scalar_cols{};
  const int32_t *row_ptr{}, *block_col{}, *row_size{}, *col_size{};
  const int64_t *row_scalar_off{}, *col_scalar_off{}, *value_off{};
  const float* values{};
};

/** Owns an immutable copy of a validated matrix in device memory (current device). */
class Matrix {
 public:
  explicit Matrix(const HostMatrix& host);
  ~Matrix();
  Matrix(const Matrix&) = delete;
  Matrix& operator=(const Matrix&) = delete;
  Matrix(Matrix&&) noexcept;
  Matrix& operator=(Matrix&&) noexcept;
  DeviceMatrix device_view() const;
  int64_t scalar_rows() const { return rows_; }
  int64_t scalar_cols() const { return cols_; }
  /** The underlying C handle (for mixing with the C ABI). */
  const vbsr_matrix* handle() const { return m_; }

 private:
  friend class Plan;
  vbsr_matrix* m_{};
  int64_t rows_{}, cols_{};
};

enum class Distribution { Uniform, LowVariance, HighVariance, Bimodal };
enum class Profile { Reference, Spec };

struct GeneratorOptions {
  int block_rows = 1024, block_cols = 1024, degree = 4;
  int rhs_width = 32;
  Distribution distribution = Distribution::HighVariance;
  bool local_columns = true;
  uint64_t seed = 1;
  Profile profile = Profile::Reference;
};

/** Generates a validated matrix; equal options give equal matrices. */
HostMatrix generate(const GeneratorOptions&);

/** Real matrices (no reference counterpart): a scalar CSR matrix as VBSR for a block partition
 * (vbsr_host_matrix_from_csr), and the binary VBSR file (vbsr_host_matrix_save / _load). */
HostMatrix from_csr(int64_t rows, int64_t cols, const std::vector<int64_t>& row_ptr,
                    const std::vector<int64_t>& col_idx, const std::vector<float>& values,
                    const std::vector<int32_t>& row_sizes, const std::vector<int32_t>& col_sizes);
void save_matrix(const HostMatrix&, const char* path);
HostMatrix load_matrix(const char* path);

/** C = A*B on the CPU with double accumulation per block (the oracle; see header comment). */
std::vector<float> cpu_reference(const HostMatrix&, const std::vector<float>& B, int rhs);

enum class Kernel { Auto, RowOwned, SplitRow };

struct PlanOptions {
  int rhs_width = 32;
  Kernel kernel = Kernel::Auto;
};

/** Execution plan; the Matrix must outlive it. execute() enqueues asynchronously. */
class Plan {
 public:
  Plan(const Matrix&, PlanOptions);
  void execute(const float* B, float* C, cudaStream_t stream = 0) const;
  int launch_count() const;
  const vbsr_plan* handle() const { return p_.get(); }

 private:
  std::shared_ptr<vbsr_plan> p_;
  PlanOptions options_{};
};

/** cuSPARSE comparator: C = A*B with A expanded to scalar CSR (ref vbsr.hpp:121-137). The
 * workspace is allocated by the first execute and kept. */
class ScalarCsrPlan {
 public:
  ScalarCsrPlan(const HostMatrix&, int rhs_width);
  ~ScalarCsrPlan();
  ScalarCsrPlan(const ScalarCsrPlan&) = delete;
  void execute(const float* B, float* C, cudaStream_t stream = 0);
  size_t workspace_bytes() const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

/** Grouped cuBLAS comparator: per slot k (the k-th block of every block row), one grouped SGEMM
 * over the blocks grouped by shape (ref vbsr.hpp:139-155). */
class GroupedGemmPlan {
 public:
  GroupedGemmPlan(const HostMatrix&, int rhs_width);
  ~GroupedGemmPlan();
  GroupedGemmPlan(const GroupedGemmPlan&) = delete;
  void execute(const float* B, float* C, cudaStream_t stream = 0);
  int launch_count() const;
  size_t workspace_bytes() const { return 0; }

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

/** Multi-GPU plan (no reference counterpart; the reference is single-GPU): the block rows split
 * into balanced shards, one per entry of `devices` (entries may repeat), each with its own plan,
 * B replica, C block and stream. replicate_B copies B (K x rhs) peer to peer along a doubling
 * tree (src_device < 0: B is host memory); execute runs every shard with no collective;
 * synchronize waits and returns the longest shard time in ms; gather_C assembles the M x rhs
 * column-major result (dst_device < 0: host memory). */
class MultiPlan {
 public:
  MultiPlan(const HostMatrix&, const std::vector<int>& devices, PlanOptions);
  void replicate_B(const float* B, int src_device = -1);
  void execute();
  float synchronize();
  void gather_C(float* C, int dst_device = -1);
  int size() const;
  const vbsr_multi_plan* handle() const { return p_.get(); }

 private:
  std::shared_ptr<vbsr_multi_plan> p_;
};

void launch_row_owned(DeviceMatrix, const int32_t* row_shape_order, int small_row_count,
                      int large_row_count, const float*, float*, int rhs, cudaStream_t);
void launch_row_owned_scalar(DeviceMatrix, const float*, float*, int rhs, cudaStream_t);

namespace detail {
inline vbsr_host_matrix_view view_of(const HostMatrix& m) {
  vbsr_host_matrix_view v{};
  v.block_rows = m.block_rows;
  v.block_cols = m.block_cols;
  v.row_ptr = m.row_ptr.data();               v.row_ptr_len = m.row_ptr.size();
  v.block_col = m.block_col.data();           v.block_col_len = m.block_col.size();
  v.row_size = m.row_size.data();             v.row_size_len = m.row_size.size();
  v.col_size = m.col_size.data();             v.col_size_len = m.col_size.size();
  v.row_scalar_off = m.row_scalar_off.data(); v.row_scalar_off_len = m.row_scalar_off.size();
  v.col_scalar_off = m.col_scalar_off.data(); v.col_scalar_off_len = m.col_scalar_off.size();
  v.value_off = m.value_off.data();           v.value_off_len = m.value_off.size();
  v.values = m.values.data();                 v.values_len = m.values.size();
  return v;
}
}  // namespace detail

}  // namespace vbsr
