// vbsr_api.cpp — the C++ drop-in API (include/varblockspmm/vbsr.hpp) over the C ABI. Status codes
// map back to the reference's exception types: VBSR_INVALID_ARGUMENT -> std::invalid_argument,
// anything else -> std::runtime_error (reference: src/format/vbsr.cpp:13-17,32-80,
// src/plan/plan.cpp:9-17, src/kernels/row_owned.cu:367-372).
#include "varblockspmm/vbsr.hpp"

#include <stdexcept>
#include <string>
#include <utility>

namespace vbsr {
namespace {
void check(vbsr_status s) {
  if (s == VBSR_OK) return;
  const std::string msg = vbsr_get_last_error();
  if (s == VBSR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

// Copies a library-owned host matrix into a HostMatrix and frees it.
HostMatrix take(vbsr_host_matrix* h) {
  vbsr_host_matrix_view v{};
  vbsr_host_matrix_view_get(h, &v);
  HostMatrix m;
  m.block_rows = v.block_rows;
  m.block_cols = v.block_cols;
  m.row_ptr.assign(v.row_ptr, v.row_ptr + v.row_ptr_len);
  m.block_col.assign(v.block_col, v.block_col + v.block_col_len);
  m.row_size.assign(v.row_size, v.row_size + v.row_size_len);
  m.col_size.assign(v.col_size, v.col_size + v.col_size_len);
  m.row_scalar_off.assign(v.row_scalar_off, v.row_scalar_off + v.row_scalar_off_len);
  m.col_scalar_off.assign(v.col_scalar_off, v.col_scalar_off + v.col_scalar_off_len);
  m.value_off.assign(v.value_off, v.value_off + v.value_off_len);
  if (v.values_len) m.values.assign(v.values, v.values + v.values_len);
  vbsr_host_matrix_free(h);
  return m;
}

vbsr_device_matrix to_c(const DeviceMatrix& a) {
  vbsr_device_matrix v{};
  v.block_rows = a.block_rows;
  v.block_cols = a.block_cols;
  v.nnzb = a.nnzb;
  v.scalar_rows = a.scalar_rows;
  v.scalar_cols = a.scalar_cols;
  v.row_ptr = a.row_ptr;
  v.block_col = a.block_col;
  v.row_size = a.row_size;
  v.col_size = a.col_size;
  v.row_scalar_off = a.row_scalar_off;
  v.col_scalar_off = a.col_scalar_off;
  v.value_off = a.value_off;
  v.values = a.values;
  return v;
}
}  // namespace

void HostMatrix::validate() const {
  const vbsr_host_matrix_view v = detail::view_of(*this);
  check(vbsr_host_validate(&v));
}

Matrix::Matrix(const HostMatrix& host) {
  const vbsr_host_matrix_view v = detail::view_of(host);
  check(vbsr_matrix_create(&v, -1, &m_));
  rows_ = host.scalar_rows();
  cols_ = host.scalar_cols();
}
Matrix::~Matrix() { vbsr_matrix_destroy(m_); }
Matrix::Matrix(Matrix&& o) noexcept : m_(std::exchange(o.m_, nullptr)), rows_(o.rows_), cols_(o.cols_) {}
Matrix& Matrix::operator=(Matrix&& o) noexcept {
  if (this != &o) {
    vbsr_matrix_destroy(m_);
    m_ = std::exchange(o.m_, nullptr);
    rows_ = o.rows_;
    cols_ = o.cols_;
  }
  return *this;
}
DeviceMatrix Matrix::device_view() const {
  DeviceMatrix d;
  if (m_ == nullptr) return d;
  vbsr_device_matrix v{};
  check(vbsr_matrix_device_view(m_, &v));
  d.block_rows = v.block_rows;
  d.block_cols = v.block_cols;
  d.nnzb = v.nnzb;
  d.scalar_rows = v.scalar_rows;
  d.scalar_cols = v.scalar_cols;
  d.row_ptr = v.row_ptr;
  d.block_col = v.block_col;
  d.row_size = v.row_size;
  d.col_size = v.col_size;
  d.row_scalar_off = v.row_scalar_off;
  d.col_scalar_off = v.col_scalar_off;
  d.value_off = v.value_off;
  d.values = v.values;
  return d;
}

HostMatrix generate(const GeneratorOptions& o) {
  vbsr_generator_options c{};
  c.block_rows = o.block_rows;
  c.block_cols = o.block_cols;
  c.degree = o.degree;
  c.rhs_width = o.rhs_width;
  c.distribution = int(o.distribution);
  c.local_columns = o.local_columns ? 1 : 0;
  c.seed = o.seed;
  c.profile = o.profile == Profile::Spec ? VBSR_PROFILE_SPEC : VBSR_PROFILE_REFERENCE;
  c.with_values = 1;
  c.threads = 0;
  vbsr_host_matrix* h = nullptr;
  check(vbsr_generate(&c, &h));
  return take(h);
}

HostMatrix from_csr(int64_t rows, int64_t cols, const std::vector<int64_t>& row_ptr,
                    const std::vector<int64_t>& col_idx, const std::vector<float>& values,
                    const std::vector<int32_t>& row_sizes, const std::vector<int32_t>& col_sizes) {
  if (row_ptr.size() != size_t(rows) + 1 || col_idx.size() != values.size() ||
      col_idx.size() != size_t(row_ptr.back()))
    throw std::invalid_argument("CSR arrays do not match the dimensions");
  vbsr_host_matrix* h = nullptr;
  check(vbsr_host_matrix_from_csr(rows, cols, row_ptr.data(), col_idx.data(), values.data(),
                                  int32_t(row_sizes.size()), row_sizes.data(),
                                  int32_t(col_sizes.size()), col_sizes.data(), &h));
  return take(h);
}

void save_matrix(const HostMatrix& m, const char* path) {
  const vbsr_host_matrix_view v = detail::view_of(m);
  check(vbsr_host_matrix_save(&v, path));
}

HostMatrix load_matrix(const char* path) {
  vbsr_host_matrix* h = nullptr;
  check(vbsr_host_matrix_load(path, &h));
  return take(h);
}

Plan::Plan(const Matrix& matrix, PlanOptions options) : options_(options) {
  vbsr_plan* p = nullptr;
  check(vbsr_plan_create(matrix.m_, options.rhs_width, int(options.kernel), &p));
  p_ = std::shared_ptr<vbsr_plan>(p, [](vbsr_plan* q) { vbsr_plan_destroy(q); });
}

void Plan::execute(const float* B, float* C, cudaStream_t stream) const {
  check(vbsr_plan_execute(p_.get(), B, C, reinterpret_cast<vbsr_stream_t>(stream)));
}

MultiPlan::MultiPlan(const HostMatrix& host, const std::vector<int>& devices,
                     PlanOptions options) {
  const vbsr_host_matrix_view v = detail::view_of(host);
  vbsr_multi_plan* p = nullptr;
  check(vbsr_multi_plan_create(&v, int(devices.size()), devices.data(), options.rhs_width,
                               int(options.kernel), 0u, &p));
  p_ = std::shared_ptr<vbsr_multi_plan>(p, [](vbsr_multi_plan* q) { vbsr_multi_plan_destroy(q); });
}

void MultiPlan::replicate_B(const float* B, int src_device) {
  check(vbsr_multi_plan_replicate_B(p_.get(), B, src_device));
}

void MultiPlan::execute() { check(vbsr_multi_plan_execute(p_.get())); }

float MultiPlan::synchronize() {
  float ms = 0.0f;
  check(vbsr_multi_plan_synchronize(p_.get(), &ms));
  return ms;
}

void MultiPlan::gather_C(float* C, int dst_device) {
  check(vbsr_multi_plan_gather_C(p_.get(), C, dst_device));
}

int MultiPlan::size() const {
  int n = 0;
  check(vbsr_multi_plan_count(p_.get(), &n));
  return n;
}

int Plan::launch_count() const {
  int n = 0;
  check(vbsr_plan_launch_count(p_.get(), &n));
  return n;
}

void launch_row_owned(DeviceMatrix a, const int32_t* order, int small, int large, const float* B,
                      float* C, int rhs, cudaStream_t stream) {
  const vbsr_device_matrix v = to_c(a);
  check(vbsr_launch_row_owned(&v, order, small, large, B, C, rhs,
                              reinterpret_cast<vbsr_stream_t>(stream)));
}

void launch_row_owned_scalar(DeviceMatrix a, const float* B, float* C, int rhs,
                             cudaStream_t stream) {
  const vbsr_device_matrix v = to_c(a);
  check(vbsr_launch_row_owned_scalar(&v, B, C, rhs, reinterpret_cast<vbsr_stream_t>(stream)));
}

}  // namespace vbsr
