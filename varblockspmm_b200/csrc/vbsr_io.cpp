// vbsr_io.cpp — getting real matrices into the engine: conversion of a scalar CSR matrix into the
// VBSR host format for a given block partition, and a binary on-disk VBSR file. Host only.
//
// No reference counterpart: the reference generates its matrices and has no loader or file format
// (its research notes leave real matrices to future work).
//
// On-disk format, little-endian, version 1:
//   8 bytes   magic "VBSRMAT1"
//   int32     block_rows R, block_cols S
//   uint64    nnzb, value count
//   arrays in this order, no padding: row_ptr (int32, R+1), block_col (int32, nnzb),
//   row_size (int32, R), col_size (int32, S), row_scalar_off (int64, R+1),
//   col_scalar_off (int64, S+1), value_off (int64, nnzb+1), values (float32; each block h x w
//   column-major, blocks in row order: the HostMatrix layout).
// A loaded file is validated like any HostMatrix.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "vbsr_internal.h"

using vbsr_b200::clear_error;
using vbsr_b200::set_error;

namespace vbsr_b200 {
vbsr_status validate_view(const vbsr_host_matrix_view* v, bool check_values);
}

namespace {

constexpr char kMagic[8] = {'V', 'B', 'S', 'R', 'M', 'A', 'T', '1'};

bool valid_block_size(int32_t s) { return s >= 8 && s <= 64 && s % 8 == 0; }

vbsr_status finish(vbsr_host_matrix* m, vbsr_host_matrix** out) {
  vbsr_host_matrix_view v;
  vbsr_host_matrix_view_get(m, &v);
  const vbsr_status st = vbsr_b200::validate_view(&v, true);
  if (st != VBSR_OK) {
    delete m;
    return st;
  }
  *out = m;
  return VBSR_OK;
}

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) std::fclose(f);
  }
};

template <class T>
bool put(FILE* f, const T* p, size_t n) {
  return n == 0 || std::fwrite(p, sizeof(T), n, f) == n;
}
template <class T>
bool get(FILE* f, std::vector<T>& v, size_t n) {
  v.resize(n);
  return n == 0 || std::fread(v.data(), sizeof(T), n, f) == n;
}

}  // namespace

extern "C" {

vbsr_status vbsr_host_matrix_from_csr(int64_t rows, int64_t cols, const int64_t* row_ptr,
                                      const int64_t* col_idx, const float* values,
                                      int32_t block_rows, const int32_t* row_sizes,
                                      int32_t block_cols, const int32_t* col_sizes,
                                      vbsr_host_matrix** out) {
  clear_error();
  if (out == nullptr || row_ptr == nullptr || row_sizes == nullptr || col_sizes == nullptr)
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (rows <= 0 || cols <= 0 || block_rows <= 0 || block_cols <= 0)
    return set_error(VBSR_INVALID_ARGUMENT, "positive dimensions required");
  const int64_t nnz = row_ptr[rows];
  if (nnz > 0 && (col_idx == nullptr || values == nullptr))
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  int64_t sum = 0;
  for (int32_t i = 0; i < block_rows; ++i) {
    if (!valid_block_size(row_sizes[i]))
      return set_error(VBSR_INVALID_ARGUMENT, "block sizes must be multiples of 8 in [8, 64]");
    sum += row_sizes[i];
  }
  if (sum != rows) return set_error(VBSR_INVALID_ARGUMENT, "row block sizes do not sum to the rows");
  sum = 0;
  for (int32_t j = 0; j < block_cols; ++j) {
    if (!valid_block_size(col_sizes[j]))
      return set_error(VBSR_INVALID_ARGUMENT, "block sizes must be multiples of 8 in [8, 64]");
    sum += col_sizes[j];
  }
  if (sum != cols)
    return set_error(VBSR_INVALID_ARGUMENT, "column block sizes do not sum to the columns");
  if (row_ptr[0] != 0) return set_error(VBSR_INVALID_ARGUMENT, "row_ptr must start at 0");
  for (int64_t r = 0; r < rows; ++r)
    if (row_ptr[r + 1] < row_ptr[r]) return set_error(VBSR_INVALID_ARGUMENT, "row_ptr must be monotone");
  for (int64_t e = 0; e < nnz; ++e)
    if (col_idx[e] < 0 || col_idx[e] >= cols)
      return set_error(VBSR_INVALID_ARGUMENT, "column index out of range");

  auto* m = new (std::nothrow) vbsr_host_matrix;
  if (m == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  try {
    m->block_rows = block_rows;
    m->block_cols = block_cols;
    m->row_size.assign(row_sizes, row_sizes + block_rows);
    m->col_size.assign(col_sizes, col_sizes + block_cols);
    m->row_scalar_off.assign(size_t(block_rows) + 1, 0);
    m->col_scalar_off.assign(size_t(block_cols) + 1, 0);
    for (int32_t i = 0; i < block_rows; ++i) m->row_scalar_off[i + 1] = m->row_scalar_off[i] + row_sizes[i];
    for (int32_t j = 0; j < block_cols; ++j) m->col_scalar_off[j + 1] = m->col_scalar_off[j] + col_sizes[j];
    // scalar column -> its block column
    std::vector<int32_t> col_block(static_cast<size_t>(cols));
    for (int32_t j = 0; j < block_cols; ++j)
      std::fill(col_block.begin() + m->col_scalar_off[j], col_block.begin() + m->col_scalar_off[j + 1], j);
    // pass 1: the block columns each block row touches (sorted), and the value offsets
    std::vector<int32_t> seen(static_cast<size_t>(block_cols), -1), slot(static_cast<size_t>(block_cols), 0);
    m->row_ptr.assign(1, 0);
    m->value_off.assign(1, 0);
    std::vector<int32_t> touched;
    for (int32_t i = 0; i < block_rows; ++i) {
      touched.clear();
      for (int64_t r = m->row_scalar_off[i]; r < m->row_scalar_off[i + 1]; ++r)
        for (int64_t e = row_ptr[r]; e < row_ptr[r + 1]; ++e) {
          const int32_t j = col_block[size_t(col_idx[e])];
          if (seen[j] != i) {
            seen[j] = i;
            touched.push_back(j);
          }
        }
      std::sort(touched.begin(), touched.end());
      for (int32_t j : touched) {
        m->block_col.push_back(j);
        m->value_off.push_back(m->value_off.back() + int64_t(row_sizes[i]) * col_sizes[j]);
      }
      m->row_ptr.push_back(int32_t(m->block_col.size()));
    }
    // pass 2: scatter the nonzeros into their dense blocks (duplicates are summed)
    m->values.assign(size_t(m->value_off.back()), 0.0f);
    for (int32_t i = 0; i < block_rows; ++i) {
      const int h = row_sizes[i];
      for (int32_t b = m->row_ptr[i]; b < m->row_ptr[i + 1]; ++b) slot[m->block_col[b]] = b;
      for (int64_t r = m->row_scalar_off[i]; r < m->row_scalar_off[i + 1]; ++r) {
        const int64_t lr = r - m->row_scalar_off[i];
        for (int64_t e = row_ptr[r]; e < row_ptr[r + 1]; ++e) {
          const int64_t c = col_idx[e];
          const int32_t j = col_block[size_t(c)];
          const int64_t lc = c - m->col_scalar_off[j];
          m->values[size_t(m->value_off[slot[j]] + lr + lc * h)] += values[e];
        }
      }
    }
  } catch (const std::bad_alloc&) {
    delete m;
    return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  }
  return finish(m, out);
}

vbsr_status vbsr_host_matrix_save(const vbsr_host_matrix_view* v, const char* path) {
  clear_error();
  if (v == nullptr || path == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  const vbsr_status st = vbsr_b200::validate_view(v, true);
  if (st != VBSR_OK) return st;
  File file;
  file.f = std::fopen(path, "wb");
  if (file.f == nullptr) return set_error(VBSR_INVALID_ARGUMENT, std::string("cannot open ") + path);
  const uint64_t nnzb = v->block_col_len, nvals = v->values_len;
  bool ok = put(file.f, kMagic, 8) && put(file.f, &v->block_rows, 1) &&
            put(file.f, &v->block_cols, 1) && put(file.f, &nnzb, 1) && put(file.f, &nvals, 1) &&
            put(file.f, v->row_ptr, v->row_ptr_len) && put(file.f, v->block_col, v->block_col_len) &&
            put(file.f, v->row_size, v->row_size_len) && put(file.f, v->col_size, v->col_size_len) &&
            put(file.f, v->row_scalar_off, v->row_scalar_off_len) &&
            put(file.f, v->col_scalar_off, v->col_scalar_off_len) &&
            put(file.f, v->value_off, v->value_off_len) && put(file.f, v->values, v->values_len);
  ok = (std::fclose(file.f) == 0) && ok;
  file.f = nullptr;
  if (!ok) return set_error(VBSR_INVALID_ARGUMENT, std::string("write failed: ") + path);
  return VBSR_OK;
}

vbsr_status vbsr_host_matrix_load(const char* path, vbsr_host_matrix** out) {
  clear_error();
  if (path == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  File file;
  file.f = std::fopen(path, "rb");
  if (file.f == nullptr) return set_error(VBSR_INVALID_ARGUMENT, std::string("cannot open ") + path);
  char magic[8];
  int32_t R = 0, S = 0;
  uint64_t nnzb = 0, nvals = 0;
  if (std::fread(magic, 1, 8, file.f) != 8 || std::memcmp(magic, kMagic, 8) != 0)
    return set_error(VBSR_INVALID_ARGUMENT, "not a VBSR file (bad magic)");
  if (std::fread(&R, 4, 1, file.f) != 1 || std::fread(&S, 4, 1, file.f) != 1 ||
      std::fread(&nnzb, 8, 1, file.f) != 1 || std::fread(&nvals, 8, 1, file.f) != 1)
    return set_error(VBSR_INVALID_ARGUMENT, "truncated VBSR file header");
  if (R <= 0 || S <= 0 || nnzb > (uint64_t(1) << 40) || nvals > (uint64_t(1) << 44))
    return set_error(VBSR_INVALID_ARGUMENT, "implausible VBSR file header");
  auto* m = new (std::nothrow) vbsr_host_matrix;
  if (m == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  bool ok = false;
  try {
    m->block_rows = R;
    m->block_cols = S;
    ok = get(file.f, m->row_ptr, size_t(R) + 1) && get(file.f, m->block_col, nnzb) &&
         get(file.f, m->row_size, size_t(R)) && get(file.f, m->col_size, size_t(S)) &&
         get(file.f, m->row_scalar_off, size_t(R) + 1) &&
         get(file.f, m->col_scalar_off, size_t(S) + 1) && get(file.f, m->value_off, nnzb + 1) &&
         get(file.f, m->values, nvals);
  } catch (const std::bad_alloc&) {
    delete m;
    return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  }
  if (!ok) {
    delete m;
    return set_error(VBSR_INVALID_ARGUMENT, "truncated VBSR file");
  }
  return finish(m, out);
}

}  // extern "C"
