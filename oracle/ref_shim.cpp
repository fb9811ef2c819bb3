// ref_shim.cpp — TEST INFRASTRUCTURE ONLY. A C-callable shim over the reference's own host code
// (King-Clawthorne/VarBlockSpMM src/format/vbsr.cpp and src/format/generator.cpp, compiled
// unchanged from the reference checkout by oracle/Makefile into oracle/_ref/libvbsr_ref.so).
// It lets the tests pin the CPU restatement (vbsr_oracle.c) and the engine's generator and
// validation against the reference itself, and lets bench.py --impl reference time the
// reference's own cpu_reference.
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "varblockspmm/vbsr.hpp"

namespace {
thread_local std::string g_err;

vbsr::HostMatrix from_view(const int32_t* dims, const int32_t* row_ptr, const int32_t* block_col,
                           const int32_t* row_size, const int32_t* col_size,
                           const int64_t* row_off, const int64_t* col_off,
                           const int64_t* value_off, const float* values, const int64_t* lens) {
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
  return m;
}

// Block rows [r0, r1) of m as a standalone HostMatrix (full column structure).
vbsr::HostMatrix row_slice(const vbsr::HostMatrix& m, int r0, int r1) {
  vbsr::HostMatrix s;
  s.block_rows = r1 - r0;
  s.block_cols = m.block_cols;
  const int b0 = m.row_ptr[r0], b1 = m.row_ptr[r1];
  const int64_t v0 = m.value_off[b0], v1 = m.value_off[b1];
  for (int i = r0; i <= r1; ++i) {
    s.row_ptr.push_back(m.row_ptr[i] - b0);
    s.row_scalar_off.push_back(m.row_scalar_off[i] - m.row_scalar_off[r0]);
  }
  s.row_size.assign(m.row_size.begin() + r0, m.row_size.begin() + r1);
  s.block_col.assign(m.block_col.begin() + b0, m.block_col.begin() + b1);
  for (int b = b0; b <= b1; ++b) s.value_off.push_back(m.value_off[b] - v0);
  s.values.assign(m.values.begin() + v0, m.values.begin() + v1);
  s.col_size = m.col_size;
  s.col_scalar_off = m.col_scalar_off;
  return s;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

void* ref_generate(int rows, int cols, int degree, int distribution, int local, uint64_t seed) {
  vbsr::GeneratorOptions o;
  o.block_rows = rows;
  o.block_cols = cols;
  o.degree = degree;
  o.distribution = static_cast<vbsr::Distribution>(distribution);
  o.local_columns = local != 0;
  o.seed = seed;
  try {
    return new vbsr::HostMatrix(vbsr::generate(o));
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void ref_free(void* h) { delete static_cast<vbsr::HostMatrix*>(h); }

// Exposes the arrays of a generated matrix: dims[2], pointers[8], lens[8].
void ref_arrays(void* h, int32_t* dims, const void** ptrs, int64_t* lens) {
  auto* m = static_cast<vbsr::HostMatrix*>(h);
  dims[0] = m->block_rows;
  dims[1] = m->block_cols;
  ptrs[0] = m->row_ptr.data();        lens[0] = int64_t(m->row_ptr.size());
  ptrs[1] = m->block_col.data();      lens[1] = int64_t(m->block_col.size());
  ptrs[2] = m->row_size.data();       lens[2] = int64_t(m->row_size.size());
  ptrs[3] = m->col_size.data();       lens[3] = int64_t(m->col_size.size());
  ptrs[4] = m->row_scalar_off.data(); lens[4] = int64_t(m->row_scalar_off.size());
  ptrs[5] = m->col_scalar_off.data(); lens[5] = int64_t(m->col_scalar_off.size());
  ptrs[6] = m->value_off.data();      lens[6] = int64_t(m->value_off.size());
  ptrs[7] = m->values.data();         lens[7] = int64_t(m->values.size());
}

// HostMatrix::validate on a copy of the given arrays: 0 = valid, 1 = invalid_argument (message in
// ref_last_error), 2 = other exception.
int ref_validate(const int32_t* dims, const int32_t* row_ptr, const int32_t* block_col,
                 const int32_t* row_size, const int32_t* col_size, const int64_t* row_off,
                 const int64_t* col_off, const int64_t* value_off, const float* values,
                 const int64_t* lens) {
  try {
    from_view(dims, row_ptr, block_col, row_size, col_size, row_off, col_off, value_off, values,
              lens)
        .validate();
    return 0;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 2;
  }
}

// vbsr::cpu_reference for block rows [r0, r1) of the given matrix, run as `threads` independent
// calls of the unchanged reference function on row slices. C receives the slice's rows
// (column-major, ld = row_scalar_off[r1] - row_scalar_off[r0]). Returns 0 on success.
int ref_cpu_reference_rows(const int32_t* dims, const int32_t* row_ptr, const int32_t* block_col,
                           const int32_t* row_size, const int32_t* col_size,
                           const int64_t* row_off, const int64_t* col_off,
                           const int64_t* value_off, const float* values, const int64_t* lens,
                           const float* B, int rhs, int r0, int r1, float* C, int threads) {
  try {
    const vbsr::HostMatrix full = from_view(dims, row_ptr, block_col, row_size, col_size, row_off,
                                            col_off, value_off, values, lens);
    const std::vector<float> input(B, B + full.scalar_cols() * rhs);
    const int rows = r1 - r0;
    if (threads < 1) threads = 1;
    if (threads > rows) threads = rows;
    std::vector<vbsr::HostMatrix> parts;
    std::vector<int> starts;
    for (int t = 0; t < threads; ++t) {
      const int a = r0 + int(int64_t(rows) * t / threads);
      const int b = r0 + int(int64_t(rows) * (t + 1) / threads);
      parts.push_back(row_slice(full, a, b));
      starts.push_back(a);
    }
    const int64_t ldc = full.row_scalar_off[r1] - full.row_scalar_off[r0];
    std::vector<std::thread> pool;
    std::vector<std::string> errs(threads);
    for (int t = 0; t < threads; ++t) {
      pool.emplace_back([&, t] {
        try {
          const std::vector<float> out = vbsr::cpu_reference(parts[t], input, rhs);
          const int64_t mt = parts[t].scalar_rows();
          const int64_t base = full.row_scalar_off[starts[t]] - full.row_scalar_off[r0];
          for (int n = 0; n < rhs; ++n)
            std::memcpy(C + base + int64_t(n) * ldc, out.data() + int64_t(n) * mt,
                        size_t(mt) * sizeof(float));
        } catch (const std::exception& e) {
          errs[t] = e.what();
        }
      });
    }
    for (auto& th : pool) th.join();
    for (auto& e : errs)
      if (!e.empty()) {
        g_err = e;
        return 1;
      }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

// Timing form of ref_cpu_reference_rows for the benchmark's reference arm: ref_prepare builds,
// outside any timed region, the per-thread row-slice HostMatrix parts and the std::vector copy of B
// that vbsr::cpu_reference takes; ref_run then runs only the reference's cpu_reference calls (one
// per thread, as independent calls on row slices) and reports their wall time; ref_release frees
// the prepared state.
struct RefPrepared {
  std::vector<vbsr::HostMatrix> parts;
  std::vector<int64_t> bases;  // first output row of each part within [r0, r1)
  std::vector<float> input;
  int rhs = 0;
  int64_t ldc = 0;
};

void* ref_prepare(const int32_t* dims, const int32_t* row_ptr, const int32_t* block_col,
                  const int32_t* row_size, const int32_t* col_size, const int64_t* row_off,
                  const int64_t* col_off, const int64_t* value_off, const float* values,
                  const int64_t* lens, const float* B, int rhs, int r0, int r1, int threads) {
  try {
    const vbsr::HostMatrix full = from_view(dims, row_ptr, block_col, row_size, col_size, row_off,
                                            col_off, value_off, values, lens);
    auto* h = new RefPrepared;
    h->rhs = rhs;
    h->input.assign(B, B + full.scalar_cols() * rhs);
    h->ldc = full.row_scalar_off[r1] - full.row_scalar_off[r0];
    const int rows = r1 - r0;
    if (threads < 1) threads = 1;
    if (threads > rows) threads = rows;
    for (int t = 0; t < threads; ++t) {
      const int a = r0 + int(int64_t(rows) * t / threads);
      const int b = r0 + int(int64_t(rows) * (t + 1) / threads);
      h->parts.push_back(row_slice(full, a, b));
      h->bases.push_back(full.row_scalar_off[a] - full.row_scalar_off[r0]);
    }
    return h;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

int ref_run(void* handle, float* C, double* seconds) {
  auto* h = static_cast<RefPrepared*>(handle);
  const int threads = int(h->parts.size());
  std::vector<std::vector<float>> outs(threads);
  std::vector<std::string> errs(threads);
  const auto t0 = std::chrono::steady_clock::now();
  {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
      pool.emplace_back([&, t] {
        try {
          outs[t] = vbsr::cpu_reference(h->parts[t], h->input, h->rhs);
        } catch (const std::exception& e) {
          errs[t] = e.what();
        }
      });
    }
    for (auto& th : pool) th.join();
  }
  const auto t1 = std::chrono::steady_clock::now();
  if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
  for (auto& e : errs)
    if (!e.empty()) {
      g_err = e;
      return 1;
    }
  if (C != nullptr)
    for (int t = 0; t < threads; ++t) {
      const int64_t mt = h->parts[t].scalar_rows();
      for (int n = 0; n < h->rhs; ++n)
        std::memcpy(C + h->bases[t] + int64_t(n) * h->ldc, outs[t].data() + int64_t(n) * mt,
                    size_t(mt) * sizeof(float));
    }
  return 0;
}

void ref_release(void* handle) { delete static_cast<RefPrepared*>(handle); }
}
