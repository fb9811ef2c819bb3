// vbsr_host.cpp — host side of the engine: last-error bookkeeping, VBSR validation, the seeded
// generators, the counter-based value generator, the multi-GPU row partition and the byte model.
// Nothing here touches a GPU.
#include <algorithm>
#include <cstring>
#include <new>
#include <random>
#include <stdexcept>
#include <thread>

#include "vbsr_internal.h"
#include "vbsr_rng.h"

namespace vbsr_b200 {

namespace {
thread_local std::string g_last_error;
}

vbsr_status set_error(vbsr_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}
void clear_error() { g_last_error.clear(); }

int default_threads(int requested) {
  if (requested > 0) return requested;
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : int(n);
}

// Runs fn(begin, end) over [0, n) split into `threads` contiguous slices.
template <class Fn>
void parallel_for(uint64_t n, int threads, Fn fn) {
  threads = std::max(1, std::min<int>(threads, int(std::max<uint64_t>(1, n / 65536))));
  if (threads == 1) {
    fn(uint64_t(0), n);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t) {
    const uint64_t b = n * uint64_t(t) / uint64_t(threads);
    const uint64_t e = n * uint64_t(t + 1) / uint64_t(threads);
    pool.emplace_back([=] { fn(b, e); });
  }
  for (auto& th : pool) th.join();
}

// The checks of HostMatrix::validate (src/format/vbsr.cpp:29-82), in its order and with its
// messages. `check_values` = false skips only the final "values length" comparison, for
// structure-only views whose values are generated on the device.
vbsr_status validate_view(const vbsr_host_matrix_view* v, bool check_values) {
  if (v == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null matrix view");
  const int R = v->block_rows, S = v->block_cols;
  if (R <= 0 || S <= 0) return set_error(VBSR_INVALID_ARGUMENT, "positive block dimensions required");
  if (v->row_ptr_len != size_t(R) + 1 || v->row_size_len != size_t(R) ||
      v->col_size_len != size_t(S))
    return set_error(VBSR_INVALID_ARGUMENT, "metadata size mismatch");
  if (v->row_scalar_off_len != size_t(R) + 1 || v->col_scalar_off_len != size_t(S) + 1)
    return set_error(VBSR_INVALID_ARGUMENT, "scalar offsets size mismatch");
  if (v->row_ptr == nullptr || v->row_size == nullptr || v->col_size == nullptr ||
      v->row_scalar_off == nullptr || v->col_scalar_off == nullptr || v->value_off == nullptr ||
      (v->block_col_len > 0 && v->block_col == nullptr))
    return set_error(VBSR_INVALID_ARGUMENT, "null metadata array");
  if (v->row_ptr[0] != 0 || v->row_ptr[R] < 0 || size_t(v->row_ptr[R]) != v->block_col_len)
    return set_error(VBSR_INVALID_ARGUMENT, "bad row_ptr");
  const size_t nnzb = v->block_col_len;
  if (v->value_off_len != nnzb + 1 || v->value_off[0] != 0 ||
      (check_values && (v->value_off[nnzb] < 0 || size_t(v->value_off[nnzb]) != v->values_len)))
    return set_error(VBSR_INVALID_ARGUMENT, "bad value offsets");
  if (check_values && v->values_len > 0 && v->values == nullptr)
    return set_error(VBSR_INVALID_ARGUMENT, "bad value offsets");
  for (int i = 0; i < R; ++i) {
    const int h = v->row_size[i];
    if (v->row_ptr[i] > v->row_ptr[i + 1] || h < 8 || h > 64 || h % 8 != 0 ||
        v->row_scalar_off[i + 1] - v->row_scalar_off[i] != h)
      return set_error(VBSR_INVALID_ARGUMENT, "bad block row");
  }
  for (int j = 0; j < S; ++j) {
    const int w = v->col_size[j];
    if (w < 8 || w > 64 || w % 8 != 0 || v->col_scalar_off[j + 1] - v->col_scalar_off[j] != w)
      return set_error(VBSR_INVALID_ARGUMENT, "bad block column");
  }
  // Walk the blocks with one forward row cursor (row_ptr is monotone by the loop above).
  int row = 0;
  for (size_t b = 0; b < nnzb; ++b) {
    while (v->row_ptr[row + 1] <= int64_t(b)) ++row;
    const int c = v->block_col[b];
    if (c < 0 || c >= S) return set_error(VBSR_INVALID_ARGUMENT, "block column out of range");
    if (v->value_off[b + 1] - v->value_off[b] != int64_t(v->row_size[row]) * v->col_size[c])
      return set_error(VBSR_INVALID_ARGUMENT, "block payload mismatch");
  }
  return VBSR_OK;
}

}  // namespace vbsr_b200

using namespace vbsr_b200;

extern "C" {

const char* vbsr_get_last_error(void) { return g_last_error.c_str(); }

vbsr_status vbsr_host_validate(const vbsr_host_matrix_view* host) {
  clear_error();
  return validate_view(host, true);
}

// ---- generators ------------------------------------------------------------------------------

namespace {

// Block size draws. PROFILE_REFERENCE: the reference's tables (generator.cpp:15-30): Uniform is
// the constant 32, LowVariance {24,32,40}, HighVariance all eight sizes, Bimodal {8,16,48,64},
// each drawn as engine() % table size. PROFILE_SPEC: the benchmark specification's
// distributions: uniform over {8..64} (engine() % 8), low-variance 32 w.p. 1/2 and 24/40 w.p.
// 1/4 each (engine() % 4 -> {32,32,24,40}), high-variance {8,16,56,64} w.p. {.3,.2,.2,.3}
// (engine() % 10), bimodal 8/64 w.p. 1/2 (engine() % 2).
int draw_size(std::mt19937_64& eng, int dist, int profile) {
  static const int all8[8] = {8, 16, 24, 32, 40, 48, 56, 64};
  if (profile == VBSR_PROFILE_REFERENCE) {
    static const int low[3] = {24, 32, 40};
    static const int bim[4] = {8, 16, 48, 64};
    switch (dist) {
      case VBSR_DIST_UNIFORM: return 32;
      case VBSR_DIST_LOW_VARIANCE: return low[eng() % 3];
      case VBSR_DIST_HIGH_VARIANCE: return all8[eng() % 8];
      case VBSR_DIST_BIMODAL: return bim[eng() % 4];
    }
    return -1;
  }
  switch (dist) {
    case VBSR_DIST_UNIFORM: return all8[eng() % 8];
    case VBSR_DIST_LOW_VARIANCE: {
      static const int low[4] = {32, 32, 24, 40};
      return low[eng() % 4];
    }
    case VBSR_DIST_HIGH_VARIANCE: {
      const uint64_t r = eng() % 10;
      return r < 3 ? 8 : r < 5 ? 16 : r < 7 ? 56 : 64;
    }
    case VBSR_DIST_BIMODAL: return (eng() % 2) ? 64 : 8;
  }
  return -1;
}

}  // namespace

vbsr_status vbsr_generate(const vbsr_generator_options* o, vbsr_host_matrix** out) {
  clear_error();
  if (o == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  // generator.cpp:8-11
  if (o->degree < 1 || o->degree > 16 || o->block_rows < 1 || o->block_cols < 1 ||
      o->degree > o->block_cols)
    return set_error(VBSR_INVALID_ARGUMENT, "invalid generator dimensions");
  if (o->distribution < 0 || o->distribution > 3)
    return set_error(VBSR_INVALID_ARGUMENT, "unknown block-size distribution");
  if (o->profile != VBSR_PROFILE_REFERENCE && o->profile != VBSR_PROFILE_SPEC)
    return set_error(VBSR_INVALID_ARGUMENT, "unknown generator profile");
  if (o->profile == VBSR_PROFILE_REFERENCE && !o->with_values)
    return set_error(VBSR_INVALID_ARGUMENT, "the reference profile always draws values");
  const int R = o->block_rows, S = o->block_cols, d = o->degree;
  const int window = std::min(17, S);
  if (o->profile == VBSR_PROFILE_SPEC && o->local_columns && d > window)
    return set_error(VBSR_INVALID_ARGUMENT, "invalid generator dimensions");

  auto* m = new (std::nothrow) vbsr_host_matrix;
  if (m == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  try {
    std::mt19937_64 eng(o->seed);
    m->block_rows = R;
    m->block_cols = S;
    m->row_size.resize(R);
    m->col_size.resize(S);
    for (auto& h : m->row_size) h = draw_size(eng, o->distribution, o->profile);
    for (auto& w : m->col_size) w = draw_size(eng, o->distribution, o->profile);
    m->row_scalar_off.resize(size_t(R) + 1);
    m->col_scalar_off.resize(size_t(S) + 1);
    m->row_scalar_off[0] = 0;
    for (int i = 0; i < R; ++i) m->row_scalar_off[i + 1] = m->row_scalar_off[i] + m->row_size[i];
    m->col_scalar_off[0] = 0;
    for (int j = 0; j < S; ++j) m->col_scalar_off[j + 1] = m->col_scalar_off[j] + m->col_size[j];

    m->row_ptr.assign(1, 0);
    m->value_off.assign(1, 0);
    m->row_ptr.reserve(size_t(R) + 1);
    m->block_col.reserve(size_t(R) * d);
    m->value_off.reserve(size_t(R) * d + 1);
    std::vector<int> picked;
    picked.reserve(d);

    if (o->profile == VBSR_PROFILE_REFERENCE) {
      // generator.cpp:40-85: column choice and value draws interleave on one engine.
      std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
      for (int i = 0; i < R; ++i) {
        picked.clear();
        while (int(picked.size()) < d) {
          const int c = o->local_columns ? (i + int(eng() % uint64_t(2 * d + 1)) - d + S) % S
                                         : int(eng() % uint64_t(S));
          if (std::find(picked.begin(), picked.end(), c) == picked.end()) picked.push_back(c);
        }
        std::sort(picked.begin(), picked.end());
        for (int c : picked) {
          m->block_col.push_back(c);
          const int64_t n = int64_t(m->row_size[i]) * m->col_size[c];
          for (int64_t t = 0; t < n; ++t) m->values.push_back(uni(eng));
          m->value_off.push_back(m->value_off.back() + n);
        }
        m->row_ptr.push_back(int(m->block_col.size()));
      }
    } else {
      // Structure first (one engine), then values from the counter-based generator, so the
      // value array is allocated once at its exact size and filled in parallel.
      for (int i = 0; i < R; ++i) {
        picked.clear();
        const int lo = std::clamp(i - 8, 0, S - window);
        while (int(picked.size()) < d) {
          const int c = o->local_columns ? lo + int(eng() % uint64_t(window))
                                         : int(eng() % uint64_t(S));
          if (std::find(picked.begin(), picked.end(), c) == picked.end()) picked.push_back(c);
        }
        std::sort(picked.begin(), picked.end());
        for (int c : picked) {
          m->block_col.push_back(c);
          m->value_off.push_back(m->value_off.back() + int64_t(m->row_size[i]) * m->col_size[c]);
        }
        m->row_ptr.push_back(int(m->block_col.size()));
      }
      if (o->with_values) {
        const uint64_t n = uint64_t(m->value_off.back());
        m->values.resize(n);
        float* dst = m->values.data();
        const uint64_t seed = o->seed;
        parallel_for(n, default_threads(o->threads), [=](uint64_t b, uint64_t e) {
          fill_uniform_range(seed, VBSR_STREAM_VALUES, b, e - b, dst + b);
        });
      }
    }
  } catch (const std::bad_alloc&) {
    delete m;
    return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  }
  vbsr_host_matrix_view v;
  vbsr_host_matrix_view_get(m, &v);
  const vbsr_status s = validate_view(&v, o->with_values != 0);
  if (s != VBSR_OK) {
    delete m;
    return s;
  }
  *out = m;
  return VBSR_OK;
}

vbsr_status vbsr_host_matrix_view_get(const vbsr_host_matrix* h, vbsr_host_matrix_view* v) {
  if (h == nullptr || v == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  v->block_rows = h->block_rows;
  v->block_cols = h->block_cols;
  v->row_ptr = h->row_ptr.data();
  v->row_ptr_len = h->row_ptr.size();
  v->block_col = h->block_col.data();
  v->block_col_len = h->block_col.size();
  v->row_size = h->row_size.data();
  v->row_size_len = h->row_size.size();
  v->col_size = h->col_size.data();
  v->col_size_len = h->col_size.size();
  v->row_scalar_off = h->row_scalar_off.data();
  v->row_scalar_off_len = h->row_scalar_off.size();
  v->col_scalar_off = h->col_scalar_off.data();
  v->col_scalar_off_len = h->col_scalar_off.size();
  v->value_off = h->value_off.data();
  v->value_off_len = h->value_off.size();
  v->values = h->values.empty() ? nullptr : h->values.data();
  v->values_len = h->values.size();
  return VBSR_OK;
}

vbsr_status vbsr_host_matrix_free(vbsr_host_matrix* h) {
  delete h;
  return VBSR_OK;
}

vbsr_status vbsr_fill_uniform(uint64_t seed, uint64_t stream, uint64_t first, uint64_t count,
                              float* out, int threads) {
  clear_error();
  if (count > 0 && out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null output");
  parallel_for(count, default_threads(threads), [=](uint64_t b, uint64_t e) {
    fill_uniform_range(seed, stream, first + b, e - b, out + b);
  });
  return VBSR_OK;
}

vbsr_status vbsr_fill_mt19937(uint32_t seed, uint64_t count, float* out) {
  clear_error();
  if (count > 0 && out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null output");
  std::mt19937 eng{seed};
  std::uniform_real_distribution<float> uni(-1.0f, 1.0f);
  for (uint64_t i = 0; i < count; ++i) out[i] = uni(eng);
  return VBSR_OK;
}

// ---- partition and byte model -----------------------------------------------------------------

vbsr_status vbsr_partition_rows(const vbsr_host_matrix_view* v, int parts, int rhs,
                                int32_t* bounds) {
  clear_error();
  vbsr_status s = validate_view(v, false);
  if (s != VBSR_OK) return s;
  if (parts < 1 || bounds == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "bad partition count");
  const int R = v->block_rows;
  std::vector<double> prefix(size_t(R) + 1, 0.0);
  for (int i = 0; i < R; ++i) {
    double sum_w = 0.0;
    for (int b = v->row_ptr[i]; b < v->row_ptr[i + 1]; ++b) sum_w += v->col_size[v->block_col[b]];
    prefix[i + 1] = prefix[i] + 4.0 * v->row_size[i] * sum_w + 4.0 * rhs * sum_w;
  }
  const double total = prefix[R];
  bounds[0] = 0;
  int r = 0;
  for (int k = 1; k < parts; ++k) {
    const double target = total * k / parts;
    while (r < R && prefix[r] < target) ++r;
    // choose the closer of r-1 and r as the cut
    int cut = r;
    if (r > 0 && target - prefix[r - 1] < prefix[r] - target) cut = r - 1;
    cut = std::max(cut, int(bounds[k - 1]));
    bounds[k] = cut;
  }
  bounds[parts] = R;
  return VBSR_OK;
}

vbsr_status vbsr_compulsory_bytes(const vbsr_host_matrix_view* v, int32_t r0, int32_t r1, int rhs,
                                  double* bytes, double* flops) {
  clear_error();
  vbsr_status s = validate_view(v, false);
  if (s != VBSR_OK) return s;
  if (r0 < 0 || r1 > v->block_rows || r0 > r1)
    return set_error(VBSR_INVALID_ARGUMENT, "bad row range");
  const double nnzb = double(v->row_ptr[r1]) - v->row_ptr[r0];
  const double hw = double(v->value_off[v->row_ptr[r1]] - v->value_off[v->row_ptr[r0]]);
  const double R = r1 - r0, S = v->block_cols;
  const double M = double(v->row_scalar_off[r1] - v->row_scalar_off[r0]);
  const double K = double(v->col_scalar_off[v->block_cols]);
  if (bytes)
    *bytes = 4 * hw + 4 * nnzb + 8 * (nnzb + 1) + 4 * (R + 1) + 4 * R + 8 * (R + 1) + 4 * S +
             8 * (S + 1) + 4 * K * rhs + 4 * M * rhs;
  if (flops) *flops = 2 * hw * rhs;
  return VBSR_OK;
}

}  // extern "C"
