// workload.cpp — TEST INFRASTRUCTURE ONLY. The benchmark workloads' inputs, generated without the
// engine library, so that bench.py's reference arm (which times the reference's own CPU path) never
// loads the product. Two pieces, each restated independently of the engine's code and pinned
// against it by tests/test_oracle_golden.py:
//   * oracle_fill_uniform: the counter-based U[-1,1) stream of the benchmark inputs. Value i of
//     (seed, stream) is SplitMix64's output function (Steele, Lea and Flood, OOPSLA 2014; the
//     constants of Vigna's public-domain splitmix64.c) applied to key + (i + 1) * 0x9E3779B97F4A7C15,
//     key = mix(seed ^ mix(stream + 0x632BE59BD9B4E019)); its top 24 bits k map to (k - 2^23) / 2^23.
//   * oracle_spec_structure: the block structure of the benchmark specification's generator
//     std::mt19937_64(seed) draws every block-row height, then every
//     block-column width, then per block row `degree` distinct columns (uniform over all columns,
//     or over the 17-wide window starting at clamp(i - 8, 0, S - 17) for the local pattern),
//     redrawing repeats, sorted. Size tables: uniform {8..64} (draw % 8), low-variance
//     {32,32,24,40}[draw % 4], high-variance {8,16,56,64} w.p. {.3,.2,.2,.3} (draw % 10),
//     bimodal draw % 2 ? 64 : 8.
#include <algorithm>
#include <cstdint>
#include <random>
#include <thread>
#include <vector>

namespace {
uint64_t mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

int spec_size(std::mt19937_64& eng, int dist) {
  switch (dist) {
    case 0: return 8 * int(eng() % 8 + 1);
    case 1: {
      const int t[4] = {32, 32, 24, 40};
      return t[eng() % 4];
    }
    case 2: {
      const uint64_t r = eng() % 10;
      return r < 3 ? 8 : (r < 5 ? 16 : (r < 7 ? 56 : 64));
    }
    case 3: return (eng() % 2) ? 64 : 8;
  }
  return -1;
}
}  // namespace

extern "C" {

int oracle_fill_uniform(uint64_t seed, uint64_t stream, uint64_t first, uint64_t count, float* out,
                        int threads) {
  const uint64_t key = mix(seed ^ mix(stream + 0x632BE59BD9B4E019ull));
  if (threads < 1) threads = 1;
  if (uint64_t(threads) > count / 65536 + 1) threads = int(count / 65536 + 1);
  auto work = [=](uint64_t a, uint64_t b) {
    for (uint64_t i = a; i < b; ++i) {
      const uint64_t z = mix(key + (first + i + 1) * 0x9E3779B97F4A7C15ull);
      out[i] = float(int32_t(z >> 40) - (1 << 23)) * (1.0f / 8388608.0f);
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t)
    pool.emplace_back(work, count * t / threads, count * (t + 1) / threads);
  work(0, count / threads);
  for (auto& th : pool) th.join();
  return 0;
}

// Fills row_size[R], col_size[S] and block_col[R * degree] (sorted per row). Returns 0, or -1 for
// arguments the generator rejects.
int oracle_spec_structure(int R, int S, int degree, int dist, int local, uint64_t seed,
                          int32_t* row_size, int32_t* col_size, int32_t* block_col) {
  const int window = S < 17 ? S : 17;
  if (R < 1 || S < 1 || degree < 1 || degree > 16 || degree > S || dist < 0 || dist > 3) return -1;
  if (local && degree > window) return -1;
  std::mt19937_64 eng(seed);
  for (int i = 0; i < R; ++i) row_size[i] = spec_size(eng, dist);
  for (int j = 0; j < S; ++j) col_size[j] = spec_size(eng, dist);
  std::vector<int> picked;
  for (int i = 0; i < R; ++i) {
    picked.clear();
    const int lo = std::clamp(i - 8, 0, S - window);
    while (int(picked.size()) < degree) {
      const int c = local ? lo + int(eng() % uint64_t(window)) : int(eng() % uint64_t(S));
      if (std::find(picked.begin(), picked.end(), c) == picked.end()) picked.push_back(c);
    }
    std::sort(picked.begin(), picked.end());
    std::copy(picked.begin(), picked.end(), block_col + int64_t(i) * degree);
  }
  return 0;
}
}
