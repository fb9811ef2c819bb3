// vbsr_rng.h — counter-based uniform generator shared by host and device.
//
// u(seed, stream, i) = a float in [-1, 1) that depends only on (seed, stream, i), so any slice of
// a 5-billion-value matrix can be produced independently, in parallel, on the host or on the
// GPU, with bit-identical results. Mixing: the SplitMix64 finaliser (Steele, Lea and Flood,
// "Fast splittable pseudorandom number generators", OOPSLA 2014; the constants of Vigna's
// public-domain splitmix64.c) applied to key + (i+1) * golden-ratio increment, where the key mixes
// seed and stream. The top 24 bits k of the result give (k - 2^23) * 2^-23, which is exact in
// fp32, so host and device agree bit for bit without relying on any float rounding mode.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define VBSR_RNG_HD __host__ __device__ __forceinline__
#else
#define VBSR_RNG_HD inline
#endif

namespace vbsr_b200 {

VBSR_RNG_HD uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

VBSR_RNG_HD uint64_t rng_key(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ mix64(stream + 0x632BE59BD9B4E019ull));
}

VBSR_RNG_HD float rng_uniform(uint64_t key, uint64_t index) {
  const uint64_t z = mix64(key + (index + 1) * 0x9E3779B97F4A7C15ull);
  const int32_t k = int32_t(z >> 40) - (1 << 23);  // [-2^23, 2^23)
  return float(k) * (1.0f / 8388608.0f);           // exact: |k| < 2^24
}

inline void fill_uniform_range(uint64_t seed, uint64_t stream, uint64_t first, uint64_t count,
                               float* out) {
  const uint64_t key = rng_key(seed, stream);
  for (uint64_t i = 0; i < count; ++i) out[i] = rng_uniform(key, first + i);
}

}  // namespace vbsr_b200
