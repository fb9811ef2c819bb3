// cpu_reference.cpp — TEST INFRASTRUCTURE ONLY. Definition of vbsr::cpu_reference for the C++
// drop-in header (include/varblockspmm/vbsr.hpp), backed by the oracle restatement
// vbsr_oracle.c. It is built into oracle/_build/libvbsr_oracle.so, never into the product
// library: the engine's execute path has no CPU implementation to fall back on.
#include <stdexcept>
#include <thread>
#include <vector>

#include "varblockspmm/vbsr.hpp"

extern "C" int vbsr_oracle_spmm(const vbsr_host_matrix_view* v, const float* B, int rhs,
                                int32_t r0, int32_t r1, float* C, double* S, int threads);

namespace vbsr {
// reference: src/format/vbsr.cpp:167-201 (same size check and message)
std::vector<float> cpu_reference(const HostMatrix& m, const std::vector<float>& input, int rhs) {
  if (input.size() != size_t(m.scalar_cols() * rhs)) throw std::invalid_argument("B size");
  std::vector<float> out(size_t(m.scalar_rows() * rhs), 0.0f);
  const vbsr_host_matrix_view v = detail::view_of(m);
  const unsigned hc = std::thread::hardware_concurrency();
  if (vbsr_oracle_spmm(&v, input.data(), rhs, 0, m.block_rows, out.data(), nullptr,
                       hc == 0 ? 1 : int(hc)) != 0)
    throw std::invalid_argument("cpu_reference: invalid matrix or rhs width");
  return out;
}
}  // namespace vbsr
