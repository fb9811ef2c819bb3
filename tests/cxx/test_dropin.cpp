// test_dropin.cpp — the C++ drop-in API (include/varblockspmm/vbsr.hpp, libvbsr_b200_cxx.so) driven
// the way the reference's own test binary drives the reference (tests/test_main.cpp:14-177):
//   * the 64-case parameter matrix (4 distributions x degrees {1,4,8,16} x RHS {8,16,32,64}, 9 x 17
//     block matrices from the reference-profile generate(), seeds 11.., local pattern on odd
//     seeds), each on a non-default stream through Plan (Kernel::RowOwned), launch_row_owned_scalar,
//     ScalarCsrPlan and GroupedGemmPlan, against cpu_reference with the reference test's acceptance
//     check (finite, max |err| <= 5e-4, relative L2 error <= 5e-5);
//   * the negative tests: malformed row_ptr and block size rejected by validate(), RHS 7 and
//     Kernel::SplitRow rejected by Plan, each as std::invalid_argument.
// Beyond the reference's test: Kernel::Auto, a moved-from Matrix, and one const Plan executed on
// two streams with different B at once. Exit status 0 and "PASS" on success.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <string>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "varblockspmm/vbsr.hpp"

namespace {

void cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// The reference test's dense input: std::mt19937(seed) through uniform_real_distribution(-1, 1).
std::vector<float> dense_input(int64_t n, uint64_t seed) {
  std::vector<float> v(static_cast<size_t>(n));
  std::mt19937 eng{unsigned(seed)};
  std::uniform_real_distribution<float> u(-1.0f, 1.0f);
  for (float& x : v) x = u(eng);
  return v;
}

struct DeviceBuffer {
  float* p = nullptr;
  size_t n = 0;
  explicit DeviceBuffer(size_t count) : n(count) {
    cuda(cudaMalloc(&p, std::max<size_t>(1, n) * sizeof(float)), "cudaMalloc");
  }
  ~DeviceBuffer() { cudaFree(p); }
  void upload(const std::vector<float>& h) {
    cuda(cudaMemcpy(p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice), "upload");
  }
  void poison(cudaStream_t s) { cuda(cudaMemsetAsync(p, 0xff, n * sizeof(float), s), "memset"); }
  std::vector<float> download() const {
    std::vector<float> h(n);
    cuda(cudaMemcpy(h.data(), p, n * sizeof(float), cudaMemcpyDeviceToHost), "download");
    return h;
  }
};

// The reference test's acceptance check (test_main.cpp:14-40).
void accept(const std::vector<float>& ref, const std::vector<float>& got, const std::string& who) {
  double max_err = 0.0, err2 = 0.0, ref2 = 0.0;
  for (size_t i = 0; i < ref.size(); ++i) {
    if (!std::isfinite(got[i])) throw std::runtime_error(who + " produced NaN/Inf");
    const double e = double(got[i]) - double(ref[i]);
    max_err = std::max(max_err, std::fabs(e));
    err2 += e * e;
    ref2 += double(ref[i]) * double(ref[i]);
  }
  const double rel = std::sqrt(err2 / (ref2 + 1e-30));
  if (max_err > 5e-4 || rel > 5e-5)
    throw std::runtime_error(who + " mismatch: max=" + std::to_string(max_err) +
                             " rel=" + std::to_string(rel));
}

int checks = 0;

void run_and_check(const std::function<void(cudaStream_t)>& run, cudaStream_t s, DeviceBuffer& out,
                   const std::vector<float>& ref, const std::string& who) {
  out.poison(s);  // every output element must be written by the path under test
  run(s);
  cuda(cudaStreamSynchronize(s), "sync");
  accept(ref, out.download(), who);
  ++checks;
}

void one_case(vbsr::Distribution dist, int degree, int rhs, bool local, uint64_t seed) {
  vbsr::GeneratorOptions o;
  o.block_rows = 9;
  o.block_cols = 17;
  o.degree = degree;
  o.distribution = dist;
  o.local_columns = local;
  o.seed = seed;
  const vbsr::HostMatrix host = vbsr::generate(o);
  const std::vector<float> B = dense_input(host.scalar_cols() * rhs, seed);
  const std::vector<float> ref = vbsr::cpu_reference(host, B, rhs);

  vbsr::Matrix matrix(host);
  DeviceBuffer dB(B.size()), dC(ref.size());
  dB.upload(B);
  cudaStream_t s;
  cuda(cudaStreamCreate(&s), "stream");
  const std::string tag = " (seed " + std::to_string(seed) + ", rhs " + std::to_string(rhs) + ")";
  vbsr::Plan direct(matrix, {rhs, vbsr::Kernel::RowOwned});
  vbsr::Plan automatic(matrix, {rhs, vbsr::Kernel::Auto});
  vbsr::ScalarCsrPlan csr(host, rhs);
  vbsr::GroupedGemmPlan grouped(host, rhs);
  run_and_check([&](cudaStream_t st) { direct.execute(dB.p, dC.p, st); }, s, dC, ref,
                "Plan(RowOwned)" + tag);
  run_and_check([&](cudaStream_t st) { automatic.execute(dB.p, dC.p, st); }, s, dC, ref,
                "Plan(Auto)" + tag);
  run_and_check(
      [&](cudaStream_t st) {
        vbsr::launch_row_owned_scalar(matrix.device_view(), dB.p, dC.p, rhs, st);
      },
      s, dC, ref, "launch_row_owned_scalar" + tag);
  run_and_check(
      [&](cudaStream_t st) {
        vbsr::launch_row_owned(matrix.device_view(), nullptr, 0, 0, dB.p, dC.p, rhs, st);
      },
      s, dC, ref, "launch_row_owned" + tag);
  run_and_check([&](cudaStream_t st) { csr.execute(dB.p, dC.p, st); }, s, dC, ref,
                "ScalarCsrPlan" + tag);
  run_and_check([&](cudaStream_t st) { grouped.execute(dB.p, dC.p, st); }, s, dC, ref,
                "GroupedGemmPlan" + tag);
  if (direct.launch_count() < 1 || grouped.launch_count() < 1)
    throw std::runtime_error("launch_count" + tag);
  cuda(cudaStreamDestroy(s), "stream destroy");
}

void expect_invalid(const std::function<void()>& f, const char* what) {
  try {
    f();
  } catch (const std::invalid_argument&) {
    ++checks;
    return;
  }
  throw std::runtime_error(std::string("not rejected with std::invalid_argument: ") + what);
}

void negative_cases() {
  vbsr::GeneratorOptions o;
  o.block_rows = 4;
  o.block_cols = 4;
  o.degree = 2;
  const vbsr::HostMatrix good = vbsr::generate(o);
  vbsr::HostMatrix bad = good;
  bad.row_ptr.back() += 1;
  expect_invalid([&] { bad.validate(); }, "malformed row_ptr");
  bad = good;
  bad.row_size[0] = 7;
  expect_invalid([&] { bad.validate(); }, "block size 7");
  vbsr::Matrix m(good);
  expect_invalid([&] { vbsr::Plan p(m, {7, vbsr::Kernel::RowOwned}); }, "RHS 7");
  expect_invalid([&] { vbsr::Plan p(m, {8, vbsr::Kernel::SplitRow}); }, "Kernel::SplitRow");
  expect_invalid([&] { vbsr::ScalarCsrPlan p(good, 12); }, "ScalarCsrPlan RHS 12");
  expect_invalid([&] { vbsr::GroupedGemmPlan p(good, 3); }, "GroupedGemmPlan RHS 3");
}

// A moved Matrix keeps working; one const Plan on two streams with different B at once.
void ownership_and_streams() {
  vbsr::GeneratorOptions o;
  o.block_rows = 300;
  o.block_cols = 300;
  o.degree = 8;
  o.distribution = vbsr::Distribution::HighVariance;
  o.local_columns = false;
  o.seed = 5;
  const vbsr::HostMatrix host = vbsr::generate(o);
  const int rhs = 32;
  vbsr::Matrix first(host);
  vbsr::Matrix matrix(std::move(first));
  const vbsr::Plan plan(matrix, {rhs, vbsr::Kernel::Auto});
  std::vector<std::vector<float>> Bs = {dense_input(host.scalar_cols() * rhs, 1),
                                        dense_input(host.scalar_cols() * rhs, 2)};
  DeviceBuffer b0(Bs[0].size()), b1(Bs[1].size());
  b0.upload(Bs[0]);
  b1.upload(Bs[1]);
  const size_t nc = size_t(host.scalar_rows()) * rhs;
  DeviceBuffer c0(nc), c1(nc);
  cudaStream_t s0, s1;
  cuda(cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking), "stream");
  cuda(cudaStreamCreateWithFlags(&s1, cudaStreamNonBlocking), "stream");
  c0.poison(s0);
  c1.poison(s1);
  for (int i = 0; i < 3; ++i) {
    plan.execute(b0.p, c0.p, s0);
    plan.execute(b1.p, c1.p, s1);
  }
  cuda(cudaStreamSynchronize(s0), "sync");
  cuda(cudaStreamSynchronize(s1), "sync");
  accept(vbsr::cpu_reference(host, Bs[0], rhs), c0.download(), "stream 0 of one plan");
  accept(vbsr::cpu_reference(host, Bs[1], rhs), c1.download(), "stream 1 of one plan");
  checks += 2;
  cudaStreamDestroy(s0);
  cudaStreamDestroy(s1);
}

// A small scalar CSR matrix through from_csr, the VBSR file and back, then Plan::execute.
void csr_and_file(const char* dir) {
  const int64_t rows = 48, cols = 40;
  std::vector<int64_t> row_ptr{0}, col_idx;
  std::vector<float> vals;
  std::mt19937 eng{3};
  std::uniform_real_distribution<float> u(-1.0f, 1.0f);
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c)
      if ((r * 7 + c * 3) % 11 == 0) {
        col_idx.push_back(c);
        vals.push_back(u(eng));
      }
    row_ptr.push_back(int64_t(col_idx.size()));
  }
  const vbsr::HostMatrix a = vbsr::from_csr(rows, cols, row_ptr, col_idx, vals, {16, 32}, {8, 32});
  const std::string path = std::string(dir) + "/dropin_test.vbsr";
  vbsr::save_matrix(a, path.c_str());
  const vbsr::HostMatrix b = vbsr::load_matrix(path.c_str());
  std::remove(path.c_str());
  if (b.values != a.values || b.block_col != a.block_col || b.value_off != a.value_off)
    throw std::runtime_error("VBSR file round trip changed the matrix");
  const int rhs = 16;
  const std::vector<float> B = dense_input(cols * rhs, 4);
  vbsr::Matrix m(b);
  vbsr::Plan plan(m, {rhs, vbsr::Kernel::Auto});
  DeviceBuffer dB(B.size()), dC(size_t(rows) * rhs);
  dB.upload(B);
  cudaStream_t s;
  cuda(cudaStreamCreate(&s), "stream");
  run_and_check([&](cudaStream_t st) { plan.execute(dB.p, dC.p, st); }, s, dC,
                vbsr::cpu_reference(b, B, rhs), "from_csr + file + Plan");
  cudaStreamDestroy(s);
  expect_invalid([&] { vbsr::load_matrix((std::string(dir) + "/missing.vbsr").c_str()); },
                 "missing VBSR file");
}

}  // namespace

int main(int argc, char** argv) {
  try {
    negative_cases();
    const vbsr::Distribution dists[] = {vbsr::Distribution::Uniform,
                                        vbsr::Distribution::LowVariance,
                                        vbsr::Distribution::HighVariance,
                                        vbsr::Distribution::Bimodal};
    uint64_t seed = 11;
    for (vbsr::Distribution d : dists)
      for (int degree : {1, 4, 8, 16})
        for (int rhs : {8, 16, 32, 64}) {
          one_case(d, degree, rhs, (seed & 1) != 0, seed);
          ++seed;
        }
    ownership_and_streams();
    csr_and_file(argc > 1 ? argv[1] : ".");
    std::printf("PASS: %d checks (64 parameter cases x 6 paths on non-default streams, negative "
                "cases, moved Matrix, one plan on two streams)\n", checks);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "FAIL: %s\n", e.what());
    return 1;
  }
}
