// vbsr_device.cu — device side of the engine: the owning device format (Matrix), the planner
// (Plan), the execute path and the C-ABI entry points that touch a GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <new>
#include <numeric>
#include <queue>
#include <string>
#include <thread>
#include <vector>

#include "vbsr_internal.h"
#include "vbsr_kernels_common.cuh"
#include "vbsr_tc.cuh"
#include "vbsr_rng.h"
#include "vbsr_tiles.h"

namespace vbsr_b200 {
vbsr_status validate_view(const vbsr_host_matrix_view* v, bool check_values);
}

using namespace vbsr_b200;

namespace {

// ---- error helpers -------------------------------------------------------------------------------

#define VBSR_CUDA(call)                                                          \
  do {                                                                           \
    const cudaError_t e_ = (call);                                               \
    if (e_ != cudaSuccess) return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e_)); \
  } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (dev >= 0 && dev != prev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// ---- format kernels ------------------------------------------------------------------------------

// Row of block b (binary search over the matrix-local row_ptr).
__device__ __forceinline__ int block_row_of(const int32_t* row_ptr, int rows, int b) {
  int lo = 0, hi = rows;  // row_ptr[lo] <= b < row_ptr[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (row_ptr[mid] <= b) lo = mid; else hi = mid;
  }
  return lo;
}

// Re-lays blocks [b_begin, b_end) from the reference layout (column-major h x w, element (r,k) at
// r + k*h) into the device format (blk_pos). `src` holds values starting at value offset src_base.
__global__ void relayout_blocks(const int32_t* row_ptr, int rows, const int32_t* row_size,
                                const int64_t* value_off, const uint32_t* blk, int b_begin,
                                const float* src, long long src_base, float* dst) {
  const int b = b_begin + int(blockIdx.x);
  const int h = row_size[block_row_of(row_ptr, rows, b)];
  const int w = int((blk[b] & 7u) + 1u) * 8;
  const long long vo = value_off[b];
  const float* s = src + (vo - src_base);
  float* d = dst + vo;
  for (int i = threadIdx.x; i < h * w; i += blockDim.x) {
    const int r = i % h, k = i / h;
    d[blk_pos(h, w, r, k)] = s[i];
  }
}

// Fills blocks in the device format with the counter-based generator: the element at reference
// (packed) position global_base + value_off[b] + r + k*h gets rng_uniform(key, that position).
__global__ void generate_blocks(const int32_t* row_ptr, int rows, const int32_t* row_size,
                                const int64_t* value_off, const uint32_t* blk, int nnzb,
                                uint64_t key, long long global_base, float* dst) {
  for (int b = blockIdx.x; b < nnzb; b += gridDim.x) {
    const int h = row_size[block_row_of(row_ptr, rows, b)];
    const int w = int((blk[b] & 7u) + 1u) * 8;
    const long long vo = value_off[b];
    for (int i = threadIdx.x; i < h * w; i += blockDim.x) {
      const int r = i % h, k = i / h;
      dst[vo + blk_pos(h, w, r, k)] = rng_uniform(key, uint64_t(global_base + vo + i));
    }
  }
}

__global__ void fill_uniform_kernel(uint64_t key, uint64_t first, uint64_t count, float* out) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
    out[i] = rng_uniform(key, first + i);
}

// ---- raw launchers (reference launch_row_owned / launch_row_owned_scalar) --------------------------

__device__ __forceinline__ float block_value(const float* blockv, int h, int w, int r, int k) {
  return blockv[blk_pos(h, w, r, k)];
}

// One output element per thread; grid (block_rows, ceil(64*rhs/256)).
__global__ void rowwise_scalar_kernel(vbsr_device_matrix a, const float* __restrict__ B,
                                      float* __restrict__ C, int rhs) {
  const int row = blockIdx.x;
  const int h = a.row_size[row];
  for (int idx = blockIdx.y * blockDim.x + threadIdx.x; idx < h * rhs;
       idx += blockDim.x * gridDim.y) {
    const int r = idx % h, n = idx / h;
    float acc = 0.0f;
    for (int b = a.row_ptr[row]; b < a.row_ptr[row + 1]; ++b) {
      const int c = a.block_col[b];
      const int w = a.col_size[c];
      const float* av = a.values + a.value_off[b];
      const float* bv = B + a.col_scalar_off[c] + (long long)n * a.scalar_cols;
      float part = 0.0f;
      for (int k = 0; k < w; ++k) part = fmaf(block_value(av, h, w, r, k), bv[k], part);
      acc += part;
    }
    C[a.row_scalar_off[row] + r + (long long)n * a.scalar_rows] = acc;
  }
}

// One CTA per block row, 256 threads; thread = (local row, group of 8 RHS columns), B read through
// the read-only cache. Used where no plan exists (a bare device view) and for B/C pointers that
// are not 16-byte aligned.
__global__ void rowwise_direct_kernel(vbsr_device_matrix a, const float* __restrict__ B,
                                      float* __restrict__ C, int rhs) {
  const int row = blockIdx.x;
  const int h = a.row_size[row];
  const int groups = rhs / 8;
  for (int idx = threadIdx.x; idx < h * groups; idx += blockDim.x) {
    const int r = idx % h, n0 = (idx / h) * 8;
    float acc[8] = {};
    for (int b = a.row_ptr[row]; b < a.row_ptr[row + 1]; ++b) {
      const int c = a.block_col[b];
      const int w = a.col_size[c];
      const float* av = a.values + a.value_off[b];
      const float* bv = B + a.col_scalar_off[c] + (long long)n0 * a.scalar_cols;
      float part[8] = {};
      for (int k = 0; k < w; ++k) {
        const float x = block_value(av, h, w, r, k);
#pragma unroll
        for (int j = 0; j < 8; ++j) part[j] = fmaf(x, __ldg(bv + k + (long long)j * a.scalar_cols), part[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += part[j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      C[a.row_scalar_off[row] + r + (long long)(n0 + j) * a.scalar_rows] = acc[j];
  }
}

bool valid_rhs(int rhs) { return rhs == 8 || rhs == 16 || rhs == 32 || rhs == 64; }

// A private non-blocking stream for the copies and kernels that build a matrix or a plan. Its work
// is ordered only by itself, and finish() waits for exactly that work, so creation neither waits
// for nor stalls other streams of the device (a legacy-stream cudaMemcpy from pageable memory or
// cudaMemset may still be in flight when it returns, so creation does not use those).
struct SetupStream {
  cudaStream_t s = nullptr;
  cudaError_t init() { return cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking); }
  cudaError_t finish() { return s ? cudaStreamSynchronize(s) : cudaSuccess; }
  ~SetupStream() {
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  }
};

template <class T>
vbsr_status upload(T** dst, const T* src, size_t n, int64_t* bytes, cudaStream_t s) {
  *dst = nullptr;
  if (n == 0) return VBSR_OK;
  VBSR_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), n * sizeof(T)));
  *bytes += int64_t(n * sizeof(T));
  if (src != nullptr)
    VBSR_CUDA(cudaMemcpyAsync(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice, s));
  return VBSR_OK;
}

void release(MatrixData& d) {
  cudaFree(d.d_row_ptr);
  cudaFree(d.d_block_col);
  cudaFree(d.d_row_size);
  cudaFree(d.d_col_size);
  cudaFree(d.d_row_off);
  cudaFree(d.d_col_off);
  cudaFree(d.d_value_off);
  cudaFree(d.d_values);
  cudaFree(d.d_blk_desc);
  d.d_row_ptr = d.d_block_col = d.d_row_size = d.d_col_size = nullptr;
  d.d_row_off = d.d_col_off = d.d_value_off = nullptr;
  d.d_values = nullptr;
  d.d_blk_desc = nullptr;
}

// Uploads the packed host values of a matrix (blocks [0, nnzb), `src` = its first value, voff the
// matrix-local value offsets) into d.d_values in the device format. Pipelined in slices of whole
// blocks (up to kSliceFloats values): host threads copy slice s into pinned staging buffer s % 2,
// the copy stream moves it to device staging buffer s % 2, and the relayout stream re-lays it out
// into d_values, so the host copy of slice s+1, the PCIe transfer of slice s and the relayout of
// slice s-1 overlap. Waits only on its own streams and events (no device-wide synchronisation).
vbsr_status upload_values(MatrixData& d, const float* src, const std::vector<int64_t>& voff) {
  constexpr int64_t kSliceFloats = int64_t(1) << 26;  // 256 MiB
  const int64_t cap = std::min<int64_t>(d.nvalues, kSliceFloats);
  float* hstage[2] = {nullptr, nullptr};
  float* dstage[2] = {nullptr, nullptr};
  cudaStream_t copy_s = nullptr, lay_s = nullptr;
  cudaEvent_t copied[2] = {nullptr, nullptr}, laid[2] = {nullptr, nullptr};
  cudaError_t e = cudaSuccess;
  auto ok = [&](cudaError_t x) {
    if (e == cudaSuccess) e = x;
    return e == cudaSuccess;
  };
  for (int i = 0; i < 2; ++i) {
    ok(cudaHostAlloc(reinterpret_cast<void**>(&hstage[i]), size_t(cap) * sizeof(float),
                     cudaHostAllocDefault));
    ok(cudaMalloc(&dstage[i], size_t(cap) * sizeof(float)));
    ok(cudaEventCreateWithFlags(&copied[i], cudaEventDisableTiming));
    ok(cudaEventCreateWithFlags(&laid[i], cudaEventDisableTiming));
  }
  ok(cudaStreamCreateWithFlags(&copy_s, cudaStreamNonBlocking));
  ok(cudaStreamCreateWithFlags(&lay_s, cudaStreamNonBlocking));
  const unsigned hc = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  int64_t b = 0;
  for (int s = 0; e == cudaSuccess && b < d.nnzb; ++s) {
    const int k = s & 1;
    int64_t be = b;
    while (be < d.nnzb && voff[be + 1] - voff[b] <= cap) ++be;
    const int64_t n = voff[be] - voff[b];
    // staging pair k was last used by slice s-2: its transfer must have read the pinned buffer
    if (s >= 2 && !ok(cudaEventSynchronize(copied[k]))) break;
    {
      const float* from = src + voff[b];
      float* to = hstage[k];
      std::vector<std::thread> pool;
      for (unsigned t = 1; t < hc; ++t)
        pool.emplace_back([=] {
          const int64_t a0 = n * t / hc, a1 = n * (t + 1) / hc;
          std::memcpy(to + a0, from + a0, size_t(a1 - a0) * sizeof(float));
        });
      std::memcpy(to, from, size_t(n / hc) * sizeof(float));
      for (auto& th : pool) th.join();
    }
    // ... and its relayout must have read the device staging buffer
    if (s >= 2 && !ok(cudaStreamWaitEvent(copy_s, laid[k], 0))) break;
    if (!ok(cudaMemcpyAsync(dstage[k], hstage[k], size_t(n) * sizeof(float),
                            cudaMemcpyHostToDevice, copy_s)))
      break;
    if (!ok(cudaEventRecord(copied[k], copy_s))) break;
    if (!ok(cudaStreamWaitEvent(lay_s, copied[k], 0))) break;
    relayout_blocks<<<unsigned(be - b), 256, 0, lay_s>>>(d.d_row_ptr, d.block_rows, d.d_row_size,
                                                        d.d_value_off, d.d_blk_desc, int(b),
                                                        dstage[k], voff[b], d.d_values);
    if (!ok(cudaGetLastError())) break;
    if (!ok(cudaEventRecord(laid[k], lay_s))) break;
    b = be;
  }
  if (copy_s) ok(cudaStreamSynchronize(copy_s));
  if (lay_s) ok(cudaStreamSynchronize(lay_s));
  for (int i = 0; i < 2; ++i) {
    cudaFreeHost(hstage[i]);
    cudaFree(dstage[i]);
    if (copied[i]) cudaEventDestroy(copied[i]);
    if (laid[i]) cudaEventDestroy(laid[i]);
  }
  if (copy_s) cudaStreamDestroy(copy_s);
  if (lay_s) cudaStreamDestroy(lay_s);
  if (e != cudaSuccess) return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e));
  return VBSR_OK;
}

// Builds the device format of block rows [r0, r1). mode 0: values from host; 1: generated.
vbsr_status build_matrix(const vbsr_host_matrix_view* v, int r0, int r1, int mode, uint64_t seed,
                         int device, vbsr_matrix** out) {
  if (out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  vbsr_status st = validate_view(v, mode == 0);
  if (st != VBSR_OK) return st;
  if (r0 < 0 || r1 > v->block_rows || r0 >= r1)
    return set_error(VBSR_INVALID_ARGUMENT, "bad block-row range");
  const int64_t K = v->col_scalar_off[v->block_cols];
  if (K >= (int64_t(1) << 31) - 64)
    return set_error(VBSR_INVALID_ARGUMENT, "scalar column count exceeds the engine's 2^31 limit");
  if (v->row_scalar_off[v->block_rows] >= (int64_t(1) << 31))
    return set_error(VBSR_INVALID_ARGUMENT, "scalar row count exceeds the engine's 2^31 limit");

  auto* m = new (std::nothrow) vbsr_matrix;
  if (m == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  MatrixData& d = m->d;
  int dev = device;
  if (dev < 0) cudaGetDevice(&dev);
  DeviceGuard guard(dev);
  d.device = dev;
  const int R = r1 - r0, S = v->block_cols;
  const int b0 = v->row_ptr[r0], b1 = v->row_ptr[r1];
  const int64_t v0 = v->value_off[b0], v1 = v->value_off[b1];
  d.block_rows = R;
  d.block_cols = S;
  d.row_begin = r0;
  d.row_end = r1;
  d.nnzb = b1 - b0;
  d.M = v->row_scalar_off[r1] - v->row_scalar_off[r0];
  d.K = K;
  d.nvalues = v1 - v0;

  try {
    d.h_row_ptr.resize(size_t(R) + 1);
    d.h_row_size.assign(v->row_size + r0, v->row_size + r1);
    d.h_row_off.resize(size_t(R) + 1);
    d.h_val_off_row.resize(R);
    d.h_sum_w.resize(R);
    for (int i = 0; i <= R; ++i) {
      d.h_row_ptr[i] = v->row_ptr[r0 + i] - b0;
      d.h_row_off[i] = v->row_scalar_off[r0 + i] - v->row_scalar_off[r0];
    }
    std::vector<int64_t> voff(size_t(d.nnzb) + 1);
    std::vector<uint32_t>& desc = d.h_blk_desc;
    desc.resize(d.nnzb);
    for (int64_t b = 0; b <= d.nnzb; ++b) voff[b] = v->value_off[b0 + b] - v0;
    for (int64_t b = 0; b < d.nnzb; ++b) {
      const int c = v->block_col[b0 + b];
      desc[b] = pack_block(v->col_scalar_off[c], v->col_size[c]);
    }
    for (int i = 0; i < R; ++i) {
      d.h_val_off_row[i] = voff[d.h_row_ptr[i]];
      int64_t sw = 0;
      for (int b = d.h_row_ptr[i]; b < d.h_row_ptr[i + 1]; ++b) sw += v->col_size[v->block_col[b0 + b]];
      d.h_sum_w[i] = sw;
    }

    int64_t bytes = 0;
    SetupStream ss;
    if (ss.init() != cudaSuccess) {
      delete m;
      return set_error(VBSR_CUDA_ERROR, "stream creation failed");
    }
#define VBSR_TRY(x)          \
  do {                       \
    st = (x);                \
    if (st != VBSR_OK) {     \
      release(d);            \
      delete m;              \
      return st;             \
    }                        \
  } while (0)
    VBSR_TRY(upload(&d.d_row_ptr, d.h_row_ptr.data(), d.h_row_ptr.size(), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_block_col, v->block_col + b0, size_t(d.nnzb), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_row_size, d.h_row_size.data(), d.h_row_size.size(), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_col_size, v->col_size, size_t(S), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_row_off, d.h_row_off.data(), d.h_row_off.size(), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_col_off, v->col_scalar_off, size_t(S) + 1, &bytes, ss.s));
    VBSR_TRY(upload(&d.d_value_off, voff.data(), voff.size(), &bytes, ss.s));
    VBSR_TRY(upload(&d.d_blk_desc, desc.data(), desc.size(), &bytes, ss.s));
    VBSR_TRY(upload<float>(&d.d_values, nullptr, size_t(d.nvalues), &bytes, ss.s));

    VBSR_TRY(ss.finish() == cudaSuccess ? VBSR_OK
                                        : set_error(VBSR_CUDA_ERROR, "metadata upload failed"));
    if (d.nnzb > 0 && mode == 0) {
      st = upload_values(d, v->values + v0, voff);
      if (st != VBSR_OK) {
        release(d);
        delete m;
        return st;
      }
    } else if (d.nnzb > 0) {
      generate_blocks<<<4096, 256, 0, ss.s>>>(d.d_row_ptr, R, d.d_row_size, d.d_value_off,
                                              d.d_blk_desc, int(d.nnzb),
                                              rng_key(seed, VBSR_STREAM_VALUES), v0, d.d_values);
      cudaError_t e2 = cudaGetLastError();
      if (e2 == cudaSuccess) e2 = ss.finish();
      if (e2 != cudaSuccess) {
        release(d);
        delete m;
        return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e2));
      }
    }
#undef VBSR_TRY
    d.device_bytes = bytes;
  } catch (const std::bad_alloc&) {
    release(d);
    delete m;
    return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  }
  *out = m;
  return VBSR_OK;
}

}  // namespace

// ---- plan ------------------------------------------------------------------------------------------

struct vbsr_plan {
  const vbsr_matrix* m = nullptr;
  int rhs = 32;
  uint32_t flags = 0;
  int device = 0;
  int num_tasks = 0;
  int smem_bytes = 0;
  int64_t stream_entries = 0;
  StageDesc* d_stream = nullptr;
  ItemDesc* d_items = nullptr;
  float* d_bstack = nullptr;     // B's operand stacks, rewritten by every execute
  bool raw_b = false;            // column-stacked form: raw-B stacks (see stack_rows)
  bool direct_b = false;         // ... read from B by the SpMM itself: no pre-pass, no d_bstack
  bool fused_stack = false;      // the SpMM's CTAs form the stacks (no separate pre-pass launch)
  uint32_t* d_stack_flag = nullptr;  // their grid arrival word (stack_arrive)
  int64_t bstack_floats = 0;
  Task* d_tasks = nullptr;
  CcItem* d_cc = nullptr;          // short block rows computed on the CUDA cores (pre-pass launch)
  int cc_count = 0;
  vbsr_plan_work work{};
  int* d_status = nullptr;
  unsigned long long* d_timing = nullptr;  // allocated on first request
  bool timing_on = false;
  int drop_stage = -1;
  long long wait_limit = 4000000000ll;  // ~2 s at 1.965 GHz
  std::string summary;
  std::vector<int> task_warps;      // team size of every task
  std::vector<double> task_cost;    // planner's cost model: the task's most loaded team
  int split_rows = 0;               // block rows cut into row parts
  int work_items = 0;               // items (block rows and row parts)
  // Every execute writes the operand stacks into d_bstack and the SpMM reads them, so two executes
  // of one plan must not overlap on the GPU. Each execute waits (cudaStreamWaitEvent) for the
  // completion event of the previous one, on whatever stream that ran, and records its own.
  mutable std::mutex exec_mu;
  cudaEvent_t done = nullptr;
  mutable bool has_done = false;
};

namespace {

constexpr int kSmemBudget = 224 * 1024;  // stage bytes per CTA (dynamic allocation adds 1 KB)
constexpr int kCcMaxH = 16;  // block rows this short (RHS <= 32) may run on the CUDA cores

// Per-team time model of one item: the bytes its stages move (A and B) plus a fixed cost per stage
// and per item, in bytes-equivalent units.
double item_cost(int h, int nw, int64_t sum_w, int nstages) {
  return 4.0 * double(h + nw) * double(sum_w) + 4096.0 * nstages + 8192.0;
}

cudaError_t set_kernel_attrs() {
  const int bytes = kSmemBudget + 1024;
  const void* kernels[] = {
      reinterpret_cast<const void*>(spmm_tc_kernel<false, false, false, false>),
      reinterpret_cast<const void*>(spmm_tc_kernel<true, false, false, false>),
      reinterpret_cast<const void*>(spmm_tc_kernel<false, false, true, false>),
      reinterpret_cast<const void*>(spmm_tc_kernel<true, false, true, false>),
      reinterpret_cast<const void*>(spmm_tc_kernel<false, false, true, true>),
      reinterpret_cast<const void*>(spmm_tc_kernel<true, false, true, true>),
      reinterpret_cast<const void*>(spmm_tc_kernel<false, true, false, false>),
      reinterpret_cast<const void*>(spmm_tc_kernel<true, true, false, false>)};
  for (const void* k : kernels) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Schedule for spmm_tc_kernel: one item per block row (or per row part of a heavy block row), one
// CTA per SM; items assigned to CTAs by longest-processing-time-first on the cost model; each
// CTA's stream cuts the item's 8-column groups into stages of stage_groups(h, rhs) groups.
vbsr_status build_schedule(vbsr_plan* p) {
  const MatrixData& d = p->m->d;
  const int rhs = p->rhs;
  int num_sm = 148;
  VBSR_CUDA(cudaDeviceGetAttribute(&num_sm, cudaDevAttrMultiProcessorCount, d.device));
  if (d.nvalues >= stage::kMaxVal || d.K >= stage::kMaxCol || d.M >= (int64_t(1) << 31))
    return set_error(VBSR_INVALID_ARGUMENT, "matrix exceeds the schedule's index range");

  // Column-stacked form: raw-B stacks when the pre-split stacks (K x 512 bytes) would not stay in
  // L2 (a stack read then comes from DRAM, and raw halves those bytes); pre-split stacks below
  // that, where the reads hit L2 and the extra split work of raw would only cost time.
  constexpr int64_t kRawStackBytes = 64ll << 20;
  const bool big = (d.K / 8) * int64_t(stack_tile_bytes(rhs, false)) > kRawStackBytes;
  p->raw_b = !row_stacked(rhs) &&
             ((p->flags & (VBSR_PLAN_STACKS_RAW | VBSR_PLAN_B_DIRECT)) ? true
              : (p->flags & VBSR_PLAN_STACKS_PRESPLIT)                 ? false
                                                                       : big);
  // Raw-B stacks read straight from B by the SpMM (no pre-pass)
  p->direct_b = p->raw_b && (p->flags & VBSR_PLAN_B_DIRECT) != 0;
  p->fused_stack = !p->direct_b && (p->flags & VBSR_PLAN_FUSED_PREPASS) != 0;
  const int R = d.block_rows;
  // Work units: one per block row, or, for a block row whose cost exceeds a CTA's fair share, one
  // per row part. A row part is rows [r0, r0 + hp) of the block row (multiples of 8) over all its
  // blocks: parts write disjoint rows of C, so no atomics and no workspace are needed. Each part
  // streams only its rows of A but the block row's whole B slice, so parts are made no smaller
  // than needed: P = ceil(cost / fair share), at most H / 8.
  struct Unit {
    int row, r0, hp;
    double cost;
  };
  auto groups_of = [&](int i) {
    int64_t g = 0;
    for (int b = d.h_row_ptr[i]; b < d.h_row_ptr[i + 1]; ++b) g += int64_t((d.h_blk_desc[b] & 7u) + 1u);
    return g;
  };
  auto unit_cost = [&](int i, int hp) {
    const int G = stage_groups(hp, rhs, p->raw_b);  // 8-column groups per stage
    return item_cost(hp, rhs, d.h_sum_w[i], int((groups_of(i) + G - 1) / G));
  };
  std::vector<double> row_cost(R);
  double total = 0.0;
  for (int i = 0; i < R; ++i) total += (row_cost[i] = unit_cost(i, d.h_row_size[i]));
  const double fair = total / double(num_sm);
  const bool may_split = !(p->flags & VBSR_PLAN_NO_SPLIT);
  std::vector<Unit> units;
  units.reserve(size_t(R));
  int split_rows = 0;
  // With VBSR_PLAN_CUDA_CORE_ROWS, short rows (h <= 16, RHS <= 32) go to the CUDA-core path of
  // the pre-pass launch, unless
  // they are heavy, both wider than 1024 columns and above a quarter of an SM's fair share: those
  // stay here, where the tensor cores' throughput pays (a CUDA-core row is one warp's work).
  const bool cc_on = row_stacked(rhs) && (p->flags & VBSR_PLAN_CUDA_CORE_ROWS) != 0;
  std::vector<CcItem> cc;
  std::vector<double> cc_cost;
  for (int i = 0; i < R; ++i) {
    const int H = d.h_row_size[i];
    if (cc_on && H <= kCcMaxH && (d.h_sum_w[i] <= 1024 || row_cost[i] <= 0.25 * fair)) {
      CcItem c{};
      c.c_row = uint32_t(d.h_row_off[i]);
      c.h = uint32_t(H);
      c.b0 = uint32_t(d.h_row_ptr[i]);
      c.b1 = uint32_t(d.h_row_ptr[i + 1]);
      c.a_off = uint64_t(d.h_val_off_row[i]);
      cc.push_back(c);
      cc_cost.push_back(double(H) * double(d.h_sum_w[i]) + 64.0);
      continue;
    }
    int parts = 1;
    if (may_split && R > 1 && row_cost[i] > fair)
      parts = std::min(H / 8, int(std::ceil(row_cost[i] / fair)));
    if (parts <= 1) {
      units.push_back({i, 0, H, row_cost[i]});
      continue;
    }
    ++split_rows;
    const int blocks8 = H / 8;
    for (int q = 0, r8 = 0; q < parts; ++q) {
      const int n8 = blocks8 / parts + (q < blocks8 % parts ? 1 : 0);  // 8-row blocks of part q
      units.push_back({i, 8 * r8, 8 * n8, unit_cost(i, 8 * n8)});
      r8 += n8;
    }
  }
  const int nunits = int(units.size());
  const int teams = std::min(num_sm, nunits);  // 0 when every row is on the CUDA cores
  std::vector<int> order(nunits);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return units[a].cost > units[b].cost; });
  using Load = std::pair<double, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int t = 0; t < teams; ++t) heap.push({0.0, t});
  std::vector<std::vector<int>> lists(teams);
  std::vector<double> load(teams, 0.0);
  for (int u : order) {
    Load l = heap.top();
    heap.pop();
    lists[l.second].push_back(u);
    l.first += units[u].cost;
    load[l.second] = l.first;
    heap.push(l);
  }

  std::vector<StageDesc> stream;
  stream.reserve(size_t(d.nnzb) * 2 + 16);
  std::vector<ItemDesc> items;
  items.reserve(size_t(nunits));
  std::vector<Task> h_tasks;
  const int slot = slot_floats(rhs);
  // A multiple of every role's warp count: every slot then has one feeder, one split warp and one
  // MMA warp, which pass through its uses in order, so a wait never meets a phase of another use.
  const int stages =
      std::min(kMaxStages, (kSmemBudget - kSmemTailPad) / (slot * 4)) / kTcRingMultiple *
      kTcRingMultiple;
  if (stages < kTcRingMultiple) return set_error(VBSR_INVALID_ARGUMENT, "stage does not fit shared memory");
  const uint64_t nwc = uint64_t(stage::nw_code(rhs));
  for (int t = 0; t < teams; ++t) {
    Task task{};
    task.item_off = int(items.size());
    task.stage_off = int(stream.size());
    std::vector<int>& l = lists[t];
    std::sort(l.begin(), l.end());  // units are in row order, parts of a row by r0
    for (int u : l) {
      const int i = units[u].row, r0 = units[u].r0, h = units[u].hp, H = d.h_row_size[i];
      const uint64_t base0 =
          (uint64_t(h / 8 - 1) << 32) | (nwc << 39) | (uint64_t(H / 8 - 1) << 41);
      ItemDesc item{};
      item.c_row = uint32_t(d.h_row_off[i] + r0);
      item.shape = uint32_t(h / 8 - 1) | (uint32_t(nwc) << 6);
      item.k0 = uint32_t(stream.size() - size_t(task.stage_off));
      const uint64_t w1 = uint64_t(items.size() - size_t(task.item_off));
      // The item's 8-column groups, block after block, in runs of G per stage. In the device
      // format group g of a block starts 8*H*g floats after the block's values and a block row's
      // blocks are consecutive, so a stage's A values are one contiguous range (a row part's rows
      // start 8*r0 floats into each group).
      int64_t val = d.h_val_off_row[i];
      const int G = stage_groups(h, rhs, p->raw_b);
      int used = 0;  // columns in the current stage
      StageDesc cur{};
      for (int b = d.h_row_ptr[i]; b < d.h_row_ptr[i + 1]; ++b) {
        const uint32_t desc = d.h_blk_desc[b];
        const int w = int((desc & 7u) + 1u) * 8;
        const int64_t col = int64_t(desc & ~7u);
        for (int g = 0; g < w / 8; ++g) {
          if (used == 8 * G) {
            cur.w[0] |= uint64_t(used / 8 - 1) << 28;
            stream.push_back(cur);
            used = 0;
          }
          if (used == 0) {
            cur = StageDesc{};
            cur.w[0] = base0 | uint64_t((val + int64_t(8) * H * g + int64_t(8) * r0) / 64);
            cur.w[1] = w1;
          }
          const int gg = used / 8;  // < kMaxStageGroups
          cur.w[2 + gg / 2] |= uint64_t((col + 8 * g) / 8) << (32 * (gg & 1));
          used += 8;
        }
        val += int64_t(H) * w;
      }
      if (used > 0) {
        cur.w[0] |= uint64_t(used / 8 - 1) << 28;
        stream.push_back(cur);
      }
      // a block row without blocks keeps n = 0: its C rows are stored as zeros
      item.n = uint32_t(stream.size() - size_t(task.stage_off)) - item.k0;
      const int64_t item_groups = d.h_sum_w[i] / 8;
      if (item_groups >= (int64_t(1) << 24))
        return set_error(VBSR_INVALID_ARGUMENT, "block row too wide for the schedule");
      item.shape |= uint32_t(item_groups) << 8;
      items.push_back(item);
    }
    task.item_end = int(items.size());
    task.stage_end = int(stream.size());
    task.team_warps = tc_warps(row_stacked(rhs));
    task.stage_floats = slot;
    task.stage_cols = 8 * kMaxStageGroups;
    task.stages = stages;
    h_tasks.push_back(task);
    p->task_warps.push_back(tc_warps(row_stacked(rhs)));
    p->task_cost.push_back(load[t]);
  }
  p->split_rows = split_rows;
  p->work_items = nunits;
  // CUDA-core rows: the most expensive first, dealt round-robin to the warps
  {
    std::vector<int> ord(cc.size());
    std::iota(ord.begin(), ord.end(), 0);
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return cc_cost[a] > cc_cost[b]; });
    std::vector<CcItem> sorted(cc.size());
    for (size_t j = 0; j < ord.size(); ++j) sorted[j] = cc[size_t(ord[j])];
    cc.swap(sorted);
  }
  p->cc_count = int(cc.size());
  {
    vbsr_plan_work& wk = p->work;
    wk.tc_items = nunits;
    wk.split_rows = split_rows;
    wk.cc_rows = int64_t(cc.size());
    wk.tc_rows = R - wk.cc_rows;
    for (const CcItem& c : cc) {
      int64_t sw = 0;
      for (uint32_t b = c.b0; b < c.b1; ++b) sw += int64_t((d.h_blk_desc[b] & 7u) + 1u) * 8;
      wk.cc_values += int64_t(c.h) * sw;
      wk.cc_scalar_rows += int64_t(c.h);
    }
    wk.tc_values = d.nvalues - wk.cc_values;
  }

  if (stream.size() >= (size_t(1) << 31))
    return set_error(VBSR_INVALID_ARGUMENT, "schedule too large");
  p->smem_bytes = stages * slot * 4 + kSmemTailPad + 1024;  // + alignment of the ring
  p->num_tasks = int(h_tasks.size());
  p->stream_entries = int64_t(stream.size());

  char buf[512];
  std::snprintf(buf, sizeof buf,
                "rhs=%d items=%d split_rows=%d cuda_core_rows=%d pipeline_stages=%zu tasks=%d "
                "teams=%d ring=%d smem=%d sms=%d kernel=tcgen05-3xtf32-%s",
                rhs, nunits, split_rows, p->cc_count, stream.size(), p->num_tasks, teams, stages,
                p->smem_bytes, num_sm,
                row_stacked(rhs) ? "row-stacked"
                : p->direct_b    ? "column-stacked-direct-b"
                : p->raw_b       ? "column-stacked-raw-b"
                                 : "column-stacked-pre-split");
  p->summary = buf;

  DeviceGuard guard(d.device);
  SetupStream ss;
  VBSR_CUDA(ss.init());
  VBSR_CUDA(cudaMalloc(&p->d_stream, std::max<size_t>(1, stream.size()) * sizeof(StageDesc)));
  VBSR_CUDA(cudaMalloc(&p->d_items, std::max<size_t>(1, items.size()) * sizeof(ItemDesc)));
  // one M x 8 tile of B's operand stack per 8-column group of B (bstack_kernel)
  p->bstack_floats = p->direct_b ? 0 : (d.K / 8) * int64_t(stack_rows(rhs, p->raw_b)) * 8;
  if ((d.K / 8) * rhs >= (int64_t(1) << 31))
    return set_error(VBSR_INVALID_ARGUMENT, "B too large for the pre-pass index range");
  VBSR_CUDA(cudaMalloc(&p->d_bstack, size_t(std::max<int64_t>(1, p->bstack_floats)) * sizeof(float)));
  // rows of RHS columns >= rhs (rhs < 32) are never written by the pre-pass: zero them once
  VBSR_CUDA(cudaMemsetAsync(p->d_bstack, 0,
                            size_t(std::max<int64_t>(1, p->bstack_floats)) * sizeof(float), ss.s));
  if (!items.empty())
    VBSR_CUDA(cudaMemcpyAsync(p->d_items, items.data(), items.size() * sizeof(ItemDesc),
                              cudaMemcpyHostToDevice, ss.s));
  VBSR_CUDA(cudaMalloc(&p->d_tasks, std::max<size_t>(1, h_tasks.size()) * sizeof(Task)));
  VBSR_CUDA(cudaMalloc(&p->d_status, kStatusWords * sizeof(int)));
  if (!stream.empty())
    VBSR_CUDA(cudaMemcpyAsync(p->d_stream, stream.data(), stream.size() * sizeof(StageDesc),
                              cudaMemcpyHostToDevice, ss.s));
  if (!h_tasks.empty())
    VBSR_CUDA(cudaMemcpyAsync(p->d_tasks, h_tasks.data(), h_tasks.size() * sizeof(Task),
                              cudaMemcpyHostToDevice, ss.s));
  VBSR_CUDA(cudaMemsetAsync(p->d_status, 0, kStatusWords * sizeof(int), ss.s));
  VBSR_CUDA(cudaMalloc(&p->d_stack_flag, sizeof(uint32_t)));
  VBSR_CUDA(cudaMemsetAsync(p->d_stack_flag, 0, sizeof(uint32_t), ss.s));
  if (!cc.empty()) {
    VBSR_CUDA(cudaMalloc(&p->d_cc, cc.size() * sizeof(CcItem)));
    VBSR_CUDA(cudaMemcpyAsync(p->d_cc, cc.data(), cc.size() * sizeof(CcItem),
                              cudaMemcpyHostToDevice, ss.s));
  }
  VBSR_CUDA(ss.finish());
  VBSR_CUDA(cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming));
  VBSR_CUDA(set_kernel_attrs());
  return VBSR_OK;
}

void free_plan(vbsr_plan* p) {
  if (p == nullptr) return;
  DeviceGuard guard(p->device);
  cudaFree(p->d_stream);
  cudaFree(p->d_items);
  cudaFree(p->d_bstack);
  cudaFree(p->d_tasks);
  cudaFree(p->d_status);
  cudaFree(p->d_stack_flag);
  cudaFree(p->d_timing);
  cudaFree(p->d_cc);
  if (p->done != nullptr) cudaEventDestroy(p->done);
  delete p;
}

// One execute on `stream`: the B pre-pass launch and then the SpMM, or only the SpMM kernel,
// which then forms B's operand stacks itself (VBSR_PLAN_FUSED_PREPASS). The short block rows on
// the CUDA cores (VBSR_PLAN_CUDA_CORE_ROWS) are CTAs of a pre-pass launch either way.
void launch_spmm(const vbsr_plan* p, const KernelParams& kp, cudaStream_t stream) {
  const int64_t bsg = bs_groups(kp.rhs);
  const int64_t chunks = (kp.K / 8 + bsg - 1) / bsg;  // bs_groups(rhs) groups per block iteration
  CcParams cc{};
  cc.items = p->d_cc;
  cc.count = p->cc_count;
  cc.values = kp.values;
  cc.blk_desc = p->m->d.d_blk_desc;
  cc.value_off = p->m->d.d_value_off;
  cc.C = kp.C;
  cc.M = kp.M;
  const int cc_blocks = p->cc_count;  // one CTA per short block row
  const bool separate = !p->direct_b && !p->fused_stack && chunks > 0 &&
                        !(p->flags & VBSR_PLAN_DIAG_SKIP_PREPASS);
  const bool prepass = separate || cc_blocks > 0;
  if (prepass) {
    const int stack = separate ? int(std::min<int64_t>(chunks, 148 * kBsBlocksPerSm)) : 0;
    const unsigned blocks = unsigned(stack + cc_blocks);
    switch (kp.rhs) {
      case 8: bstack_kernel<8, false><<<blocks, 256, 0, stream>>>(kp.B, kp.K, p->d_bstack, stack, cc); break;
      case 16: bstack_kernel<16, false><<<blocks, 256, 0, stream>>>(kp.B, kp.K, p->d_bstack, stack, cc); break;
      case 32: bstack_kernel<32, false><<<blocks, 256, 0, stream>>>(kp.B, kp.K, p->d_bstack, stack, cc); break;
      default:
        if (p->raw_b)
          bstack_kernel<64, true><<<blocks, 256, 0, stream>>>(kp.B, kp.K, p->d_bstack, stack, cc);
        else
          bstack_kernel<64, false><<<blocks, 256, 0, stream>>>(kp.B, kp.K, p->d_bstack, stack, cc);
        break;
    }
  }
  if (p->num_tasks == 0) return;  // every row on the CUDA cores
  // programmatic dependent launch: the SpMM's prologue overlaps the pre-pass (its feeders wait
  // for the pre-pass with griddepcontrol.wait before the first copy)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p->num_tasks));
  cfg.blockDim = dim3(32 * tc_warps(row_stacked(kp.rhs)));
  cfg.dynamicSmemBytes = size_t(p->smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool check = (p->flags & VBSR_PLAN_BOUNDS_CHECK) != 0;
  if (!prepass) cfg.numAttrs = 0;  // no pre-pass launch to overlap
  if (row_stacked(kp.rhs))
    cudaLaunchKernelEx(&cfg, check ? spmm_tc_kernel<true, true, false, false>
                                   : spmm_tc_kernel<false, true, false, false>, kp);
  else if (p->direct_b)
    cudaLaunchKernelEx(&cfg, check ? spmm_tc_kernel<true, false, true, true>
                                   : spmm_tc_kernel<false, false, true, true>, kp);
  else if (p->raw_b)
    cudaLaunchKernelEx(&cfg, check ? spmm_tc_kernel<true, false, true, false>
                                   : spmm_tc_kernel<false, false, true, false>, kp);
  else
    cudaLaunchKernelEx(&cfg, check ? spmm_tc_kernel<true, false, false, false>
                                   : spmm_tc_kernel<false, false, false, false>, kp);
}

// Enqueues one execute on `stream` after the plan's previous execute (on any stream) has finished
// with the operand-stack buffer, then records its own completion. Waiting on an event recorded
// outside a stream capture is not allowed inside one, so a captured execute is ordered only by the
// graph the caller builds (executes captured on one stream are ordered by that stream).
vbsr_status enqueue_execute(const vbsr_plan* p, const KernelParams& kp, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(p->exec_mu);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  VBSR_CUDA(cudaStreamIsCapturing(stream, &cs));
  const bool capturing = cs != cudaStreamCaptureStatusNone;
  if (!capturing && p->has_done) VBSR_CUDA(cudaStreamWaitEvent(stream, p->done, 0));
  launch_spmm(p, kp, stream);
  VBSR_CUDA(cudaGetLastError());
  if (!capturing) {
    VBSR_CUDA(cudaEventRecord(p->done, stream));
    p->has_done = true;
  }
  return VBSR_OK;
}

// Launch parameters of one execute: the plan's schedule and the caller's B and C.
vbsr_status fill_params(const vbsr_plan* p, const float* B, float* C, int* status,
                        unsigned long long* timing, KernelParams* kp) {
  const MatrixData& d = p->m->d;
  kp->bstack = p->d_bstack;
  kp->stages = p->d_stream;
  kp->items = p->d_items;
  kp->tasks = p->d_tasks;
  kp->values = d.d_values;
  kp->B = B;
  kp->C = C;
  kp->M = d.M;
  kp->K = d.K;
  kp->nvalues = d.nvalues;
  kp->rhs = p->rhs;
  kp->status = status;
  kp->drop_stage = p->drop_stage;
  kp->wait_limit = p->wait_limit;
  kp->timing = timing;
  // per-CTA cycle counters of instrumented builds follow the timestamps (plan-owned buffer only)
  kp->prof = (timing != nullptr && timing == p->d_timing) ? timing + 2 * p->num_tasks : nullptr;
  kp->diag = int(p->flags & (VBSR_PLAN_DIAG_SKIP_COPIES | VBSR_PLAN_DIAG_SKIP_MATH |
                             VBSR_PLAN_DIAG_SKIP_PREPASS));
  kp->stack_flag = p->fused_stack ? p->d_stack_flag : nullptr;
  return VBSR_OK;
}

vbsr_status launch_view_kernel(const vbsr_device_matrix* a, const float* B, float* C, int rhs,
                               cudaStream_t stream, bool scalar) {
  if (a == nullptr || (a->block_rows > 0 && (B == nullptr || C == nullptr)))
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  if (!valid_rhs(rhs)) return set_error(VBSR_INVALID_ARGUMENT, "unsupported rhs width");
  if (a->block_rows == 0) return VBSR_OK;
  if (scalar) {
    const int per_row = (64 * rhs + 255) / 256;
    rowwise_scalar_kernel<<<dim3(a->block_rows, per_row), 256, 0, stream>>>(*a, B, C, rhs);
  } else {
    rowwise_direct_kernel<<<a->block_rows, 256, 0, stream>>>(*a, B, C, rhs);
  }
  VBSR_CUDA(cudaGetLastError());
  return VBSR_OK;
}

}  // namespace

extern "C" {

vbsr_status vbsr_matrix_create(const vbsr_host_matrix_view* host, int device, vbsr_matrix** out) {
  clear_error();
  if (host == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null matrix view");
  return build_matrix(host, 0, host->block_rows, 0, 0, device, out);
}

vbsr_status vbsr_matrix_create_rows(const vbsr_host_matrix_view* host, int32_t row_begin,
                                    int32_t row_end, int device, vbsr_matrix** out) {
  clear_error();
  return build_matrix(host, row_begin, row_end, 0, 0, device, out);
}

vbsr_status vbsr_matrix_create_rows_generated(const vbsr_host_matrix_view* host, int32_t row_begin,
                                              int32_t row_end, uint64_t seed, int device,
                                              vbsr_matrix** out) {
  clear_error();
  return build_matrix(host, row_begin, row_end, 1, seed, device, out);
}

vbsr_status vbsr_matrix_destroy(vbsr_matrix* m) {
  clear_error();
  if (m == nullptr) return VBSR_OK;
  {
    DeviceGuard guard(m->d.device);
    release(m->d);
  }
  delete m;
  return VBSR_OK;
}

vbsr_status vbsr_matrix_info_get(const vbsr_matrix* m, vbsr_matrix_info* o) {
  clear_error();
  if (m == nullptr || o == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  const MatrixData& d = m->d;
  o->block_rows = d.block_rows;
  o->block_cols = d.block_cols;
  o->nnzb = d.nnzb;
  o->scalar_rows = d.M;
  o->scalar_cols = d.K;
  o->value_count = d.nvalues;
  o->device_bytes = d.device_bytes;
  o->device = d.device;
  o->row_begin = d.row_begin;
  o->row_end = d.row_end;
  return VBSR_OK;
}

vbsr_status vbsr_matrix_device_view(const vbsr_matrix* m, vbsr_device_matrix* o) {
  clear_error();
  if (m == nullptr || o == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  const MatrixData& d = m->d;
  o->block_rows = d.block_rows;
  o->block_cols = d.block_cols;
  o->nnzb = int32_t(d.nnzb);
  o->scalar_rows = d.M;
  o->scalar_cols = d.K;
  o->row_ptr = d.d_row_ptr;
  o->block_col = d.d_block_col;
  o->row_size = d.d_row_size;
  o->col_size = d.d_col_size;
  o->row_scalar_off = d.d_row_off;
  o->col_scalar_off = d.d_col_off;
  o->value_off = d.d_value_off;
  o->values = d.d_values;
  return VBSR_OK;
}

vbsr_status vbsr_plan_create_ex(const vbsr_matrix* m, int rhs, int kernel, uint32_t flags,
                                vbsr_plan** out) {
  clear_error();
  if (m == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  // plan.cpp:9-17
  if (!valid_rhs(rhs)) return set_error(VBSR_INVALID_ARGUMENT, "rhs_width must be 8,16,32,64");
  if (kernel == VBSR_KERNEL_SPLIT_ROW)
    return set_error(VBSR_INVALID_ARGUMENT,
                     "split-row was not justified by the 1.0 regime map; use RowOwned or "
                     "GroupedGemmPlan");
  if (kernel != VBSR_KERNEL_AUTO && kernel != VBSR_KERNEL_ROW_OWNED)
    return set_error(VBSR_INVALID_ARGUMENT, "unknown kernel");
  auto* p = new (std::nothrow) vbsr_plan;
  if (p == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  p->m = m;
  p->rhs = rhs;
  p->flags = flags;
  p->device = m->d.device;
  vbsr_status st;
  try {
    st = build_schedule(p);
  } catch (const std::bad_alloc&) {
    st = set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  }
  if (st != VBSR_OK) {
    free_plan(p);
    return st;
  }
  *out = p;
  return VBSR_OK;
}

vbsr_status vbsr_plan_create(const vbsr_matrix* m, int rhs, int kernel, vbsr_plan** out) {
  return vbsr_plan_create_ex(m, rhs, kernel, 0u, out);
}

vbsr_status vbsr_plan_destroy(vbsr_plan* p) {
  clear_error();
  free_plan(p);
  return VBSR_OK;
}

vbsr_status vbsr_plan_execute(const vbsr_plan* p, const float* B, float* C, vbsr_stream_t stream) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  if (B == nullptr || C == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null B or C");
  DeviceGuard guard(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((reinterpret_cast<uintptr_t>(B) & 15u) || (reinterpret_cast<uintptr_t>(C) & 15u)) {
    // TMA bulk copies and 16-byte stores need 16-byte aligned panels; unaligned caller buffers
    // take the plain-load row kernel instead.
    vbsr_device_matrix view;
    vbsr_matrix_device_view(p->m, &view);
    return launch_view_kernel(&view, B, C, p->rhs, s, false);
  }
  if (p->num_tasks == 0 && p->cc_count == 0) return VBSR_OK;
  KernelParams kp;
  vbsr_status st = fill_params(p, B, C, p->d_status, p->timing_on ? p->d_timing : nullptr, &kp);
  if (st != VBSR_OK) return st;
  return enqueue_execute(p, kp, s);
}

// ---- execute without allocating ---------------------------------------------------------------------
//
// vbsr_plan_execute keeps the kernel's status word (and, when timing is switched on, its per-CTA
// timestamps) in device memory that the plan allocated with cudaMalloc. Some callers are not
// allowed to have device memory allocated on their behalf at all: code running inside a host
// framework that owns every device allocation (serving runtimes with their own pool, plugins whose
// host forbids cudaMalloc/cudaFree because they synchronise the device), or code paths that must
// never trigger an implicit device synchronisation. For them, vbsr_plan_execute_noalloc below keeps
// that scratch in one fixed array compiled into this library instead.
//
// Layout of the array: words 0..1 hold the kernel's status words (four 32-bit values), followed by
// one (start, end) pair of 64-bit timestamps per CTA, for at most kNoAllocMaxCtas CTAs (16 KB in
// total). Every GPU that loads this library holds the array until the process exits.
constexpr int kNoAllocMaxCtas = 1024;
static __device__ __align__(256) unsigned long long g_noalloc_scratch[2 + 2 * kNoAllocMaxCtas];

namespace {
// Device address of g_noalloc_scratch, looked up once per device. In host code the symbol's name
// is only a host-side stand-in, so the address must come from cudaGetSymbolAddress with that
// device current.
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
unsigned long long* g_noalloc_ptr[kMaxDevices] = {};

vbsr_status noalloc_scratch(int device, unsigned long long** out) {
  if (device < 0 || device >= kMaxDevices)
    return set_error(VBSR_INVALID_ARGUMENT, "device ordinal out of range for the static scratch");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e));
    g_noalloc_ptr[device] = static_cast<unsigned long long*>(ptr);
  }
  *out = g_noalloc_ptr[device];
  return VBSR_OK;
}
}  // namespace

vbsr_status vbsr_plan_execute_noalloc(const vbsr_plan* p, const float* B, float* C,
                                      vbsr_stream_t stream, uint64_t* cta_times,
                                      int cta_times_len) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  if (B == nullptr || C == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null B or C");
  if (p->num_tasks > kNoAllocMaxCtas)
    return set_error(VBSR_INVALID_ARGUMENT,
                     "plan launches " + std::to_string(p->num_tasks) +
                         " CTAs; vbsr_plan_execute_noalloc supports at most " +
                         std::to_string(kNoAllocMaxCtas));
  DeviceGuard guard(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((reinterpret_cast<uintptr_t>(B) & 15u) || (reinterpret_cast<uintptr_t>(C) & 15u)) {
    // unaligned buffers: the plain-load row kernel, which uses no scratch and records no status
    // and no timestamps; in reporting mode the call still waits and reports zero timestamps
    vbsr_device_matrix view;
    vbsr_matrix_device_view(p->m, &view);
    const vbsr_status st = launch_view_kernel(&view, B, C, p->rhs, s, false);
    if (st != VBSR_OK || cta_times == nullptr) return st;
    if (cta_times_len > 0) std::memset(cta_times, 0, size_t(cta_times_len) * sizeof(uint64_t));
    VBSR_CUDA(cudaStreamSynchronize(s));
    return VBSR_OK;
  }
  if (p->num_tasks == 0 && p->cc_count == 0) return VBSR_OK;
  unsigned long long* scratch = nullptr;
  vbsr_status st = noalloc_scratch(p->device, &scratch);
  if (st != VBSR_OK) return st;
  // the array keeps the previous call's contents: clear the status words and the timestamps
  const size_t used = (2 + 2 * size_t(p->num_tasks)) * sizeof(unsigned long long);
  VBSR_CUDA(cudaMemsetAsync(scratch, 0, used, s));
  KernelParams kp;
  st = fill_params(p, B, C, reinterpret_cast<int*>(scratch), scratch + 2, &kp);
  if (st != VBSR_OK) return st;
  st = enqueue_execute(p, kp, s);
  if (st != VBSR_OK || cta_times == nullptr) return st;
  // Reporting mode: wait for this launch, then return its status and CTA timestamps.
  int words[kStatusWords] = {0, 0, 0, 0};
  VBSR_CUDA(cudaMemcpyAsync(words, scratch, sizeof words, cudaMemcpyDeviceToHost, s));
  const int n = std::max(0, std::min(cta_times_len, 2 * p->num_tasks));
  if (n > 0)
    VBSR_CUDA(cudaMemcpyAsync(cta_times, scratch + 2, size_t(n) * sizeof(uint64_t),
                              cudaMemcpyDeviceToHost, s));
  VBSR_CUDA(cudaStreamSynchronize(s));
  if (words[kStatusCode] == VBSR_TIMEOUT)
    return set_error(VBSR_TIMEOUT, "pipeline wait timed out in CTA " + std::to_string(words[kStatusInfo]));
  if (words[kStatusCode] == VBSR_BOUNDS_VIOLATION)
    return set_error(VBSR_BOUNDS_VIOLATION, "index out of bounds (info " + std::to_string(words[kStatusInfo]) + ")");
  if (words[kStatusCode] != 0) return set_error(VBSR_CUDA_ERROR, "unknown device status");
  return VBSR_OK;
}

vbsr_status vbsr_plan_launch_count(const vbsr_plan* p, int* out) {
  clear_error();
  if (p == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  // the SpMM kernel, plus the pre-pass launch when the stacks are formed separately or short rows
  // run on the CUDA cores
  *out = 1 + ((!p->direct_b && !p->fused_stack) || p->cc_count > 0 ? 1 : 0);
  return VBSR_OK;
}

vbsr_status vbsr_plan_check_status(const vbsr_plan* p, vbsr_stream_t stream) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  DeviceGuard guard(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int words[kStatusWords] = {0, 0, 0, 0};
  VBSR_CUDA(cudaMemcpyAsync(words, p->d_status, sizeof words, cudaMemcpyDeviceToHost, s));
  VBSR_CUDA(cudaMemsetAsync(p->d_status, 0, sizeof words, s));
  VBSR_CUDA(cudaStreamSynchronize(s));
  if (words[kStatusCode] == VBSR_TIMEOUT)
    return set_error(VBSR_TIMEOUT, "pipeline wait timed out in CTA " + std::to_string(words[kStatusInfo]));
  if (words[kStatusCode] == VBSR_BOUNDS_VIOLATION)
    return set_error(VBSR_BOUNDS_VIOLATION, "index out of bounds in work item " + std::to_string(words[kStatusInfo]));
  if (words[kStatusCode] != 0) return set_error(VBSR_CUDA_ERROR, "unknown device status");
  return VBSR_OK;
}

vbsr_status vbsr_plan_describe(const vbsr_plan* p, char* buf, size_t len) {
  clear_error();
  if (p == nullptr || buf == nullptr || len == 0) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  std::snprintf(buf, len, "%s", p->summary.c_str());
  return VBSR_OK;
}

vbsr_status vbsr_plan_set_debug(vbsr_plan* p, int drop_stage, int64_t wait_limit_cycles) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  p->drop_stage = drop_stage < 0 ? -1 : drop_stage;
  p->wait_limit = wait_limit_cycles > 0 ? wait_limit_cycles : 4000000000ll;
  return VBSR_OK;
}

vbsr_status vbsr_plan_cta_timing(vbsr_plan* p, int enable, uint64_t* out, int out_len,
                                 vbsr_stream_t stream) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  DeviceGuard guard(p->device);
  if (enable && p->d_timing == nullptr)
    VBSR_CUDA(cudaMalloc(&p->d_timing, std::max(1, 18 * p->num_tasks) * sizeof(uint64_t)));
  if (enable && out == nullptr) {  // switching on: start from zeroed counters
    SetupStream ss;
    VBSR_CUDA(ss.init());
    VBSR_CUDA(cudaMemsetAsync(p->d_timing, 0, std::max(1, 18 * p->num_tasks) * sizeof(uint64_t),
                              ss.s));
    VBSR_CUDA(ss.finish());
  }
  if (out != nullptr && p->d_timing != nullptr) {
    const int n = std::min(out_len, 18 * p->num_tasks);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    VBSR_CUDA(cudaMemcpyAsync(out, p->d_timing, size_t(n) * sizeof(uint64_t),
                              cudaMemcpyDeviceToHost, s));
    VBSR_CUDA(cudaStreamSynchronize(s));
  }
  p->timing_on = enable != 0;
  return VBSR_OK;
}

vbsr_status vbsr_plan_task_stats(const vbsr_plan* p, int32_t* team_warps, double* model_cost,
                                 int n) {
  clear_error();
  if (p == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null plan");
  for (int i = 0; i < n && i < p->num_tasks; ++i) {
    if (team_warps) team_warps[i] = p->task_warps[i];
    if (model_cost) model_cost[i] = p->task_cost[i];
  }
  return VBSR_OK;
}

vbsr_status vbsr_plan_work_info(const vbsr_plan* p, vbsr_plan_work* out) {
  clear_error();
  if (p == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = p->work;
  return VBSR_OK;
}

vbsr_status vbsr_plan_num_tasks(const vbsr_plan* p, int* out) {
  clear_error();
  if (p == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = p->num_tasks;
  return VBSR_OK;
}

vbsr_status vbsr_launch_row_owned(const vbsr_device_matrix* a, const int32_t* row_shape_order,
                                  int small_row_count, int large_row_count, const float* B,
                                  float* C, int rhs, vbsr_stream_t stream) {
  clear_error();
  (void)row_shape_order;
  (void)small_row_count;
  (void)large_row_count;
  return launch_view_kernel(a, B, C, rhs, reinterpret_cast<cudaStream_t>(stream), false);
}

vbsr_status vbsr_launch_row_owned_scalar(const vbsr_device_matrix* a, const float* B, float* C,
                                         int rhs, vbsr_stream_t stream) {
  clear_error();
  return launch_view_kernel(a, B, C, rhs, reinterpret_cast<cudaStream_t>(stream), true);
}

vbsr_status vbsr_fill_uniform_device(uint64_t seed, uint64_t stream, uint64_t first,
                                     uint64_t count, float* out, vbsr_stream_t cuda_stream) {
  clear_error();
  if (count == 0) return VBSR_OK;
  if (out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null output");
  const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 65536);
  fill_uniform_kernel<<<unsigned(blocks), 256, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
      rng_key(seed, stream), first, count, out);
  VBSR_CUDA(cudaGetLastError());
  return VBSR_OK;
}

#ifdef VBSR_TRACE
// development builds only
vbsr_status vbsr_debug_trace(long long* stages, long long* items) {
  VBSR_CUDA(cudaMemcpyFromSymbol(stages, g_trace, sizeof(g_trace)));
  VBSR_CUDA(cudaMemcpyFromSymbol(items, g_trace_items, sizeof(g_trace_items)));
  return VBSR_OK;
}
#endif
}  // extern "C"
