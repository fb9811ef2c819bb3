// vbsr_multi.cpp — the multi-GPU plan: one process drives the block-row shards of a matrix on
// several GPUs.
//
// The reference is single-GPU; its API has no counterpart. The partition, the B replication
// and the C gather follow the plan described for this engine:
// - contiguous block-row ranges of balanced cost (vbsr_partition_rows);
// - one shard matrix and plan per range, on its GPU;
// - a full B replica per shard, copied peer to peer along a doubling tree (no NCCL on the compute
//   path);
// - each shard writes its own disjoint rows of C, so execute has no reduction and no exchange.
// A gather assembles the column-major M x N result from the shards for the caller.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "vbsr_b200.h"
#include "vbsr_internal.h"

using vbsr_b200::clear_error;
using vbsr_b200::set_error;

namespace {

#define VBSR_MCUDA(call)                                                                 \
  do {                                                                                   \
    const cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess) return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e_));    \
  } while (0)

// Restores the caller's current device on scope exit.
struct Guard {
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (dev >= 0 && dev != prev) cudaSetDevice(dev);
  }
  ~Guard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

struct Shard {
  int device = 0;
  int32_t row_begin = 0, row_end = 0;
  int64_t c_row0 = 0, c_rows = 0;  // first scalar row of the shard in C, and its row count
  vbsr_matrix* m = nullptr;
  vbsr_plan* p = nullptr;
  float* B = nullptr;  // full K x rhs replica
  float* C = nullptr;  // c_rows x rhs, ld c_rows
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_b = nullptr;                       // the replica is complete
  cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr;     // bracket the last execute
};

}  // namespace

struct vbsr_multi_plan {
  int rhs = 32;
  int64_t K = 0, M = 0;
  bool executed = false;
  std::vector<Shard> shards;
};

namespace {

void release(vbsr_multi_plan* mp) {
  for (Shard& s : mp->shards) {
    Guard g(s.device);
    if (s.stream) cudaStreamSynchronize(s.stream);
    if (s.p) vbsr_plan_destroy(s.p);
    if (s.m) vbsr_matrix_destroy(s.m);
    cudaFree(s.B);
    cudaFree(s.C);
    if (s.ev_b) cudaEventDestroy(s.ev_b);
    if (s.ev_t0) cudaEventDestroy(s.ev_t0);
    if (s.ev_t1) cudaEventDestroy(s.ev_t1);
    if (s.stream) cudaStreamDestroy(s.stream);
  }
  mp->shards.clear();
}

vbsr_status create(const vbsr_host_matrix_view* host, int ngpus, const int* devices, int rhs,
                   int kernel, uint32_t flags, bool generated, uint64_t seed,
                   vbsr_multi_plan** out) {
  if (out == nullptr || host == nullptr || devices == nullptr)
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (ngpus < 1) return set_error(VBSR_INVALID_ARGUMENT, "ngpus must be at least 1");
  if (ngpus > host->block_rows)
    return set_error(VBSR_INVALID_ARGUMENT, "more shards than block rows");
  int ndev = 0;
  VBSR_MCUDA(cudaGetDeviceCount(&ndev));
  for (int r = 0; r < ngpus; ++r)
    if (devices[r] < 0 || devices[r] >= ndev)
      return set_error(VBSR_INVALID_ARGUMENT, "device ordinal out of range");
  std::vector<int32_t> bounds(size_t(ngpus) + 1);
  vbsr_status st = vbsr_partition_rows(host, ngpus, rhs, bounds.data());
  if (st != VBSR_OK) return st;

  auto* mp = new (std::nothrow) vbsr_multi_plan;
  if (mp == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  mp->rhs = rhs;
  mp->K = host->col_scalar_off[host->block_cols];
  mp->M = host->row_scalar_off[host->block_rows];
  mp->shards.resize(size_t(ngpus));
  // Peer access between the GPUs that will copy B replicas and C blocks to one another, where the
  // hardware allows it (a setting of this process's contexts only).
  for (int a = 0; a < ngpus; ++a)
    for (int b = 0; b < ngpus; ++b) {
      const int da = devices[a], db = devices[b];
      int ok = 0;
      if (da == db || cudaDeviceCanAccessPeer(&ok, da, db) != cudaSuccess || !ok) continue;
      Guard g(da);
      const cudaError_t e = cudaDeviceEnablePeerAccess(db, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();  // clear the sticky-free error
      else if (e != cudaSuccess) {
        release(mp);
        delete mp;
        return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e));
      }
    }
  for (int r = 0; r < ngpus; ++r) {
    Shard& s = mp->shards[size_t(r)];
    s.device = devices[r];
    s.row_begin = bounds[size_t(r)];
    s.row_end = bounds[size_t(r) + 1];
    s.c_row0 = host->row_scalar_off[s.row_begin];
    s.c_rows = host->row_scalar_off[s.row_end] - s.c_row0;
    st = generated ? vbsr_matrix_create_rows_generated(host, s.row_begin, s.row_end, seed,
                                                       s.device, &s.m)
                   : vbsr_matrix_create_rows(host, s.row_begin, s.row_end, s.device, &s.m);
    if (st == VBSR_OK) st = vbsr_plan_create_ex(s.m, rhs, kernel, flags, &s.p);
    if (st == VBSR_OK) {
      Guard g(s.device);
      cudaError_t e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaMalloc(&s.B, size_t(std::max<int64_t>(1, mp->K * rhs)) * 4);
      if (e == cudaSuccess) e = cudaMalloc(&s.C, size_t(std::max<int64_t>(1, s.c_rows * rhs)) * 4);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.ev_b, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreate(&s.ev_t0);
      if (e == cudaSuccess) e = cudaEventCreate(&s.ev_t1);
      if (e != cudaSuccess) st = set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e));
    }
    if (st != VBSR_OK) {
      const std::string msg = vbsr_get_last_error();
      release(mp);
      delete mp;
      return set_error(st, msg);
    }
  }
  *out = mp;
  return VBSR_OK;
}

}  // namespace

extern "C" {

vbsr_status vbsr_multi_plan_create(const vbsr_host_matrix_view* host, int ngpus,
                                   const int* devices, int rhs, int kernel, uint32_t flags,
                                   vbsr_multi_plan** out) {
  clear_error();
  if (host != nullptr && host->values == nullptr)
    return set_error(VBSR_INVALID_ARGUMENT, "values required (see the _generated variant)");
  return create(host, ngpus, devices, rhs, kernel, flags, false, 0, out);
}

vbsr_status vbsr_multi_plan_create_generated(const vbsr_host_matrix_view* host, int ngpus,
                                             const int* devices, int rhs, int kernel,
                                             uint32_t flags, uint64_t seed,
                                             vbsr_multi_plan** out) {
  clear_error();
  return create(host, ngpus, devices, rhs, kernel, flags, true, seed, out);
}

vbsr_status vbsr_multi_plan_destroy(vbsr_multi_plan* mp) {
  clear_error();
  if (mp == nullptr) return VBSR_OK;
  release(mp);
  delete mp;
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_shard(const vbsr_multi_plan* mp, int rank, vbsr_multi_shard* out) {
  clear_error();
  if (mp == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  if (rank < 0 || rank >= int(mp->shards.size()))
    return set_error(VBSR_INVALID_ARGUMENT, "rank out of range");
  const Shard& s = mp->shards[size_t(rank)];
  out->device = s.device;
  out->row_begin = s.row_begin;
  out->row_end = s.row_end;
  out->c_row0 = s.c_row0;
  out->c_rows = s.c_rows;
  out->B = s.B;
  out->C = s.C;
  out->plan = s.p;
  out->stream = reinterpret_cast<vbsr_stream_t>(s.stream);
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_count(const vbsr_multi_plan* mp, int* ngpus) {
  clear_error();
  if (mp == nullptr || ngpus == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *ngpus = int(mp->shards.size());
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_replicate_B(vbsr_multi_plan* mp, const float* B, int src_device) {
  clear_error();
  if (mp == nullptr || (B == nullptr && mp->K > 0))
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  const size_t bytes = size_t(mp->K) * size_t(mp->rhs) * sizeof(float);
  const int n = int(mp->shards.size());
  if (bytes == 0) return VBSR_OK;
  // A replica is overwritten only after the previous call's copies out of it are done: rank i fed
  // ranks i + 2^t (2^t > i) in the tree below, and each of those recorded ev_b right after its copy.
  for (int i = 0; i < n; ++i) {
    Shard& s = mp->shards[size_t(i)];
    Guard g(s.device);
    for (int have = 1; have < n; have *= 2)
      if (i < have && i + have < n)
        VBSR_MCUDA(cudaStreamWaitEvent(s.stream, mp->shards[size_t(i + have)].ev_b, 0));
  }
  // rank 0 first, from the caller's buffer (host memory, or device memory on src_device)
  {
    Shard& s0 = mp->shards[0];
    Guard g(s0.device);
    if (src_device < 0) {
      VBSR_MCUDA(cudaMemcpyAsync(s0.B, B, bytes, cudaMemcpyHostToDevice, s0.stream));
    } else {
      VBSR_MCUDA(cudaMemcpyPeerAsync(s0.B, s0.device, B, src_device, bytes, s0.stream));
    }
    VBSR_MCUDA(cudaEventRecord(s0.ev_b, s0.stream));
  }
  // doubling tree: in round t the ranks [0, have) each copy their replica to rank i + have
  for (int have = 1; have < n; have *= 2) {
    for (int i = 0; i < have && i + have < n; ++i) {
      Shard& src = mp->shards[size_t(i)];
      Shard& dst = mp->shards[size_t(i + have)];
      Guard g(dst.device);
      VBSR_MCUDA(cudaStreamWaitEvent(dst.stream, src.ev_b, 0));
      VBSR_MCUDA(cudaMemcpyPeerAsync(dst.B, dst.device, src.B, src.device, bytes, dst.stream));
    }
    // a rank's replica event is recorded once all copies of this round that read it are queued
    for (int i = 0; i < have && i + have < n; ++i) {
      Shard& dst = mp->shards[size_t(i + have)];
      Guard g(dst.device);
      VBSR_MCUDA(cudaEventRecord(dst.ev_b, dst.stream));
    }
  }
  // Each rank's executes and gathers run on its own stream after its copy, so they see the new
  // replica, and a later replicate's copy into it waits for them.
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_execute(vbsr_multi_plan* mp) {
  clear_error();
  if (mp == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  for (Shard& s : mp->shards) {
    Guard g(s.device);
    VBSR_MCUDA(cudaEventRecord(s.ev_t0, s.stream));
    const vbsr_status st =
        vbsr_plan_execute(s.p, s.B, s.C, reinterpret_cast<vbsr_stream_t>(s.stream));
    if (st != VBSR_OK) return st;
    VBSR_MCUDA(cudaEventRecord(s.ev_t1, s.stream));
  }
  mp->executed = true;
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_synchronize(vbsr_multi_plan* mp, float* max_ms) {
  clear_error();
  if (mp == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  float worst = 0.0f;
  for (Shard& s : mp->shards) {
    Guard g(s.device);
    VBSR_MCUDA(cudaStreamSynchronize(s.stream));
    const vbsr_status st = vbsr_plan_check_status(s.p, reinterpret_cast<vbsr_stream_t>(s.stream));
    if (st != VBSR_OK) return st;
    if (mp->executed) {
      float ms = 0.0f;
      VBSR_MCUDA(cudaEventElapsedTime(&ms, s.ev_t0, s.ev_t1));
      worst = std::max(worst, ms);
    }
  }
  if (max_ms != nullptr) *max_ms = worst;
  return VBSR_OK;
}

vbsr_status vbsr_multi_plan_gather_C(vbsr_multi_plan* mp, float* C, int dst_device) {
  clear_error();
  if (mp == nullptr || (C == nullptr && mp->M > 0))
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  const size_t pitch = size_t(mp->M) * sizeof(float);
  for (Shard& s : mp->shards) {
    if (s.c_rows == 0) continue;
    Guard g(s.device);
    const size_t width = size_t(s.c_rows) * sizeof(float);
    float* dst = C + s.c_row0;
    if (dst_device < 0 || dst_device == s.device) {
      VBSR_MCUDA(cudaMemcpy2DAsync(dst, pitch, s.C, width, width, size_t(mp->rhs),
                                   dst_device < 0 ? cudaMemcpyDeviceToHost
                                                  : cudaMemcpyDeviceToDevice,
                                   s.stream));
    } else {
      cudaMemcpy3DPeerParms prm;
      std::memset(&prm, 0, sizeof(prm));
      prm.srcPtr = make_cudaPitchedPtr(s.C, width, width, size_t(mp->rhs));
      prm.srcDevice = s.device;
      prm.dstPtr = make_cudaPitchedPtr(dst, pitch, width, size_t(mp->rhs));
      prm.dstDevice = dst_device;
      prm.extent = make_cudaExtent(width, size_t(mp->rhs), 1);
      VBSR_MCUDA(cudaMemcpy3DPeerAsync(&prm, s.stream));
    }
  }
  for (Shard& s : mp->shards) {
    Guard g(s.device);
    VBSR_MCUDA(cudaStreamSynchronize(s.stream));
  }
  return VBSR_OK;
}

// ---- Buffers shared between processes (one process per GPU) -------------------------------------
//
// A replica of B per rank, filled over NVLink by copy-engine peer copies between processes: each
// rank allocates its buffer here (cudaMalloc, so the IPC handle covers exactly the buffer and the
// mapping in another process starts at the buffer's first byte), exports its handle, and maps the
// other ranks' buffers with vbsr_shared_buffer_open. The copies themselves are plain
// cudaMemcpyAsync calls, one per chunk.

struct vbsr_shared_buffer {
  int device = 0;
  int64_t bytes = 0;
  void* ptr = nullptr;
};

vbsr_status vbsr_shared_buffer_create(int device, int64_t bytes, vbsr_shared_buffer** out) {
  clear_error();
  if (out == nullptr || bytes <= 0) return set_error(VBSR_INVALID_ARGUMENT, "bad argument");
  *out = nullptr;
  auto* b = new (std::nothrow) vbsr_shared_buffer;
  if (b == nullptr) return set_error(VBSR_OUT_OF_MEMORY, "host allocation failed");
  Guard g(device);
  b->device = device;
  b->bytes = bytes;
  const cudaError_t e = cudaMalloc(&b->ptr, size_t(bytes));
  if (e != cudaSuccess) {
    delete b;
    return set_error(VBSR_CUDA_ERROR, cudaGetErrorString(e));
  }
  *out = b;
  return VBSR_OK;
}

vbsr_status vbsr_shared_buffer_destroy(vbsr_shared_buffer* b) {
  clear_error();
  if (b == nullptr) return VBSR_OK;
  {
    Guard g(b->device);
    cudaFree(b->ptr);
  }
  delete b;
  return VBSR_OK;
}

vbsr_status vbsr_shared_buffer_ptr(const vbsr_shared_buffer* b, void** ptr) {
  clear_error();
  if (b == nullptr || ptr == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  *ptr = b->ptr;
  return VBSR_OK;
}

vbsr_status vbsr_shared_buffer_export(const vbsr_shared_buffer* b, vbsr_ipc_handle* out) {
  clear_error();
  if (b == nullptr || out == nullptr) return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(out->bytes), "IPC handle size");
  Guard g(b->device);
  cudaIpcMemHandle_t h;
  VBSR_MCUDA(cudaIpcGetMemHandle(&h, b->ptr));
  std::memcpy(out->bytes, &h, sizeof h);
  return VBSR_OK;
}

vbsr_status vbsr_shared_buffer_open(const vbsr_ipc_handle* handle, int device, void** peer_ptr) {
  clear_error();
  if (handle == nullptr || peer_ptr == nullptr)
    return set_error(VBSR_INVALID_ARGUMENT, "null argument");
  Guard g(device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof h);
  VBSR_MCUDA(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return VBSR_OK;
}

vbsr_status vbsr_shared_buffer_close(void* peer_ptr, int device) {
  clear_error();
  if (peer_ptr == nullptr) return VBSR_OK;
  Guard g(device);
  VBSR_MCUDA(cudaIpcCloseMemHandle(peer_ptr));
  return VBSR_OK;
}

vbsr_status vbsr_copy_async(void* dst, const void* src, int64_t bytes, vbsr_stream_t stream) {
  clear_error();
  if (bytes < 0 || (bytes > 0 && (dst == nullptr || src == nullptr)))
    return set_error(VBSR_INVALID_ARGUMENT, "bad copy arguments");
  if (bytes == 0) return VBSR_OK;
  VBSR_MCUDA(cudaMemcpyAsync(dst, src, size_t(bytes), cudaMemcpyDefault,
                             reinterpret_cast<cudaStream_t>(stream)));
  return VBSR_OK;
}

}  // extern "C"
