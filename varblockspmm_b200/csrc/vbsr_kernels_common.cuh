// vbsr_kernels_common.cuh — pieces shared by the engine's kernels: launch parameters, the
// per-team stage descriptors and their register windows, bounded mbarrier waits, the status word.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

typedef unsigned long long u64;

struct KernelParams {
  // B (K x rhs, column-major) as a 3-D tensor (k, j, q) with RHS column c = q * half + j, where
  // half = 8 (rhs <= 32) or 16 (rhs = 64); see the operand stack in vbsr_tc.cuh.
  CUtensorMap b_map;
  int b_boxes;          // TMA boxes per 8-column group (one per quadrant: rhs/half)
  uint32_t b_group_bytes;  // bytes the boxes of one group write to shared memory
  const StageDesc* stages;  // per-team stage descriptors
  const Task* tasks;
  const float* values;  // device-format values
  const float* B;
  float* C;
  long long M, K, nvalues;
  int rhs;
  int* status;
  int drop_stage;       // debug: stage number (team 0 of each CTA) whose copies are withheld
  long long wait_limit; // SM clocks a single wait may take before it is declared stalled
  u64* timing;          // optional: per CTA (start, end) global timer in ns
  int diag;             // VBSR_PLAN_DIAG_* bits (performance analysis only)
};

// ---- stage descriptors -----------------------------------------------------------------------------

struct Stage {
  u64 w0, w1, w2, w3;
  __device__ __forceinline__ long long a_start() const { return (long long)(w0 & 0xfffffffull) * 64; }
  __device__ __forceinline__ int cols() const { return int(((w0 >> 28) & 3u) + 1u) * 8; }
  __device__ __forceinline__ bool first() const { return (w0 >> 30) & 1u; }
  __device__ __forceinline__ bool last() const { return (w0 >> 31) & 1u; }
  __device__ __forceinline__ int h() const { return int(((w0 >> 32) & 7u) + 1u) * 8; }
  __device__ __forceinline__ bool empty() const { return (w0 >> 35) & 1u; }
  __device__ __forceinline__ int n0() const { return int((w0 >> 36) & 7u) * 8; }
  __device__ __forceinline__ int nw() const { return 8 << int((w0 >> 39) & 3u); }
  __device__ __forceinline__ int c_row() const { return int(w1 & 0x7fffffffull); }
  __device__ __forceinline__ int group_col(int g) const {  // scalar column of 8-column group g
    const u64 w = g < 2 ? w2 : w3;
    return int((w >> (32 * (g & 1))) & 0xfffffffull) * 8;
  }
};

// A team's stage list [pos, end) seen through a window of 32 descriptors (lane i holds stage
// wbase + i) and the following window, loaded one window ahead; reading a stage is four
// independent shuffles. All lanes keep identical pos / wbase / end.
struct StageWin {
  ulonglong4 cur, next;
  int pos, wbase, end;

  __device__ __forceinline__ static ulonglong4 load(const StageDesc* s, int i, int end) {
    if (i >= end) return make_ulonglong4(0, 0, 0, 0);
    const ulonglong2* q = reinterpret_cast<const ulonglong2*>(s + i);
    const ulonglong2 a = __ldg(q), b = __ldg(q + 1);
    return make_ulonglong4(a.x, a.y, b.x, b.y);
  }
  __device__ __forceinline__ void init(const StageDesc* s, int b, int e, int lane) {
    pos = b;
    wbase = b;
    end = e;
    cur = load(s, b + lane, e);
    next = load(s, b + 32 + lane, e);
  }
  __device__ __forceinline__ bool done() const { return pos >= end; }
  __device__ __forceinline__ Stage peek() const {
    const int src = (pos - wbase) & 31;
    Stage st;
    st.w0 = __shfl_sync(0xffffffffu, cur.x, src);
    st.w1 = __shfl_sync(0xffffffffu, cur.y, src);
    st.w2 = __shfl_sync(0xffffffffu, cur.z, src);
    st.w3 = __shfl_sync(0xffffffffu, cur.w, src);
    return st;
  }
  __device__ __forceinline__ void advance(const StageDesc* s, int lane) {
    if (++pos - wbase == 32) {
      wbase += 32;
      cur = next;
      next = load(s, wbase + 32 + lane, end);
    }
  }
};

__device__ __forceinline__ void record_status(int* status, int code, int info) {
  if (atomicCAS(status + kStatusCode, 0, code) == 0) status[kStatusInfo] = info;
}

// Warp-collective wait for phase `parity` of `bar`; every lane polls the barrier itself (so each
// lane gets the barrier's acquire ordering), and every decision is made uniformly by the warp.
// mbarrier.try_wait suspends the warp in hardware while the phase is pending, so waiting warps do
// not take issue slots from the warps that compute. Returns false if the CTA aborted or the wait
// exceeded p.wait_limit SM clocks.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, const KernelParams& p,
                                           volatile int* abort_flag, int lane) {
#ifdef VBSR_WAIT_LANE0
  {
    int ok = 0;
    if (lane == 0) ok = mbar_try(bar, parity);
    if (__shfl_sync(0xffffffffu, ok, 0)) {
      __syncwarp();
      return true;
    }
  }
#endif
  if (__all_sync(0xffffffffu, mbar_try(bar, parity))) return true;
  const long long t0 = clock64();
  while (true) {
    if (__all_sync(0xffffffffu, mbar_try(bar, parity))) return true;
    int stop = 0;
    if (lane == 0) {
      if (*abort_flag) {
        stop = 1;
      } else if (clock64() - t0 > p.wait_limit) {
        record_status(p.status, VBSR_TIMEOUT, int(blockIdx.x));
        *abort_flag = 1;
        stop = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}

// ---- producer side (run by each team's leader warp) ----------------------------------------------

// Issue cursor of a team: walks the team's stream ahead of the consumers.
__device__ __forceinline__ u64 global_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace vbsr_b200
