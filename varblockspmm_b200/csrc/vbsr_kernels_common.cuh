// vbsr_kernels_common.cuh — pieces shared by the engine's kernels: launch parameters, the
// per-team instruction-stream entries and their register windows, bounded mbarrier waits, the
// status word, and the team's issue cursor.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

typedef unsigned long long u64;

struct KernelParams {
  CUtensorMap b_full;   // B as a K x rhs tensor, box 8 columns x rhs rows
  CUtensorMap b_half;   // same, box 8 columns x rhs/2 rows (items of split rows)
  const u64* stream;    // per-team instruction streams
  const Task* tasks;
  const float* values;  // re-laid-out values
  const float* B;
  float* C;
  long long M, K, nvalues;
  int rhs;
  int* status;
  int drop_stage;       // debug: chunk number (per CTA, team 0) the producer withholds; < 0 off
  long long wait_limit; // SM clocks a single wait may take before it is declared stalled
  u64* timing;          // optional: per CTA (start, end) global timer in ns
  int diag;             // VBSR_PLAN_DIAG_* bits (performance analysis only)
};

// ---- stream entries ------------------------------------------------------------------------------

__device__ __forceinline__ bool is_header(u64 e) { return (e >> 63) != 0; }
__device__ __forceinline__ int hdr_crow(u64 e) { return int(e & 0x7fffffffull); }
__device__ __forceinline__ int hdr_h(u64 e) { return int(((e >> 31) & 7u) + 1u) * 8; }
__device__ __forceinline__ int hdr_n0(u64 e) { return int((e >> 34) & 7u) * 8; }
__device__ __forceinline__ int hdr_nw(u64 e) { return 8 << int((e >> 37) & 3u); }
__device__ __forceinline__ long long chk_val(u64 e) { return (long long)(e & 0xfffffffull) * 64; }
__device__ __forceinline__ long long chk_colk(u64 e) { return (long long)((e >> 28) & 0xfffffffull) * 8; }
__device__ __forceinline__ int chk_w(u64 e) { return int(((e >> 56) & 7u) + 1u) * 8; }
__device__ __forceinline__ int chk_k0(u64 e) { return int((e >> 59) & 1u) * 32; }
__device__ __forceinline__ int chk_kc(u64 e) { return int(((e >> 60) & 3u) + 1u) * 8; }
__device__ __forceinline__ bool chk_stage_end(u64 e) { return ((e >> 62) & 1u) != 0; }

// A team stream [pos, end) seen through a window of 32 entries (lane i holds entry wbase + i) and
// the following window, loaded one window ahead. All lanes keep identical pos/wbase/end.
struct StreamWin {
  u64 cur, next;
  int pos, wbase, end;

  __device__ __forceinline__ void init(const u64* s, int b, int e, int lane) {
    pos = b;
    wbase = b;
    end = e;
    cur = (b + lane < e) ? __ldg(s + b + lane) : 0ull;
    next = (b + 32 + lane < e) ? __ldg(s + b + 32 + lane) : 0ull;
  }
  __device__ __forceinline__ bool done() const { return pos >= end; }
  __device__ __forceinline__ u64 peek() const {
    return __shfl_sync(0xffffffffu, cur, (pos - wbase) & 31);
  }
  __device__ __forceinline__ void advance(const u64* s, int lane) {
    if (++pos - wbase == 32) {
      wbase += 32;
      cur = next;
      const int i = wbase + 32 + lane;
      next = (i < end) ? __ldg(s + i) : 0ull;
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
struct Issuer {
  StreamWin win;
  int h, n0, nw;        // item the cursor is in
  int slot;             // next ring slot
  uint32_t ph;          // ring phase of that slot
  uint32_t filled;      // bit s: slot s has been filled at least once
  uint32_t lastpar;     // bit s: phase parity of the last fill of slot s
  int issued;           // chunks issued so far (debug drop hook)
};

__device__ __forceinline__ u64 global_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace vbsr_b200
