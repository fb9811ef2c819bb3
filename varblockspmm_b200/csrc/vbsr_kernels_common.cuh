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
  const StageDesc* stages;  // stage descriptors of all CTAs
  const ItemDesc* items;    // item descriptors of all CTAs
  const Task* tasks;
  const float* values;  // device-format values
  const float* B;
  const float* bstack;  // B's operand stacks (bstack_kernel), M x 8 floats per 8-column group
  float* C;
  long long M, K, nvalues;
  int rhs;
  int* status;
  int drop_stage;       // debug: stage number (team 0 of each CTA) whose copies are withheld
  long long wait_limit; // SM clocks a single wait may take before it is declared stalled
  u64* timing;          // optional: per CTA (start, end) global timer in ns
  u64* prof;            // instrumented builds only (VBSR_PROF): 16 cycle counters per CTA
  int diag;             // VBSR_PLAN_DIAG_* bits (performance analysis only)
  // Fused pre-pass: the SpMM's own CTAs form the operand stacks, then arrive on this word (a
  // self-resetting grid arrival counter, see stack_arrive); nullptr: a separate pre-pass launch.
  uint32_t* stack_flag;
};

// ---- stage descriptors -----------------------------------------------------------------------------

struct Stage {
  u64 w0, g[6];  // descriptor words 0 and 2..7
  __device__ __forceinline__ long long a_start() const { return (long long)(w0 & 0xfffffffull) * 64; }
  __device__ __forceinline__ int groups() const { return int((w0 >> 28) & 15u) + 1; }
  __device__ __forceinline__ int h() const { return int(((w0 >> 32) & 7u) + 1u) * 8; }
  __device__ __forceinline__ int n0() const { return int((w0 >> 36) & 7u) * 8; }
  __device__ __forceinline__ int nw() const { return 8 << int((w0 >> 39) & 3u); }
  // height of the stage's block row; h() < H() when the item is a row part of it (groups are then
  // H * 8 floats apart in the device format, and the part's h rows start a_start() into each)
  __device__ __forceinline__ int H() const { return int(((w0 >> 41) & 7u) + 1u) * 8; }
  // bytes from the stage's first A value to the end of its last group's rows
  __device__ __forceinline__ long long a_span_bytes() const {
    return 32ll * (H() * (groups() - 1) + h());
  }
  __device__ __forceinline__ int group_col(int i) const {  // scalar column of group i
    const int k = i >> 1;  // selected without indexing, so the words stay in registers
    const u64 w = k == 0 ? g[0]
                         : (k == 1 ? g[1] : (k == 2 ? g[2] : (k == 3 ? g[3] : (k == 4 ? g[4] : g[5]))));
    return int((w >> (32 * (i & 1))) & 0xfffffffull) * 8;
  }
};

struct Item {
  uint32_t c_row, shape, k0, n;
  __device__ __forceinline__ int h() const { return int((shape & 7u) + 1u) * 8; }
  __device__ __forceinline__ int n0() const { return int((shape >> 3) & 7u) * 8; }
  __device__ __forceinline__ int nw() const { return 8 << int((shape >> 6) & 3u); }
  __device__ __forceinline__ int groups() const { return int(shape >> 8); }
  // groups of the item's stage i (0 <= i < n), with G groups per full stage (stage_groups(h, rhs))
  __device__ __forceinline__ int stage_groups(int i, int G) const {
    const int r = groups() - i * G;
    return r < G ? r : G;
  }
};

// Every `stride`-th stage descriptor from `first` on (count of them), seen through a window of 32
// (lane i holds element wbase + i) and the following window, loaded one window ahead; reading a
// stage is fourteen shuffles. All lanes keep identical pos / wbase.
struct StageWin {
  Stage cur, next;
  const StageDesc* base;
  int pos, wbase, count, stride;

  __device__ __forceinline__ Stage load(int i) const {
    Stage st{};
    if (i >= count) return st;
    const ulonglong2* q = reinterpret_cast<const ulonglong2*>(base + (long long)i * stride);
    const ulonglong2 a = __ldg(q), b = __ldg(q + 1), c = __ldg(q + 2), d = __ldg(q + 3);
    st.w0 = a.x;
    st.g[0] = b.x;
    st.g[1] = b.y;
    st.g[2] = c.x;
    st.g[3] = c.y;
    st.g[4] = d.x;
    st.g[5] = d.y;
    return st;
  }
  __device__ __forceinline__ void init(const StageDesc* s, int first, int stride_, int n, int lane) {
    base = s + first;
    stride = stride_;
    count = first < n ? (n - first + stride_ - 1) / stride_ : 0;
    pos = 0;
    wbase = 0;
    cur = load(lane);
    next = load(32 + lane);
  }
  __device__ __forceinline__ Stage get() const {
    const int src = (pos - wbase) & 31;
    Stage st;
    st.w0 = __shfl_sync(0xffffffffu, cur.w0, src);
#pragma unroll
    for (int i = 0; i < 6; ++i) st.g[i] = __shfl_sync(0xffffffffu, cur.g[i], src);
    return st;
  }
  // Word 0 of the descriptor d < 32 positions ahead (from this window or the next).
  __device__ __forceinline__ u64 word0_ahead(int d) const {
    const int idx = pos - wbase + d;
    const int src = idx & 31;
    const u64 va = __shfl_sync(0xffffffffu, cur.w0, src), vb = __shfl_sync(0xffffffffu, next.w0, src);
    return idx < 32 ? va : vb;
  }
  __device__ __forceinline__ bool has_ahead(int d) const { return pos + d < count; }
  __device__ __forceinline__ void advance(int lane) {
    if (++pos - wbase == 32) {
      wbase += 32;
      cur = next;
      next = load(wbase + 32 + lane);
    }
  }
};

// The CTA's item descriptors through a window of 32, like StageWin (stride 1).
struct ItemWin {
  uint4 cur, next;
  const ItemDesc* base;
  int pos, wbase, count;

  __device__ __forceinline__ uint4 load(int i) const {
    if (i >= count) return make_uint4(0, 0, 0, 0);
    return __ldg(reinterpret_cast<const uint4*>(base + i));
  }
  __device__ __forceinline__ void init(const ItemDesc* s, int n, int lane) {
    base = s;
    count = n;
    pos = 0;
    wbase = 0;
    cur = load(lane);
    next = load(32 + lane);
  }
  __device__ __forceinline__ bool done() const { return pos >= count; }
  __device__ __forceinline__ Item get() const {
    const int src = (pos - wbase) & 31;
    Item it;
    it.c_row = __shfl_sync(0xffffffffu, cur.x, src);
    it.shape = __shfl_sync(0xffffffffu, cur.y, src);
    it.k0 = __shfl_sync(0xffffffffu, cur.z, src);
    it.n = __shfl_sync(0xffffffffu, cur.w, src);
    return it;
  }
  __device__ __forceinline__ void advance(int lane) {
    if (++pos - wbase == 32) {
      wbase += 32;
      cur = next;
      next = load(wbase + 32 + lane);
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
constexpr unsigned kWaitHintNs = 20000u;  // suspend-time hint of one try_wait probe
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, const KernelParams& p,
                                           volatile int* abort_flag, int lane) {
  if (__all_sync(0xffffffffu, mbar_try(bar, parity))) return true;
  const long long t0 = clock64();
  while (true) {
    // suspended in hardware for up to ~20 us per probe, so a waiting warp issues few instructions
    if (__all_sync(0xffffffffu, mbar_try_hint(bar, parity, kWaitHintNs))) return true;
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
