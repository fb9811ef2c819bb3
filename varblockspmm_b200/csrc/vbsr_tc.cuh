// vbsr_tc.cuh — the sm_100a SpMM kernel on 5th-generation tensor cores (tcgen05, TMEM).
//
// Per work item (one block row i: an h x nw tile of C) the kernel computes the transposed product
//     D (M x h) = sum over the row's blocks b of  S_b (M x w) * A_b^T (w x h)
// with tcgen05.mma kind::tf32 (N = h, K = 8 per MMA) and an fp32 accumulator in tensor memory.
//
// FP32 accuracy (3xTF32 with a stacked operand). The tensor core reads an fp32 operand as tf32 by
// ignoring its low 13 mantissa bits (truncation), so for x = hi + lo with hi = trunc_tf32(x) the
// raw value already acts as hi and only lo = x - hi has to be formed (exactly, in fp32). The M side
// of the MMA is the operand stack S: for every RHS column c the raw B value (hi) and its lo part
// sit in two rows of S. One MMA with the raw A then yields B_hi*A_hi and B_lo*A_hi, a second MMA
// with A_lo yields B_hi*A_lo and B_lo*A_lo, and the epilogue adds each column's two rows: all
// cross terms of 3xTF32 in two MMAs per 8 block columns instead of three. M = 64 for nw <= 32 and
// M = 128 for nw = 64. The stack is built per quadrant q (32 TMEM lanes, the part of the
// accumulator one warp may read): with half = M / 8 columns per quadrant, S rows 2*half*q + j and
// 2*half*q + half + j hold hi and lo of column c = half*q + j, and in TMEM (M = 64: row r lives in
// lane r % 16 + 32 * (r / 16); M = 128: lane r) they land in lanes j and half + j of quadrant q, so
// a warp adds them with one shuffle.
//
// CTA = four MMA warps and two feeder warps, one CTA per SM. A single wait-and-release round on an
// mbarrier costs a warp ~200 cycles even when the barrier has already completed, so every warp
// handles only a share of the stages: stage k of the CTA (counting non-empty stages) is fed by
// feeder k % 2 and multiplied by MMA warp k % 4. The CTA's list of stage descriptors (compiled by
// the planner; vbsr_internal.h) is walked by every warp; the ring has D slots, stage k uses slot
// k % D. A feeder copies the stage's A values with one cp.async.bulk (contiguous in the device
// format, which holds every 8-column group as the K-major, 32-byte-swizzled operand tile the MMA
// reads) and the B rows with one 3-D cp.async.bulk.tensor box per group and
// quadrant, placed directly on the stack's hi rows. The owning MMA warp forms the stage's lo parts
// (A_lo next to A, B_lo into the stack; loads batched for memory-level parallelism), fences them
// for the async proxy, issues two MMAs per group into its own partial accumulator, and releases
// the slot with tcgen05.commit. An item's result is read one item later (so the tensor cores work
// on item j while item j-1 is stored): each warp reads its quadrant of the partials that received
// stages with tcgen05.ld, sums them, adds hi and lo rows, and stores h consecutive floats of its
// RHS columns. Every wait is bounded (see wait_phase); after an abort each warp drains its copies
// and MMAs before the CTA releases its tensor memory.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_kernels_common.cuh"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

constexpr int kTcMmaWarps = 4;              // MMA warps (one per TMEM quadrant)
constexpr int kTcFeeders = 2;               // feeder warps
constexpr int kTcWarps = kTcMmaWarps + kTcFeeders;
constexpr int kTcThreads = 32 * kTcWarps;
__host__ __device__ constexpr int stack_m(int nw) { return nw > 32 ? 128 : 64; }
// 8-column groups per stage: 4 (32 block columns) for rhs <= 32, 3 for rhs = 64, so that a slot
// is 24 KB either way and eight slots fit in shared memory.
__host__ __device__ constexpr int stage_groups(int rhs) { return rhs > 32 ? 3 : 4; }
// Slot layout (floats), G = groups per stage: raw A (up to 64 rows x 8G columns, group after
// group, h x 8 each) at 0, A_lo at the same offsets + 512 G, then the operand stacks of the
// groups (M x 8 each) from 1024 G.
__host__ __device__ constexpr int slot_alo(int G) { return 512 * G; }
__host__ __device__ constexpr int slot_stack(int G) { return 1024 * G; }
__host__ __device__ constexpr int slot_floats(int rhs) {
  return slot_stack(stage_groups(rhs)) + stage_groups(rhs) * stack_m(rhs) * 8;
}
// TMEM: 2 accumulator buffers (items alternate) x 4 partials (one per MMA warp) x 64 columns.
constexpr int kTmemAlloc = 512;

// ---- tcgen05 wrappers ------------------------------------------------------------------------------

__device__ __forceinline__ void tc_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// tcgen05.ld of 8 consecutive accumulator columns without waiting (see tc_wait_ld).
__device__ __forceinline__ void tc_ld8_nowait(uint32_t taddr, float* v) {
  uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
               : "r"(taddr)
               : "memory");
  v[0] = __uint_as_float(r0); v[1] = __uint_as_float(r1); v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3); v[4] = __uint_as_float(r4); v[5] = __uint_as_float(r5);
  v[6] = __uint_as_float(r6); v[7] = __uint_as_float(r7);
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// K-major, 32-byte-swizzled operand: rows of 8 tf32 (32 bytes), 8-row atoms 256 bytes apart.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t smem_byte_addr) {
  return uint64_t((smem_byte_addr >> 4) & 0x3FFFu) | (uint64_t(16 >> 4) << 16) |
         (uint64_t(256 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(6) << 61);
}

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major, M x N.
__device__ __forceinline__ uint32_t tf32_idesc(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// lo = x - trunc_tf32(x), exact in fp32.
__device__ __forceinline__ float lo_part(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
__device__ __forceinline__ float4 lo_part4(float4 x) {
  return make_float4(lo_part(x.x), lo_part(x.y), lo_part(x.z), lo_part(x.w));
}

// ---- CTA pieces ----------------------------------------------------------------------------------

// Barriers (shared-memory addresses).
struct CtaBars {
  uint32_t full0, empty0;   // per slot: copies landed / the stage's MMAs have read the slot
  uint32_t acc0, accfree0;  // per accumulator buffer: MMAs of the item done / D read by all warps
  uint32_t drain0;          // per MMA warp: end-of-kernel drain of its MMAs
};

// Optional cycle counters (instrumented builds only): per CTA 16 slots after the 2 * tasks
// start/end timestamps of the timing buffer.
#ifdef VBSR_PROF
#define VBSR_PROF_T0(v) const long long v = clock64()
#define VBSR_PROF_ADD(p, slot, t0)                                                          \
  do {                                                                                     \
    if ((p).timing && (threadIdx.x & 31) == 0)                                             \
      atomicAdd((p).timing + 2 * gridDim.x + 16 * blockIdx.x + (slot),                     \
                (unsigned long long)(clock64() - (t0)));                                   \
  } while (0)
#else
#define VBSR_PROF_T0(v)
#define VBSR_PROF_ADD(p, slot, t0) do { } while (0)
#endif

// Feeder warp f: fills the slots of the stages k with k % kTcFeeders == f, each once the MMAs of
// the slot's previous stage have completed.
template <bool CHECK>
__device__ void tc_feeder(const KernelParams& p, const Task& task, float* slots,
                          const CtaBars& cb, int f, int lane, volatile int* abort_flag) {
  const int D = task.stages, SF = task.stage_floats;
  StageWin win;
  win.init(p.stages, task.team_off[0], task.team_off[1], lane);
  int k = 0;  // non-empty stages seen
  uint32_t filled = 0, lastpar = 0;
  const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
  VBSR_PROF_T0(t_all);
  while (!win.done()) {
    const Stage st = win.peek();
    win.advance(p.stages, lane);
    if (st.empty()) continue;
    const int kk = k++;
    if (kk % kTcFeeders != f) continue;
    const int s = kk % D;
    const uint32_t ph = uint32_t(kk / D) & 1u;
    const uint32_t full_bar = cb.full0 + 8u * s;
    VBSR_PROF_T0(t_w);
    if (!wait_phase(cb.empty0 + 8u * s, ph ^ 1u, p, abort_flag, lane)) break;
    VBSR_PROF_ADD(p, 7, t_w);
    const int h = st.h(), nw = st.nw(), n0 = st.n0(), cols = st.cols(), groups = cols >> 3;
    const long long a0 = st.a_start();
    bool ok = true;
    if (CHECK) {
      ok = a0 + (long long)h * cols <= p.nvalues && n0 + nw <= p.rhs && nw <= 64 &&
           stack_m(nw) == stack_m(p.rhs) && cols <= task.stage_cols;
      for (int g = 0; g < groups; ++g) ok = ok && st.group_col(g) + 8 <= p.K;
    }
    if (kk == p.drop_stage) {
      // withhold the stage entirely (debug): no arrival, no copies
    } else if ((p.diag & VBSR_PLAN_DIAG_SKIP_COPIES) || !ok) {
      if (lane == 0) {
        if (!ok) record_status(p.status, VBSR_BOUNDS_VIOLATION, int(blockIdx.x));
        mbar_arrive(full_bar);  // release the MMA warp without touching memory
      }
    } else {
      float* sp = slots + s * SF;
      const int M = stack_m(nw), half = M / 8, nb = p.b_boxes;
      if (lane == 0) {
        mbar_arrive_expect_tx(full_bar,
                              uint32_t(h * 4 * cols) + uint32_t(groups) * p.b_group_bytes);
        bulk_g2s(smem_addr(sp), p.values + a0, uint32_t(h * 4 * cols), full_bar, pol_a);
      } else if (lane <= groups * nb) {
        const int g = (lane - 1) / nb, q = (lane - 1) % nb;
        tensor3d_g2s(smem_addr(sp + slot_stack(task.stage_cols >> 3) + g * M * 8 + q * 2 * half * 8), &p.b_map,
                     st.group_col(g), 0, n0 / half + q, full_bar, pol_b);
      }
      filled |= 1u << s;
      lastpar = (lastpar & ~(1u << s)) | (ph << s);
    }
  }
  VBSR_PROF_ADD(p, 6, t_all);
  // After an abort wait (bounded) for every copy still in flight before the CTA exits.
  if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
    for (int sl = 0; sl < D; ++sl) {
      if (!(filled & (1u << sl))) continue;
      const uint32_t bar = cb.full0 + 8u * sl;
      const uint32_t par = (lastpar >> sl) & 1u;
      const long long t1 = clock64();
      while (!mbar_try(bar, par) && clock64() - t1 < p.wait_limit) {
      }
    }
  }
}

// An item as the MMA warps remember it for the lagged epilogue.
struct ItemInfo {
  int h, nw, n0, c_row;
  int k0;  // the CTA's running non-empty stage count at the item's first stage, mod 4
  int n;   // non-empty stages of the item
};

// Epilogue of one item: D -> C, by MMA warp w (TMEM quadrant w). Partial k (64 columns further
// for each k) holds the stages owned by warp k; only partials that received a stage are read.
// Lane j < half of quadrant w holds hi of RHS column n0 + half*w + j, lane half + j its lo.
template <bool CHECK>
__device__ __forceinline__ bool tc_epilogue(const KernelParams& p, const CtaBars& cb, int buf,
                                            uint32_t parity, uint32_t tmem_buf, int w, int lane,
                                            const ItemInfo& it, volatile int* abort_flag) {
  VBSR_PROF_T0(t_w);
  if (!wait_phase(cb.acc0 + 8u * buf, parity, p, abort_flag, lane)) return false;
  VBSR_PROF_ADD(p, 4, t_w);
  tc_fence_after();
  const int h = it.h;
  const int M = stack_m(it.nw), half = M / 8, quads = it.nw / half;
  uint32_t use = 0;
  if (!(p.diag & VBSR_PLAN_DIAG_SKIP_MATH))
    for (int i = 0; i < 4 && i < it.n; ++i) use |= 1u << ((it.k0 + i) & 3);
  if (w < quads) {
    const uint32_t taddr = tmem_buf + (uint32_t(32 * w) << 16);
    const bool store = !(CHECK && ((long long)it.c_row + h > p.M || it.n0 + it.nw > p.rhs));
    if (CHECK && !store && w == 0 && lane == 0)
      record_status(p.status, VBSR_BOUNDS_VIOLATION, it.c_row);
    const int col = it.n0 + half * w + lane;
    float4* dst = reinterpret_cast<float4*>(p.C + (long long)col * p.M + it.c_row);
    // passes of 16 accumulator columns: 4 partials x 16 values in flight per pass
    for (int c0 = 0; c0 < h; c0 += 16) {
      const bool two = c0 + 8 < h;
      float v[4][16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (use & (1u << k)) {
          tc_ld8_nowait(taddr + uint32_t(64 * k + c0), v[k]);
          if (two) tc_ld8_nowait(taddr + uint32_t(64 * k + c0 + 8), v[k] + 8);
        }
      }
      tc_wait_ld();
      float r[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) a += (use & (1u << k)) ? v[k][i] : 0.0f;
        r[i] = a + __shfl_down_sync(0xffffffffu, a, half);
      }
      if (lane < half && store) {
        dst[c0 / 4] = make_float4(r[0], r[1], r[2], r[3]);
        dst[c0 / 4 + 1] = make_float4(r[4], r[5], r[6], r[7]);
        if (two) {
          dst[c0 / 4 + 2] = make_float4(r[8], r[9], r[10], r[11]);
          dst[c0 / 4 + 3] = make_float4(r[12], r[13], r[14], r[15]);
        }
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(cb.accfree0 + 8u * buf);  // this warp is done with the buffer
  return true;
}

// lo parts of a whole stage: A_lo next to A (2h float4s per group, groups contiguous) and B_lo
// into the stacks' lo rows. Eight independent loads per lane are in flight before the stores.
__device__ __forceinline__ void split_stage(float* sp, int G, int groups, int h, int nw, int lane) {
  const float4* a = reinterpret_cast<const float4*>(sp);
  float4* alo = reinterpret_cast<float4*>(sp + slot_alo(G));
  const int na = 2 * h * groups;
  for (int i0 = 0; i0 < na; i0 += 256) {
    float4 x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < na) x[u] = a[i];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < na) alo[i] = lo_part4(x[u]);
    }
  }
  const int M = stack_m(nw), half = M / 8;
  float4* stk = reinterpret_cast<float4*>(sp + slot_stack(G));
  // per group: M * 2 float4s; hi rows of quadrant q are float4s [4*half*q, 4*half*q + 2*half),
  // the lo rows 2*half float4s later
  const int per_group = 2 * nw, nb = per_group * groups;
  for (int i0 = 0; i0 < nb; i0 += 256) {
    float4 x[8];
    int o[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 32 * u + lane;
      const int g = i / per_group, r = i - g * per_group;
      const int q = r / (2 * half), rr = r - q * 2 * half;
      o[u] = g * 2 * M + 4 * half * q + rr;
      if (i < nb) x[u] = stk[o[u]];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < nb) stk[o[u] + 2 * half] = lo_part4(x[u]);
    }
  }
}

// MMA warp w (0..3): splits and multiplies the stages it owns (k % 4 == w), and stores each
// item's result (its TMEM quadrant) one item later.
template <bool CHECK>
__device__ void tc_mma_warp(const KernelParams& p, const Task& task, float* slots,
                            const CtaBars& cb, uint32_t tmem_base, int w, int lane,
                            volatile int* abort_flag) {
  const int D = task.stages, SF = task.stage_floats, G = task.stage_cols >> 3;
  StageWin win;
  win.init(p.stages, task.team_off[0], task.team_off[1], lane);
  int k = 0;       // non-empty stages seen
  int j = 0;       // items started
  ItemInfo cur{8, 8, 0, 0, 0, 0}, prev{8, 8, 0, 0, 0, 0};
  uint32_t tmem_d = tmem_base, idesc = 0, started = 0;
  const bool math = !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH);
  const uint32_t sbase = smem_addr(slots);
  bool ok = true;
  VBSR_PROF_T0(t_all);
  while (!win.done()) {
    const Stage st = win.peek();
    win.advance(p.stages, lane);
    if (st.first()) {
      cur = ItemInfo{st.h(), st.nw(), st.n0(), st.c_row(), k & 3, 0};
      const int buf = j & 1;
      // the buffer's previous item (j-2) must have been read out by every warp
      VBSR_PROF_T0(t_f);
      if (j >= 2 && !wait_phase(cb.accfree0 + 8u * buf, uint32_t(((j - 2) >> 1) & 1), p,
                                abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 5, t_f);
      tc_fence_after();
      tmem_d = tmem_base + uint32_t(256 * buf + 64 * w);
      idesc = tf32_idesc(stack_m(cur.nw), cur.h);
      started = 0;
    }
    if (!st.empty()) {
      const int kk = k++;
      ++cur.n;
      if ((kk & 3) == w) {
        const int s = kk % D;
        VBSR_PROF_T0(t_w);
        if (!wait_phase(cb.full0 + 8u * s, uint32_t(kk / D) & 1u, p, abort_flag, lane)) {
          ok = false;
          break;
        }
        VBSR_PROF_ADD(p, 1, t_w);
        const int groups = st.cols() >> 3;
        if (math) {
          VBSR_PROF_T0(t_s);
          split_stage(slots + s * SF, G, groups, cur.h, cur.nw, lane);
          fence_proxy_async_smem();
          __syncwarp();
          VBSR_PROF_ADD(p, 2, t_s);
        }
        VBSR_PROF_T0(t_m);
        if (lane == 0) {
          if (math) {
            tc_fence_after();
            const uint32_t sa = sbase + 4u * uint32_t(s * SF);
            const int M = stack_m(cur.nw);
            for (int g = 0; g < groups; ++g) {
              const uint64_t sdesc = sw32_desc(sa + 4u * uint32_t(slot_stack(G) + g * M * 8));
              const uint64_t adesc = sw32_desc(sa + 4u * uint32_t(g * 8 * cur.h));
              const uint64_t ldesc = sw32_desc(sa + 4u * uint32_t(slot_alo(G) + g * 8 * cur.h));
              tc_mma_tf32(tmem_d, sdesc, adesc, idesc, started);
              tc_mma_tf32(tmem_d, sdesc, ldesc, idesc, 1u);
              started = 1u;
            }
          }
          tc_commit(cb.empty0 + 8u * s);  // the slot is free once these MMAs have read it
        }
        __syncwarp();
        VBSR_PROF_ADD(p, 3, t_m);
      }
    }
    if (st.last()) {
      if (lane == 0) tc_commit(cb.acc0 + 8u * (j & 1));  // this warp's part of the item is issued
      __syncwarp();
      if (j > 0) {
        const int pj = j - 1;
        VBSR_PROF_T0(t_e);
        if (!tc_epilogue<CHECK>(p, cb, pj & 1, uint32_t((pj >> 1) & 1),
                                tmem_base + uint32_t(256 * (pj & 1)), w, lane, prev, abort_flag)) {
          ok = false;
          break;
        }
        VBSR_PROF_ADD(p, 8, t_e);
      }
      prev = cur;
      ++j;
    }
  }
  if (ok && j > 0) {
    const int pj = j - 1;
    tc_epilogue<CHECK>(p, cb, pj & 1, uint32_t((pj >> 1) & 1), tmem_base + uint32_t(256 * (pj & 1)),
                       w, lane, prev, abort_flag);
  }
  VBSR_PROF_ADD(p, 0, t_all);
  // Every MMA this warp issued has completed before the CTA releases its tensor memory (bounded).
  if (lane == 0) tc_commit(cb.drain0 + 8u * w);
  __syncwarp();
  {
    const long long t0 = clock64();
    while (!mbar_try(cb.drain0 + 8u * w, 0) && clock64() - t0 < p.wait_limit) {
    }
  }
}

template <bool CHECK>
__global__ void __launch_bounds__(kTcThreads, 1) spmm_tc_kernel(const __grid_constant__ KernelParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  float* slots = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[2][kMaxStages];  // full, empty
  __shared__ __align__(8) uint64_t accbars[2][2];        // acc done, acc free
  __shared__ __align__(8) uint64_t drainbars[kTcMmaWarps];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const Task task = p.tasks[blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tc_alloc(smem_addr(&tmem_slot), kTmemAlloc);
    tc_relinquish();
  }
  if (threadIdx.x == 32) {
    if (p.timing) p.timing[2 * blockIdx.x] = global_ns();
    for (int s = 0; s < task.stages; ++s) {
      mbar_init(smem_addr(&bars[0][s]), 1u);                    // TMA: one arrival + tx bytes
      mbar_init(smem_addr(&bars[1][s]), 1u);                    // the owner's tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&accbars[0][b]), uint32_t(kTcMmaWarps));
      mbar_init(smem_addr(&accbars[1][b]), uint32_t(kTcMmaWarps));
    }
    for (int w = 0; w < kTcMmaWarps; ++w) mbar_init(smem_addr(&drainbars[w]), 1u);
    abort_flag = 0;
    mbar_fence_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  CtaBars cb;
  cb.full0 = smem_addr(&bars[0][0]);
  cb.empty0 = smem_addr(&bars[1][0]);
  cb.acc0 = smem_addr(&accbars[0][0]);
  cb.accfree0 = smem_addr(&accbars[1][0]);
  cb.drain0 = smem_addr(&drainbars[0]);
  if (warp < kTcMmaWarps)
    tc_mma_warp<CHECK>(p, task, slots, cb, tmem_base, warp, lane, &abort_flag);
  else
    tc_feeder<CHECK>(p, task, slots, cb, warp - kTcMmaWarps, lane, &abort_flag);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem_base, kTmemAlloc);
  }
  if (threadIdx.x == 0 && p.timing) p.timing[2 * blockIdx.x + 1] = global_ns();
}

}  // namespace vbsr_b200
