// vbsr_tc.cuh — the sm_100a SpMM kernel on 5th-generation tensor cores (tcgen05, TMEM).
//
// Per work item (one block row i: an h x nw tile of C) the kernel computes the transposed product
//     D (64 x h) = sum over the row's blocks b of  B_b^T (64 x w) * A_b^T (w x h)
// with tcgen05.mma kind::tf32 (M = 64: the item's nw RHS columns, padded; N = h; K = 8 per MMA) and
// an fp32 accumulator in tensor memory. FP32 accuracy comes from the 3xTF32 split: every staged
// operand x is split into hi = x with its low 13 mantissa bits cleared (exactly representable in
// tf32) and lo = x - hi (exact in fp32), and three MMAs accumulate hi*hi + hi*lo + lo*hi. The
// dropped lo*lo term and the tf32 conversion of lo are below 2^-19 relative per product.
//
// CTA = two teams, one CTA per SM. A team has four worker warps (warp w sits in TMEM sub-partition
// w, so together they read all 64 accumulator rows) and two issuer warps. A single thread can issue
// a tcgen05.mma only every ~55 cycles, while the tensor core overlaps MMAs from several issuers, so
// the two issuers of a team take alternate 8-column groups, each into its own partial accumulator,
// and the epilogue adds the two partials. Each team walks its list of stage descriptors (compiled
// by the planner; vbsr_internal.h) and owns a ring of D stages of 32 block columns:
//   * issuer 0 keeps the TMA ring D-1 stages ahead: the stage's A values with one cp.async.bulk
//     (contiguous in the device format, which already holds every 8-column group as the K-major
//     32-byte-swizzled operand tile the MMA reads), B with one 2-D cp.async.bulk.tensor box of
//     8 columns x nw rows (SWIZZLE_32B) per group;
//   * when a stage lands, the team's 128 threads split A and B into hi and lo in a compute slot,
//     fence the generic-proxy writes for the async proxy and arrive on the slot's "split"
//     mbarrier (one arrival per warp; no named barriers, so every wait stays bounded), which also
//     frees the landing slot for the next copies;
//   * the issuers' MMAs read the compute slot; their tcgen05.commit frees it;
//   * at the end of an item the thread commits to the team's accumulator barrier, and the four
//     warps load D with tcgen05.ld and store C (each thread: one RHS column, h consecutive rows).
// Every wait is bounded (see wait_phase); after an abort each leader drains its copies and MMAs
// before the CTA releases its tensor memory.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_kernels_common.cuh"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

#ifndef VBSR_TC_TEAMS
#define VBSR_TC_TEAMS 2
#endif
constexpr int kTcTeams = VBSR_TC_TEAMS;     // teams per CTA
constexpr int kTcIssuers = 2;               // MMA-issuing warps per team
constexpr int kTcWarps = (4 + kTcIssuers) * kTcTeams;  // per team: 4 worker warps + issuers
constexpr int kTcThreads = 32 * kTcWarps;
constexpr int kTcCols = 32;                 // block columns per stage
constexpr int kTcM = 64;                    // MMA M (RHS columns, padded)
// Two rings per team (floats):
//   landing slot (kTcLand of them, filled by TMA): A raw at kLdA (up to 64 rows x 32 columns),
//     B raw boxes at kLdB (one 8-column box per group, padded to 64 rows);
//   compute slot (kTcComp of them, read by the MMAs): A hi | A lo | B hi | B lo.
// A landing slot is free again as soon as the workers have split it; a compute slot when the MMAs
// that read it have completed.
constexpr int kBoxFloats = kTcM * 8;                    // one 8-column B box, padded to 64 rows
constexpr int kLdA = 0;
constexpr int kLdB = 64 * kTcCols;
constexpr int kLandFloats = kLdB + (kTcCols / 8) * kBoxFloats;       // 4096 floats = 16 KB
constexpr int kCpA = 0, kCpALo = 64 * kTcCols;
constexpr int kCpB = 2 * 64 * kTcCols, kCpBLo = kCpB + (kTcCols / 8) * kBoxFloats;
constexpr int kCompFloats = kCpBLo + (kTcCols / 8) * kBoxFloats;     // 8192 floats = 32 KB
constexpr int kTcComp = 2;                                           // compute slots per team
constexpr int kTcStageFloats = kLandFloats;  // (reported as the stage size)
// per team: 2 buffers (items alternate) x kTcIssuers partial accumulators x 64 columns
constexpr int kTmemCols = 2 * kTcIssuers * 64 * kTcTeams;
constexpr int kTmemAlloc = kTmemCols <= 128 ? 128 : (kTmemCols <= 256 ? 256 : 512);
static_assert(kTmemCols <= 512, "tensor memory holds 512 columns");
constexpr int kTeamTmem = 2 * kTcIssuers * 64;          // columns per team

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

// ---- team pieces --------------------------------------------------------------------------------

// Barriers of one team (shared-memory addresses).
struct TeamBars {
  uint32_t full0, landfree0;       // per landing slot: TMA landed / split done reading it
  uint32_t split0, cfree0;         // per compute slot: hi-lo written / MMAs done reading it
  uint32_t acc0, accfree0;         // per accumulator buffer: MMAs of the item done / D read
  uint32_t drain;                  // end-of-kernel drain of the issuers' MMAs
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

// TMA feed cursor (issuer 0 of a team): runs D-1 non-empty stages ahead of the MMAs.
struct Feeder {
  StageWin win;
  int slot;             // next ring slot
  uint32_t ph;          // ring phase of that slot
  uint32_t filled;      // bit s: slot s has been filled at least once
  uint32_t lastpar;     // bit s: phase parity of the last fill of slot s
  int issued;           // stages issued so far (debug drop hook)
};

// Issues the copies of the next non-empty stage into the next landing slot, once the workers have
// split the slot's previous contents. Warp-collective. Returns false on abort.
template <bool CHECK>
__device__ __forceinline__ bool feed_next(const KernelParams& p, Feeder& f, float* team_stages,
                                          int D, const TeamBars& tb, int team, int lane,
                                          volatile int* abort_flag) {
  while (!f.win.done() && f.win.peek().empty()) f.win.advance(p.stages, lane);
  if (f.win.done()) return true;
  const Stage st = f.win.peek();
  f.win.advance(p.stages, lane);
  const int s = f.slot;
  const uint32_t full_bar = tb.full0 + 8u * s;
  if (!wait_phase(tb.landfree0 + 8u * s, f.ph ^ 1u, p, abort_flag, lane)) return false;
  const int h = st.h(), nw = st.nw(), n0 = st.n0(), cols = st.cols();
  const long long a0 = st.a_start();
  const bool drop = (team == 0 && f.issued == p.drop_stage);
  ++f.issued;
  bool ok = true;
  if (CHECK) {
    ok = a0 + (long long)h * cols <= p.nvalues && n0 + nw <= p.rhs && nw <= kTcM;
    for (int g = 0; g < cols / 8; ++g) ok = ok && st.group_col(g) + 8 <= p.K;
  }
  if (drop) {
    // withhold the stage entirely (debug): no arrival, no copies
  } else if ((p.diag & VBSR_PLAN_DIAG_SKIP_COPIES) || !ok) {
    if (lane == 0) {
      if (!ok) record_status(p.status, VBSR_BOUNDS_VIOLATION, int(blockIdx.x));
      mbar_arrive(full_bar);  // release the workers without touching memory
    }
  } else {
    float* sp = team_stages + s * kLandFloats;
    if (lane == 0) {
      mbar_arrive_expect_tx(full_bar, uint32_t((h + nw) * 4 * cols));
      bulk_g2s(smem_addr(sp + kLdA), p.values + a0, uint32_t(h * 4 * cols), full_bar,
               policy_evict_first());
    } else if (lane <= (cols >> 3)) {
      const int g = lane - 1;
      const CUtensorMap* map = (nw == p.rhs) ? &p.b_full : &p.b_half;
      tensor2d_g2s(smem_addr(sp + kLdB + g * kBoxFloats), map, st.group_col(g), n0, full_bar,
                   policy_evict_last());
    }
    f.filled |= 1u << s;
    f.lastpar = (f.lastpar & ~(1u << s)) | (f.ph << s);
  }
  if (++f.slot == D) {
    f.slot = 0;
    f.ph ^= 1u;
  }
  return true;
}

// hi = x with the low 13 mantissa bits cleared, lo = x - hi, over n4 float4s read at src and
// written at the same positions of dst_hi / dst_lo, spread over the team's 128 worker threads.
__device__ __forceinline__ void split_hi_lo(const float* src, float* dst_hi, float* dst_lo, int n4,
                                            int tid) {
  for (int i = tid; i < n4; i += 128) {
    const float4 x = reinterpret_cast<const float4*>(src)[i];
    float4 hi, lo;
    hi.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    hi.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    hi.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    hi.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    lo.x = x.x - hi.x;
    lo.y = x.y - hi.y;
    lo.z = x.z - hi.z;
    lo.w = x.w - hi.w;
    reinterpret_cast<float4*>(dst_hi)[i] = hi;
    reinterpret_cast<float4*>(dst_lo)[i] = lo;
  }
}

// An item as the workers remember it for the lagged epilogue.
struct ItemInfo {
  int h, nw, n0, c_row, groups;
};

// Epilogue of one item: D -> C. Each worker warp reads its TMEM sub-partition; thread `lane` < 16
// of warp wq holds accumulator row m = 16*wq + lane = RHS column n0 + m, i.e.
// C[c_row .. c_row+h-1, n0+m], stored as h consecutive floats. Partial 0 holds the even 8-column
// groups, partial 1 (64 columns further) the odd ones.
template <bool CHECK>
__device__ __forceinline__ bool tc_epilogue(const KernelParams& p, const TeamBars& tb, int buf,
                                            uint32_t parity, uint32_t tmem_acc, int wq, int lane,
                                            const ItemInfo& it, volatile int* abort_flag) {
  if (!wait_phase(tb.acc0 + 8u * buf, parity, p, abort_flag, lane)) return false;
  tc_fence_after();
  const int h = it.h;
  const uint32_t taddr = tmem_acc + (uint32_t(32 * wq) << 16);
  const int m = 16 * wq + lane;
  const bool store = !(CHECK && ((long long)it.c_row + h > p.M || it.n0 + it.nw > p.rhs));
  if (CHECK && !store && wq == 0 && lane == 0)
    record_status(p.status, VBSR_BOUNDS_VIOLATION, it.c_row);
  const bool use0 = it.groups > 0 && !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH);
  const bool use1 = it.groups > 1 && !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH);
  float4* dst = reinterpret_cast<float4*>(p.C + (long long)(it.n0 + m) * p.M + it.c_row);
  // two passes of up to 32 columns (both partials), to bound the registers
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float v[32], u[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = 32 * half + 8 * c;
      if (col < h) {
        tc_ld8_nowait(taddr + uint32_t(col), v + 8 * c);
        tc_ld8_nowait(taddr + 64u + uint32_t(col), u + 8 * c);
      }
    }
    tc_wait_ld();
    if (lane < 16 && m < it.nw && store) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int col = 32 * half + 8 * c;
        if (col < h) {
          float r[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            r[i] = (use0 ? v[8 * c + i] : 0.0f) + (use1 ? u[8 * c + i] : 0.0f);
          dst[col / 4] = make_float4(r[0], r[1], r[2], r[3]);
          dst[col / 4 + 1] = make_float4(r[4], r[5], r[6], r[7]);
        }
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(tb.accfree0 + 8u * buf);  // this warp is done with the buffer
  return true;
}

// Worker warp wq (0..3) of a team: split every stage into hi / lo as it lands, and store each
// item's result one item later (so the tensor cores work on item j while item j-1 is stored).
template <bool CHECK>
__device__ void tc_worker(const KernelParams& p, const Task& task, float* land, float* comp,
                          const TeamBars& tb, uint32_t tmem_team, int team, int wq, int lane,
                          volatile int* abort_flag) {
  const int D = task.stages;
  const int tid = wq * 32 + lane;
  int c = 0;            // compute slot
  uint32_t cph = 0;     // its phase
  StageWin win;
  win.init(p.stages, task.team_off[team], task.team_off[team + 1], lane);
  int s = 0;
  uint32_t ph = 0;
  int j = 0;  // items completed (stages seen with the last-of-item flag)
  ItemInfo cur{8, 8, 0, 0, 0}, prev{8, 8, 0, 0, 0};
  bool ok = true;
  VBSR_PROF_T0(t_all);
  while (ok && !win.done()) {
    const Stage st = win.peek();
    win.advance(p.stages, lane);
    if (st.first()) cur = ItemInfo{st.h(), st.nw(), st.n0(), st.c_row(), 0};
    if (!st.empty()) {
      VBSR_PROF_T0(t_w);
      if (!wait_phase(tb.full0 + 8u * s, ph, p, abort_flag, lane)) {
        ok = false;
        break;
      }
      // the compute slot must have been released by the MMAs of its previous stage
      if (!wait_phase(tb.cfree0 + 8u * c, cph ^ 1u, p, abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 6, t_w);
      VBSR_PROF_T0(t_s);
      const int cols = st.cols();
      if (!(p.diag & VBSR_PLAN_DIAG_SKIP_MATH)) {
        const float* lp = land + s * kLandFloats;
        float* cp = comp + c * kCompFloats;
        split_hi_lo(lp + kLdA, cp + kCpA, cp + kCpALo, (cur.h * cols) / 4, tid);
        for (int g = 0; g < cols / 8; ++g)
          split_hi_lo(lp + kLdB + g * kBoxFloats, cp + kCpB + g * kBoxFloats,
                      cp + kCpBLo + g * kBoxFloats, cur.nw * 2, tid);
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(tb.landfree0 + 8u * s);  // the landing slot can be refilled
        mbar_arrive(tb.split0 + 8u * c);     // the compute slot is ready for the MMAs
      }
      VBSR_PROF_ADD(p, 7, t_s);
      cur.groups += cols / 8;
      if (++s == D) {
        s = 0;
        ph ^= 1u;
      }
      if (++c == kTcComp) {
        c = 0;
        cph ^= 1u;
      }
    }
    if (st.last()) {
      if (j > 0) {
        const int pj = j - 1;
        VBSR_PROF_T0(t_e);
        if (!tc_epilogue<CHECK>(p, tb, pj & 1, uint32_t((pj >> 1) & 1),
                                tmem_team + uint32_t(128 * (pj & 1)), wq, lane, prev,
                                abort_flag)) {
          ok = false;
          break;
        }
        VBSR_PROF_ADD(p, 9, t_e);
      }
      prev = cur;
      ++j;
    }
  }
  if (ok && j > 0) {
    const int pj = j - 1;
    tc_epilogue<CHECK>(p, tb, pj & 1, uint32_t((pj >> 1) & 1),
                       tmem_team + uint32_t(128 * (pj & 1)), wq, lane, prev, abort_flag);
  }
  VBSR_PROF_ADD(p, 5, t_all);
}

// Issuer warp `half` (0 or 1) of a team: lane 0 issues the MMAs of every other 8-column group
// (group index % 2 == half, counted from the item's start) into its partial accumulator once the
// workers have split the stage; issuer 0 also keeps the TMA ring D-1 stages ahead.
template <bool CHECK>
__device__ void tc_issuer(const KernelParams& p, const Task& task, float* land, float* comp,
                          const TeamBars& tb, uint32_t tmem_team, int team, int half, int lane,
                          volatile int* abort_flag) {
  const int D = task.stages;
  const int b = task.team_off[team], e = task.team_off[team + 1];
  StageWin win;
  win.init(p.stages, b, e, lane);
  Feeder f;
  f.slot = 0;
  f.ph = 0;
  f.filled = f.lastpar = 0;
  f.issued = 0;
  const bool feeder = half == 0;
  bool ok = true;
  if (feeder) {
    f.win.init(p.stages, b, e, lane);
    for (int i = 0; i < D - 1 && ok; ++i)
      ok = feed_next<CHECK>(p, f, land, D, tb, team, lane, abort_flag);
  }
  int s = 0;  // compute slot
  uint32_t ph = 0;
  int j = 0;  // items started
  const uint32_t sbase = smem_addr(comp);
  uint32_t tmem_d = tmem_team, idesc = 0, accumulate = 0;
  int gi = 0, h = 8;
  VBSR_PROF_T0(t_all);
  while (ok && !win.done()) {
    const Stage st = win.peek();
    win.advance(p.stages, lane);
    if (st.first()) {
      const int buf = j & 1;
      tmem_d = tmem_team + uint32_t(128 * buf + 64 * half);
      // the buffer's previous item (j-2) must have been read out by the workers
      VBSR_PROF_T0(t_f);
      if (j >= 2 && !wait_phase(tb.accfree0 + 8u * buf, uint32_t(((j - 2) >> 1) & 1), p,
                                abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 3, t_f);
      tc_fence_after();
      h = st.h();
      idesc = tf32_idesc(kTcM, h);
      accumulate = 0;
      gi = 0;
    }
    if (!st.empty()) {
      VBSR_PROF_T0(t_sp);
      if (!wait_phase(tb.split0 + 8u * s, ph, p, abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 1, t_sp);
      VBSR_PROF_T0(t_m);
      tc_fence_after();
      if (lane == 0 && !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH)) {
        const uint32_t sp = sbase + 4u * uint32_t(s * kCompFloats);
        uint64_t a_hi = sw32_desc(sp + 4u * kCpB);
        uint64_t b_hi = sw32_desc(sp + 4u * kCpA);
        const uint64_t da_lo = uint64_t((4u * (kCpBLo - kCpB)) >> 4);
        const uint64_t db_lo = uint64_t((4u * (kCpALo - kCpA)) >> 4);
        const uint64_t da = uint64_t((4u * kBoxFloats) >> 4), db = uint64_t((32u * h) >> 4);
        const int groups = st.cols() / 8;
        for (int g = 0; g < groups; ++g, ++gi) {
          if ((gi & 1) == half) {
            tc_mma_tf32(tmem_d, a_hi, b_hi, idesc, accumulate);
            tc_mma_tf32(tmem_d, a_hi, b_hi + db_lo, idesc, 1u);
            tc_mma_tf32(tmem_d, a_hi + da_lo, b_hi, idesc, 1u);
            accumulate = 1u;
          }
          a_hi += da;
          b_hi += db;
        }
      } else {
        gi += st.cols() / 8;
      }
      if (lane == 0) tc_commit(tb.cfree0 + 8u * s);  // frees the slot once these MMAs read it
      __syncwarp();
      VBSR_PROF_ADD(p, 4, t_m);
      VBSR_PROF_T0(t_i);
      if (feeder && !feed_next<CHECK>(p, f, land, D, tb, team, lane, abort_flag)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 2, t_i);
      if (++s == kTcComp) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (st.last()) {
      if (lane == 0) tc_commit(tb.acc0 + 8u * (j & 1));  // the item's accumulator is complete
      __syncwarp();
      ++j;
    }
  }
  VBSR_PROF_ADD(p, 0, t_all);
  // Every MMA this warp issued has completed before the CTA releases its tensor memory (bounded).
  if (lane == 0) tc_commit(tb.drain);
  __syncwarp();
  {
    const long long t0 = clock64();
    while (!mbar_try(tb.drain, 0) && clock64() - t0 < p.wait_limit) {
    }
  }
  // After an abort also wait (bounded) for every copy still in flight.
  if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
    for (int sl = 0; sl < D; ++sl) {
      if (!(f.filled & (1u << sl))) continue;
      const uint32_t bar = tb.full0 + 8u * sl;
      const uint32_t par = (f.lastpar >> sl) & 1u;
      const long long t1 = clock64();
      while (!mbar_try(bar, par) && clock64() - t1 < p.wait_limit) {
      }
    }
  }
}

template <bool CHECK>
__global__ void __launch_bounds__(kTcThreads, 1) spmm_tc_kernel(const __grid_constant__ KernelParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  float* stages = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[2][kTcTeams][kMaxStages];  // full, landfree
  __shared__ __align__(8) uint64_t cbars[2][kTcTeams][kTcComp];    // split, cfree
  __shared__ __align__(8) uint64_t accbars[2][kTcTeams][2];        // acc done, acc free
  __shared__ __align__(8) uint64_t drainbars[kTcTeams];
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
    for (int j = 0; j < kTcTeams; ++j) {
      for (int s = 0; s < task.stages; ++s) {
        mbar_init(smem_addr(&bars[0][j][s]), 1u);  // TMA: one arrival + transaction bytes
        mbar_init(smem_addr(&bars[1][j][s]), 4u);  // one arrival per worker warp
      }
      for (int c = 0; c < kTcComp; ++c) {
        mbar_init(smem_addr(&cbars[0][j][c]), 4u);                    // one per worker warp
        mbar_init(smem_addr(&cbars[1][j][c]), uint32_t(kTcIssuers));  // tcgen05.commit per issuer
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(smem_addr(&accbars[0][j][b]), uint32_t(kTcIssuers));
        mbar_init(smem_addr(&accbars[1][j][b]), 4u);
      }
      mbar_init(smem_addr(&drainbars[j]), uint32_t(kTcIssuers));
    }
    abort_flag = 0;
    mbar_fence_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  // warps 0..4*kTcTeams-1 are workers (team = warp/4, sub-partition = warp%4); the remaining
  // warps are the teams' issuers (kTcIssuers consecutive warps per team)
  const bool worker = warp < 4 * kTcTeams;
  const int iw = warp - 4 * kTcTeams;
  const int team = worker ? (warp >> 2) : (iw / kTcIssuers);
  TeamBars tb;
  tb.full0 = smem_addr(&bars[0][team][0]);
  tb.landfree0 = smem_addr(&bars[1][team][0]);
  tb.split0 = smem_addr(&cbars[0][team][0]);
  tb.cfree0 = smem_addr(&cbars[1][team][0]);
  tb.acc0 = smem_addr(&accbars[0][team][0]);
  tb.accfree0 = smem_addr(&accbars[1][team][0]);
  tb.drain = smem_addr(&drainbars[team]);
  float* land = stages + team * (task.stages * kLandFloats + kTcComp * kCompFloats);
  float* comp = land + task.stages * kLandFloats;
  const uint32_t tmem_team = tmem_base + uint32_t(kTeamTmem * team);
  if (worker)
    tc_worker<CHECK>(p, task, land, comp, tb, tmem_team, team, warp & 3, lane, &abort_flag);
  else
    tc_issuer<CHECK>(p, task, land, comp, tb, tmem_team, team, iw % kTcIssuers, lane,
                     &abort_flag);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem_base, kTmemAlloc);
  }
  if (threadIdx.x == 0 && p.timing) p.timing[2 * blockIdx.x + 1] = global_ns();
}

}  // namespace vbsr_b200
