// vbsr_tc.cuh — the sm_100a SpMM kernel on 5th-generation tensor cores (tcgen05, TMEM).
//
// Per work item (one block row i: an h x nw tile of C) the kernel sums over the row's 8-column
// groups g with tcgen05.mma kind::tf32 (K = 8) into fp32 accumulators in tensor memory, in one of
// two forms (template parameter TR):
//   row-stacked (rhs <= 32):    D (M x 2 rhs) = sum_g [A_g ; A_g,lo] (M x 8) * S_g^T, one MMA per
//                               group, M = 64 for h <= 32 and 128 otherwise;
//   column-stacked (rhs = 64):  D (128 x h) = sum_g S_g (128 x 8) * (A_g + A_g,lo)^T, two MMAs per
//                               group (raw A, then A_lo, on the N side).
// S_g is the operand stack of group g of B: rows of raw B (hi) and of their lo parts.
//
// FP32 accuracy (3xTF32). The tensor core reads an fp32 operand as tf32 by ignoring its low 13
// mantissa bits (truncation), so for x = hi + lo with hi = trunc_tf32(x) the raw value already
// acts as hi and only lo = x - hi has to be formed (exactly, in fp32). Both forms produce the four
// products A_hi*B_hi, A_hi*B_lo, A_lo*B_hi and A_lo*B_lo (the last one below the tolerance but
// harmless), and the epilogue adds, for every C element, the accumulator entries that hold them.
//
// The stacks of all 8-column groups of B are formed once per execute by a small pre-pass
// (bstack_kernel) in global memory, already in the MMA's K-major, 32-byte-swizzled layout, so a
// run of a block's groups arrives with one contiguous bulk copy. In the row-stacked form the A and
// A_lo rows of a group alternate in 8-row blocks, so a C row's A and A_lo accumulator rows sit in
// one TMEM quadrant, 8 lanes apart. In the column-stacked form S is built per quadrant q (32 TMEM
// lanes): with half = 16 columns per quadrant, S rows 32q + j and 32q + 16 + j hold hi and lo of
// column 16q + j, so they land in lanes j and 16 + j of quadrant q. Either way a warp adds the
// pair with one shuffle.
//
// One CTA per SM; warp numbers below are the row-stacked form's (the column-stacked form has 12
// split warps, then MMA warps 12..15, feeders 16..19 and one epilogue set, warps 20..23):
//   warps 0..3   split warps: stage k (the CTA's k-th non-empty stage) is split by warp k % 4
//                (column-stacked: by team k % 4 of three warps), which forms A_lo (row-stacked:
//                spreads the stage's A in place into alternating A / A_lo blocks), fences the
//                writes for the async proxy and hands the slot on;
//   warps 4..7   MMA warps: stage k is issued by MMA warp k % 4 into the warp's own accumulator,
//                and the slot is released with tcgen05.commit;
//   warps 8..11  feeders: stage k is copied by feeder k % 4 with cp.async.bulk: the stage's A in
//                one copy, the stacks S in one copy per run of consecutive groups of a block;
//   warps 12..19 epilogue warps, two sets of four: set e stores the items j with j % 2 == e
//                (TMEM buffer e); warp q of a set reads TMEM quadrant q as soon as the item's
//                MMAs are done and stores its C rows.
// A single wait-and-release round on an mbarrier costs a warp ~150-200 cycles even when the
// barrier has already completed (and a wait next to MMA issue as much), which is why every role
// is spread over several warps. The ring has D slots, D a multiple of every role's warp count,
// stage k uses slot k % D: each slot then has one feeder, one split warp and one MMA warp, all
// passing through its uses in order. Every warp walks the CTA's list of stage descriptors
// (compiled by the planner; vbsr_internal.h). Every wait is bounded (see wait_phase); after an
// abort the feeders wait for their copies and the MMA warps for their MMAs before the CTA releases
// its tensor memory.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_kernels_common.cuh"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

// Warp roles (one CTA per SM), per form (template parameter TR of the kernel):
//                     split   MMA   feeders   epilogue   warps   registers (at most)
//   row-stacked         4      4       4       8 (two sets)  20       96
//   column-stacked     12      4       4       4 (one set)   24       80
// The column-stacked split warps also form B_lo, in teams of three per stage.
// Epilogue warps come last and start at a multiple of 4 (a warp reaches the TMEM lanes
// 32 (warp % 4) ... only); epilogue set e stores the items j with j % sets == e. Every slot
// count is a multiple of each role's warp count (kTcRingMultiple).
template <bool TR>
struct Roles {
  static constexpr int split = TR ? 4 : 12;
  static constexpr int epi_sets = TR ? 2 : 1;
  static constexpr int mma0 = split, feeder0 = split + 4, epi0 = split + 8;
  static constexpr int warps = epi0 + 4 * epi_sets;
  static_assert(epi0 % 4 == 0, "role layout");
};
constexpr int kCsSplitTeam = 3;  // column-stacked form: warps that split one stage
constexpr int kTcMmaWarps = 4;  // MMA-issuing warps
constexpr int kTcFeeders = 4;   // feeder warps
constexpr int kTcRingMultiple = 8;
constexpr int kPrefetchAhead = 2;  // A is prefetched into L2 this many own stages ahead
__host__ __device__ constexpr int tc_warps(bool tr) { return tr ? Roles<true>::warps : Roles<false>::warps; }
__host__ __device__ constexpr int stack_m(int nw) { return nw > 32 ? 128 : 64; }
// RHS widths up to 32 use the row-stacked form (one MMA per group, the operand stack S on the N
// side); width 64 the column-stacked form (two MMAs per group, S on the M side). S has
// stack_rows(rhs) rows of 32 bytes per 8-column group.
__host__ __device__ constexpr bool row_stacked(int rhs) { return rhs <= 32; }
// Column-stacked form, two stack layouts (the plan picks one; `raw` below):
//   pre-split: the pre-pass writes hi and lo rows (M = 128 per group), two MMAs per group;
//   raw:       the pre-pass writes only the raw B rows (64 per group), the split warps form their
//              lo rows in shared memory, and each group takes three M = 64 MMAs.
// Raw halves the stacks' bytes in global memory, which pays when they do not stay in L2.
__host__ __device__ constexpr int stack_rows(int rhs, bool raw) {
  return row_stacked(rhs) ? 2 * rhs : (raw ? rhs : stack_m(rhs));
}
// Bytes of one group's stack in global memory, and in a shared-memory slot.
__host__ __device__ constexpr int stack_tile_bytes(int rhs, bool raw) {
  return 32 * stack_rows(rhs, raw);
}
__host__ __device__ constexpr int stack_slot_bytes(int rhs, bool raw) {
  return (!row_stacked(rhs) && raw) ? 2 * stack_tile_bytes(rhs, raw) : stack_tile_bytes(rhs, raw);
}
// A slot (26 KB by default) holds one stage of G groups: their A values and A_lo parts in the first
// 64 h G bytes (column-stacked form: raw A of group after group, then the A_lo parts at byte
// 32 h G; row-stacked form: per group, 8-row blocks of raw A and of A_lo alternating), then their
// operand stacks S (stack_tile_bytes each) from byte 64 h G. A stage takes as many consecutive
// groups of its item as fit, at most kMaxStageGroups: G = stage_groups(h, rhs).
constexpr int kSlotBytes = 26 * 1024;
constexpr int kMaxStageGroups = 8;
__host__ __device__ constexpr int slot_floats(int rhs) { return (void)rhs, kSlotBytes / 4; }
__host__ __device__ constexpr int stage_groups(int h, int rhs, bool raw) {
  return kSlotBytes / (64 * h + stack_slot_bytes(rhs, raw)) < kMaxStageGroups
             ? kSlotBytes / (64 * h + stack_slot_bytes(rhs, raw))
             : kMaxStageGroups;
}
__host__ __device__ constexpr int slot_stack_bytes(int h, int groups) { return 64 * h * groups; }
// The row-stacked MMA reads M = 64 or 128 rows from a group's first byte, up to 1.5 KB beyond the
// group's 64 h bytes (rows it does not use); the shared memory allocation ends with this pad.
constexpr int kSmemTailPad = 2048;
constexpr int kTrM64MaxH = 32;  // row-stacked items with h <= this use M = 64
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

// ---- fused pre-pass ------------------------------------------------------------------------------
//
// With VBSR_PLAN_FUSED_PREPASS the SpMM's own CTAs form B's operand stacks (the same tiles
// bstack_kernel writes) before their pipelines start, so an execute is one launch. Work is flat
// over the 16-byte pieces of the tiles' raw (hi) rows: piece f is half (f & 1) of column
// c = (f >> 1) mod rhs in tile g = f / (2 rhs). Lanes take
// consecutive pieces, so a warp's stores fill 512 contiguous bytes of a tile (and the lo piece of a
// hi piece, its row's lo row, 512 more), and each lane pair reads one whole 32-byte sector of a
// column of B. Each lane keeps kStackUnroll pieces in flight.
constexpr int kStackUnroll = 4;
template <bool TR, bool RAW>
__device__ __forceinline__ void stack_rows_of(int c, int rhs, int& hi, int& lo) {
  if (TR) {  // rows c: raw B of column c; rows rhs + c: its lo part
    hi = c;
    lo = rhs + c;
  } else if (RAW) {  // raw rows only
    hi = c;
    lo = -1;
  } else {  // pre-split, per quadrant q of 16 columns: 16 rows of hi, then 16 of lo
    hi = 32 * (c >> 4) + (c & 15);
    lo = hi + 16;
  }
}
template <bool TR, bool RAW>
__device__ void stack_fused(const KernelParams& p, long long gw, long long nwarps, int lane) {
  const long long ngroups = p.K >> 3;
  const int rhs = p.rhs, lg = __ffs(rhs) - 1, rows = stack_rows(rhs, RAW);
  const long long pieces = ngroups << (lg + 1), k4 = p.K >> 2;
  const float4* B4 = reinterpret_cast<const float4*>(p.B);
  float4* out = reinterpret_cast<float4*>(const_cast<float*>(p.bstack));
  for (long long u0 = gw; (u0 << 5) < pieces; u0 += nwarps * kStackUnroll) {
    float4 v[kStackUnroll];
    long long dst[kStackUnroll];
    int lo_off[kStackUnroll];
#pragma unroll
    for (int k = 0; k < kStackUnroll; ++k) {
      const long long f = ((u0 + nwarps * k) << 5) + lane;
      dst[k] = -1;
      if (f < pieces) {
        const long long g = f >> (lg + 1);
        const int c = int(f >> 1) & (rhs - 1), pos = int(f & 1);
        int hi, lo;
        stack_rows_of<TR, RAW>(c, rhs, hi, lo);
        // the swizzle: the 16-byte half u of the row's 32 bytes sits at position u ^ ((row >> 2) & 1)
        // (a lo row has the same parity as its hi row)
        const int u = pos ^ ((hi >> 2) & 1);
        v[k] = __ldcs(B4 + c * k4 + 2 * g + u);
        dst[k] = g * (2 * rows) + 2 * hi + pos;
        lo_off[k] = lo >= 0 ? 2 * (lo - hi) : 0;
      }
    }
#pragma unroll
    for (int k = 0; k < kStackUnroll; ++k) {
      if (dst[k] < 0) continue;
      out[dst[k]] = v[k];
      if (lo_off[k] != 0) out[dst[k] + lo_off[k]] = lo_part4(v[k]);
    }
  }
}
// Grid arrival on p.stack_flag, once per CTA after all its stack stores (by one thread, after a
// CTA barrier). CTA 0 adds 2^31 - (grid - 1), every other CTA 1: the word's top bit flips exactly
// when the last CTA arrives, and its low bits are back where they started, so the word needs no
// reset between executes (executes of one plan never overlap). Returns the top bit seen before
// this CTA's arrival; the stacks are complete once the word's top bit differs from it.
__device__ __forceinline__ uint32_t stack_arrive(const KernelParams& p) {
  __threadfence();
  const uint32_t add = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1u) : 1u;
  return atomicAdd(p.stack_flag, add) & 0x80000000u;
}
// Bounded wait (lane 0 polls) for every CTA's stacks; false after a timeout or another warp's abort.
__device__ __forceinline__ bool wait_stacks(const KernelParams& p, uint32_t sense,
                                            volatile int* abort_flag, int lane) {
  int ok = 1;
  if (lane == 0) {
    const long long t0 = clock64();
    while (((ld_acquire_gpu(p.stack_flag) ^ sense) & 0x80000000u) == 0u) {
      if (*abort_flag) {
        ok = 0;
        break;
      }
      if (clock64() - t0 > p.wait_limit) {
        record_status(p.status, VBSR_TIMEOUT, int(blockIdx.x));
        *abort_flag = 1;
        ok = 0;
        break;
      }
      __nanosleep(256);
    }
    fence_proxy_async_global();  // the bulk copies that follow read what the other CTAs stored
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// ---- CTA pieces ----------------------------------------------------------------------------------

// Barriers (shared-memory addresses).
struct CtaBars {
  uint32_t full0;           // per slot: copies landed
  uint32_t split0;          // per slot: lo parts written
  uint32_t empty0;          // per slot: the stage's MMAs have read the slot
  uint32_t acc0, accfree0;  // per accumulator buffer: MMAs of the item done / D read by all warps
  uint32_t drain0;          // per MMA warp: end-of-kernel drain of its MMAs
};

#include "vbsr_dev_instrument.cuh"

// Feeder warp f: fills the slots of the stages k with k % kTcFeeders == f, each once the MMAs of
// the slot's previous stage have completed.
// DIRECT (column-stacked raw form only): the stacks' raw rows come straight from B instead of from
// the pre-pass: per run of consecutive groups of one block, RHS column c's 8 * n values are
// contiguous in column-major B, and the lanes copy them in 16-byte pieces (cp.async) into the
// slot's swizzled stack rows; each lane's copies then arrive on the full barrier
// (cp.async.mbarrier.arrive), which therefore expects 1 + 32 arrivals.
template <bool CHECK, bool RAW, bool DIRECT>
__device__ void tc_feeder(const KernelParams& p, const Task& task, uint32_t slots,
                          const CtaBars& cb, int f, int lane, volatile int* abort_flag,
                          uint32_t stack_sense) {
  const int D = task.stages, SF = task.stage_floats;
  const int nst = task.stage_end - task.stage_off;
  StageWin win;
  win.init(p.stages + task.stage_off, f, kTcFeeders, nst, lane);
  int s = f;  // slot of this feeder's next stage (its slots are f, f + kTcFeeders, ...)
  uint32_t ph = 0;
  uint32_t filled = 0, lastpar = 0;
  const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
  // The feeders are the only warps that read the stacks. Fused pre-pass: wait for every CTA's
  // share of them. Separate pre-pass launch: the SpMM is its programmatic dependent, so that its
  // prologue overlaps the pre-pass, and waits for it here.
  bool go = true;
  if (!DIRECT) {
    if (p.stack_flag != nullptr)
      go = wait_stacks(p, stack_sense, abort_flag, lane);
    else
      griddep_wait();
  }
  VBSR_PROF_T0(t_all);
  for (int kk = f; go && kk < nst; kk += kTcFeeders) {
    const Stage st = win.get();
    if (kPrefetchAhead > 0 && win.has_ahead(kPrefetchAhead) &&
        !(p.diag & VBSR_PLAN_DIAG_SKIP_COPIES)) {
      // the A values of this feeder's stage kPrefetchAhead turns later, into L2 (one TMA op)
      Stage pf;
      pf.w0 = win.word0_ahead(kPrefetchAhead);
      if (lane == 0) bulk_prefetch_l2(p.values + pf.a_start(), uint32_t(pf.a_span_bytes()));
    }
    win.advance(lane);
    const uint32_t full_bar = cb.full0 + 8u * s;
    // Everything the copies need is worked out before the wait, so that only their issue is on the
    // slot's critical path. A: the stage's groups are contiguous in the device format: one copy.
    // S: consecutive groups of one block have consecutive pre-pass tiles, so each run of them is
    // one copy, issued by the lane of the run's first group.
    const int h = st.h(), nw = st.nw(), n0 = st.n0(), groups = st.groups(), H = st.H();
    const long long a0 = st.a_start();
    const uint32_t sp = slots + 4u * uint32_t(s * SF);
    const int T = stack_tile_bytes(p.rhs, RAW);
    const int col = lane < groups ? st.group_col(lane) : 0;
    const int prev = __shfl_up_sync(0xffffffffu, col, 1);
    const bool start = lane < groups && (lane == 0 || col != prev + 8);
    const uint32_t starts = __ballot_sync(0xffffffffu, start);
    const uint32_t later = starts & ~((2u << lane) - 1u);
    const int end = later ? __ffs(later) - 1 : groups;
    const uint32_t s_dst = sp + uint32_t(slot_stack_bytes(h, groups) + T * lane);
    const float* s_src = p.bstack + (long long)(col >> 3) * (T / 4);
    const uint32_t s_bytes = uint32_t(T * (end - lane));
    const uint32_t tx = uint32_t(groups * (32 * h + (DIRECT ? 0 : T))),
                   a_bytes = uint32_t(32 * h * groups);
    const float* a_src = p.values + a0;
    asm volatile("" ::"r"(s_dst), "l"(s_src), "r"(s_bytes), "r"(tx), "r"(a_bytes), "l"(a_src));
    VBSR_PROF_T0(t_w);
    if (!wait_phase(cb.empty0 + 8u * s, ph ^ 1u, p, abort_flag, lane)) break;
    VBSR_PROF_ADD(p, 7, t_w);
    VBSR_TRACE_ST(kk, 0);
    bool ok = true;
    if (CHECK) {
      ok = a0 + st.a_span_bytes() / 4 <= p.nvalues && n0 == 0 && nw == p.rhs && h <= H &&
           groups <= stage_groups(h, p.rhs, RAW);
      for (int g = 0; g < groups; ++g) ok = ok && st.group_col(g) + 8 <= p.K;
    }
    if (kk == p.drop_stage) {
      // withhold the stage entirely (debug): no arrival, no copies
    } else if ((p.diag & VBSR_PLAN_DIAG_SKIP_COPIES) || !ok) {
      if (lane == 0) {
        if (!ok) record_status(p.status, VBSR_BOUNDS_VIOLATION, int(blockIdx.x));
        mbar_arrive(full_bar);  // release the split warp without touching memory
      }
      if (DIRECT) mbar_arrive(full_bar);  // the lanes' copy arrivals
    } else {
      VBSR_TRACE_ST(kk, 7);
      if (lane == 0) {
        mbar_arrive_expect_tx(full_bar, tx);
        if (H == h) bulk_g2s(sp, a_src, a_bytes, full_bar, pol_a);  // one contiguous range
      }
      __syncwarp();
      // a row part: its rows of each group are a separate range (groups H * 8 floats apart); the
      // slot holds them as consecutive h-row groups, the layout of an unsplit item of height h
      if (H != h && lane < groups)
        bulk_g2s(sp + uint32_t(32 * h * lane), a_src + 8ll * H * lane, uint32_t(32 * h), full_bar,
                 pol_a);
      if (DIRECT) {
        // runs in order; run r: groups [r, end_r), first scalar column col_r
        const uint32_t s0 = sp + uint32_t(slot_stack_bytes(h, groups));
        for (uint32_t rs = starts; rs != 0; rs &= rs - 1) {
          const int r = __ffs(rs) - 1;
          const int n2 = 2 * (__shfl_sync(0xffffffffu, end, r) - r);  // 16-byte pieces per column
          const float* src0 = p.B + __shfl_sync(0xffffffffu, col, r);
          const uint32_t dst0 = s0 + uint32_t(T * r);
          for (int i = lane; i < p.rhs * n2; i += 32) {
            const int c = i / n2, j = i - c * n2;
            const uint32_t dst = dst0 + uint32_t(T * (j >> 1) + 32 * c +
                                                 16 * ((j & 1) ^ ((c >> 2) & 1)));
            cp_async16(dst, src0 + (long long)c * p.K + 4 * j);
          }
        }
        cp_async_arrive(full_bar);
      } else if (start) {
        bulk_g2s(s_dst, s_src, s_bytes, full_bar, pol_b);
      }
      filled |= 1u << s;
      VBSR_TRACE_ST(kk, 1);
      lastpar = (lastpar & ~(1u << s)) | (ph << s);
    }
    if ((s += kTcFeeders) >= D) {
      s -= D;
      ph ^= 1u;
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

// Epilogue of one item: D -> C, by epilogue warp w (TMEM quadrant w). Partial i (64 columns after
// partial 0) holds the stages issued by MMA warp i; only partials that received a stage are read.
// Within a partial, column r is row r of the tile. Lane j < half of quadrant w holds hi of RHS
// column n0 + half*w + j, lane half + j its lo.
template <bool CHECK, bool RAW>
__device__ __forceinline__ bool tc_epilogue(const KernelParams& p, const CtaBars& cb, int buf,
                                            uint32_t parity, uint32_t tmem_buf, int w, int lane,
                                            const Item& it, volatile int* abort_flag) {
  VBSR_PROF_T0(t_w);
  if (!wait_phase(cb.acc0 + 8u * buf, parity, p, abort_flag, lane)) return false;
  VBSR_PROF_ADD(p, 4, t_w);
  tc_fence_after();
  const int h = it.h(), nw = it.nw(), n0 = it.n0();
  // raw-B: 16 columns per quadrant (M = 64 layout: lanes 0..15), hi and lo already summed
  const int half = RAW ? 16 : stack_m(nw) / 8, quads = nw / half;
  uint32_t use = 0;  // bit i: partial i received a stage of the item
  if (!(p.diag & VBSR_PLAN_DIAG_SKIP_MATH))
    for (uint32_t i = 0; i < kTcMmaWarps && i < it.n; ++i) use |= 1u << ((it.k0 + i) & 3u);
  if (w < quads) {
    const uint32_t taddr = tmem_buf + (uint32_t(32 * w) << 16);
    const bool store = lane < half &&
                       !(CHECK && ((long long)it.c_row + h > p.M || n0 + nw > p.rhs));
    if (CHECK && w == 0 && lane == 0 && ((long long)it.c_row + h > p.M || n0 + nw > p.rhs))
      record_status(p.status, VBSR_BOUNDS_VIOLATION, int(it.c_row));
    const int col = n0 + half * w + lane;
    float4* dst = reinterpret_cast<float4*>(p.C + (long long)col * p.M + it.c_row);
    // passes of 8 tile rows: 4 partials x 8 values in flight per pass
    for (int c0 = 0; c0 < h; c0 += 8) {
      float v[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (use & (1u << i)) tc_ld8_nowait(taddr + uint32_t(64 * i + c0), v[i]);
      tc_wait_ld();
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (use & (1u << i)) a += v[i][e];
        r[e] = RAW ? a : a + __shfl_down_sync(0xffffffffu, a, half);
      }
      if (store) {
        dst[c0 / 4] = make_float4(r[0], r[1], r[2], r[3]);
        dst[c0 / 4 + 1] = make_float4(r[4], r[5], r[6], r[7]);
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(cb.accfree0 + 8u * buf);  // this warp is done with the buffer
  return true;
}

// Row-stacked epilogue of one item, by epilogue warp w (TMEM quadrant w). Partial i (64 columns
// after partial 0) holds the stages issued by MMA warp i; only partials that received a stage are
// read. Accumulator row r is row r of the groups' interleaved [A | A_lo] operand, column c < rhs its
// product with raw B of RHS column c and column rhs + c with that column's lo part. Quadrant w
// holds, for M = 64 (h <= 32), tile rows 8w + j in lanes j (A) and 8 + j (A_lo); for M = 128, tile
// rows 16w + j and 16w + 8 + j in lanes j, 16 + j (A) and 8 + j, 24 + j (A_lo). A lane adds its
// hi and lo columns, then the A_lo lane's sum with one shuffle, and stores its row of C.
template <bool CHECK>
__device__ __forceinline__ bool tc_epilogue_rows(const KernelParams& p, const CtaBars& cb, int buf,
                                                 uint32_t parity, uint32_t tmem_buf, int w,
                                                 int lane, const Item& it,
                                                 volatile int* abort_flag) {
  VBSR_PROF_T0(t_w);
  if (!wait_phase(cb.acc0 + 8u * buf, parity, p, abort_flag, lane)) return false;
  VBSR_PROF_ADD(p, 4, t_w);
  tc_fence_after();
  const int h = it.h(), R = p.rhs;
  uint32_t use = 0;  // bit i: partial i received a stage of the item
  if (!(p.diag & VBSR_PLAN_DIAG_SKIP_MATH))
    for (uint32_t i = 0; i < kTcMmaWarps && i < it.n; ++i) use |= 1u << ((it.k0 + i) & 3u);
  const bool m64 = h <= kTrM64MaxH;
  const int row0 = m64 ? 8 * w : 16 * w;  // the quadrant's first tile row
  if (row0 < h) {
    const bool bad = CHECK && ((long long)it.c_row + h > p.M || it.n0() + it.nw() > p.rhs);
    if (CHECK && w == 0 && lane == 0 && bad) record_status(p.status, VBSR_BOUNDS_VIOLATION, int(it.c_row));
    const int n = row0 + (lane & 7) + (m64 ? 0 : 8 * (lane >> 4));
    const bool store = (lane & 8) == 0 && (!m64 || lane < 16) && n < h && !bad;
    float* dst = p.C + (long long)it.c_row + n;  // RHS column c at dst + c * M
    const uint32_t taddr = tmem_buf + (uint32_t(32 * w) << 16);
    for (int c0 = 0; c0 < R; c0 += 8) {
      float v[4][8], a[8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (use & (1u << i)) tc_ld8_nowait(taddr + uint32_t(64 * i + c0), v[i]);
      tc_wait_ld();
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a[e] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (use & (1u << i)) a[e] += v[i][e];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (use & (1u << i)) tc_ld8_nowait(taddr + uint32_t(64 * i + R + c0), v[i]);
      tc_wait_ld();
#pragma unroll
      for (int e = 0; e < 8; ++e) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (use & (1u << i)) a[e] += v[i][e];
        a[e] += __shfl_xor_sync(0xffffffffu, a[e], 8);
      }
      if (store) {
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[(long long)(c0 + e) * p.M] = a[e];
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(cb.accfree0 + 8u * buf);  // this warp is done with the buffer
  return true;
}

// Row-stacked form: the stage's A arrives as U = h G / 8 blocks of 8 rows (256 bytes), block u at
// byte 256 u; it is spread in place so that block u sits at byte 512 u followed by its A_lo block.
// Block u's destination covers the sources of blocks 2u and 2u + 1 only, so passes over the
// blocks from the last one down, each loading all its blocks before storing any, never overwrite a
// block that is still to be read. Block 0 stays where it is. The 32-byte swizzle is a function of
// the address bits below 256, which the move preserves.
__device__ __forceinline__ void split_stage_rows(uint32_t sp, int groups, int h, int lane) {
  const int units = (h >> 3) * groups;
  constexpr int kPassUnits = 16;  // blocks per pass: kPassUnits / 2 float4s per lane
  for (int top = units; top > 0; top -= kPassUnits) {
    const int u0 = top > kPassUnits ? top - kPassUnits : 0;
    float4 x[kPassUnits / 2];
#pragma unroll
    for (int v = 0; v < kPassUnits / 2; ++v) {
      const int i = 32 * v + lane;  // float4 i of the pass: block u0 + i / 16, piece i % 16
      if (u0 + (i >> 4) < top) x[v] = lds128(sp + 256u * uint32_t(u0) + 16u * uint32_t(i));
    }
    __syncwarp();
#pragma unroll
    for (int v = 0; v < kPassUnits / 2; ++v) {
      const int i = 32 * v + lane, u = u0 + (i >> 4);
      if (u < top) {
        const uint32_t d = sp + 512u * uint32_t(u) + 16u * uint32_t(i & 15);
        if (u > 0) sts128(d, x[v]);
        sts128(d + 256u, lo_part4(x[v]));
      }
    }
    __syncwarp();
  }
}

// lo parts of n float4s at shared address sp, written lo_off bytes further (the chunks of 128
// float4s with index % parts == part; 2 KB chunks measured as fast as 1 KB ones here, 512 B ones
// slower).
__device__ __forceinline__ void split_flat(uint32_t sp, int n, uint32_t lo_off, int lane,
                                           int part = 0, int parts = 1) {
  constexpr int U = 4;
  for (int i0 = 32 * U * part; i0 < n; i0 += 32 * U * parts) {
    float4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < n) x[u] = lds128(sp + 16u * i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < n) sts128(sp + lo_off + 16u * i, lo_part4(x[u]));
    }
  }
}

// Column-stacked form: A_lo of a whole stage at shared address sp: the stage's A (2h float4s per
// group, groups one after another) at sp, its A_lo at the same offsets 32 h G bytes further. The
// chunks are 64 float4s (two loads per lane in flight before their stores): a stage's A is only
// 2-5 KB, and chunks this small share it evenly among the warps of a team (with 4 KB chunks
// one warp often had nearly all of it; large config kernel 12.06 -> 11.59 ms).
__device__ __forceinline__ void split_stage(uint32_t sp, int groups, int h, int lane,
                                            int part = 0, int parts = 1) {
  constexpr int U = 2;
  const int n = 2 * h * groups;  // float4s
  const uint32_t lo = uint32_t(32 * h * groups);
  for (int i0 = 32 * U * part; i0 < n; i0 += 32 * U * parts) {
    float4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < n) x[u] = lds128(sp + 16u * i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 32 * u + lane;
      if (i < n) sts128(sp + lo + 16u * i, lo_part4(x[u]));
    }
  }
}

// Split warp w: forms the lo parts of the stages k with k % Roles<TR>::split == w (slots w,
// w + Roles<TR>::split, ...).
template <bool CHECK, bool TR, bool RAW>
__device__ void tc_split_warp(const KernelParams& p, const Task& task, uint32_t slots,
                              const CtaBars& cb, uint32_t tmem_base, int w, int lane,
                              volatile int* abort_flag) {
  // Column-stacked form: a stage is split by a team of kCsSplitTeam warps, each taking every
  // kCsSplitTeam-th chunk of the A and B_lo work (no chunk is read by another member, so the
  // members need no barrier between them; each arrives on the slot's split barrier).
  constexpr int kTeam = TR ? 1 : kCsSplitTeam;
  constexpr int kTcSplitWarps = Roles<TR>::split / kTeam;  // teams
  const int member = w % kTeam;
  w /= kTeam;
  const int D = task.stages, SF = task.stage_floats;
  ItemWin iw;
  iw.init(p.items + task.item_off, task.item_end - task.item_off, lane);
  int kk = w;      // this team's next stage
  int ms = w;      // its slot
  uint32_t mph = 0;
  const bool math = !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH);
  bool ok = true;
  VBSR_PROF_T0(t_all);
  while (ok && !iw.done()) {
    const Item it = iw.get();
    iw.advance(lane);
    const int h = it.h(), G = stage_groups(h, p.rhs, RAW);
    for (const int kend = int(it.k0 + it.n); kk < kend; kk += kTcSplitWarps) {
      const int groups = it.stage_groups(kk - int(it.k0), G);
      const int s = ms;
      const uint32_t par = mph;
      if ((ms += kTcSplitWarps) >= D) {
        ms -= D;
        mph ^= 1u;
      }
      VBSR_PROF_T0(t_w);
      if (!wait_phase(cb.full0 + 8u * s, par, p, abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 1, t_w);
      VBSR_TRACE_ST(kk, 2);
      VBSR_PROF_T0(t_s);
      if (math) {
        if (TR) {
          split_stage_rows(slots + 4u * uint32_t(s * SF), groups, h, lane);
        } else {
          split_stage(slots + 4u * uint32_t(s * SF), groups, h, lane, member, kTeam);
          if (RAW) {  // the stacks' lo rows: the raw rows (T per group) are followed by theirs
            const int T = stack_tile_bytes(p.rhs, RAW);
            split_flat(slots + 4u * uint32_t(s * SF) + uint32_t(slot_stack_bytes(h, groups)),
                       T * groups / 16, uint32_t(T * groups), lane, member, kTeam);
          }
        }
        VBSR_TRACE_ST(kk, 6);
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(cb.split0 + 8u * s);
      VBSR_TRACE_ST(kk, 3);
      VBSR_PROF_ADD(p, 2, t_s);
    }
  }
  VBSR_PROF_ADD(p, 0, t_all);
}

// Epilogue warp q (TMEM quadrant q) of epilogue set `set`: stores the results of the set's items as
// soon as their MMAs are done.
template <bool CHECK, bool TR, bool RAW>
__device__ void tc_epi_warp(const KernelParams& p, const Task& task, const CtaBars& cb,
                            uint32_t tmem_base, int q, int set, int lane,
                            volatile int* abort_flag) {
  ItemWin iw;
  iw.init(p.items + task.item_off, task.item_end - task.item_off, lane);
  VBSR_PROF_T0(t_all);
  for (int j = 0; !iw.done(); ++j) {
    const Item it = iw.get();
    iw.advance(lane);
    constexpr int kEpiSets = Roles<TR>::epi_sets;
    if (kEpiSets > 1 && j % kEpiSets != set) continue;  // another set's item
    VBSR_PROF_T0(t_e);
    if (q == 0) VBSR_TRACE_IT(j, 0);
    const uint32_t par = uint32_t((j >> 1) & 1), tbuf = tmem_base + uint32_t(256 * (j & 1));
    if (!(TR ? tc_epilogue_rows<CHECK>(p, cb, j & 1, par, tbuf, q, lane, it, abort_flag)
             : tc_epilogue<CHECK, RAW>(p, cb, j & 1, par, tbuf, q, lane, it, abort_flag)))
      break;
    VBSR_PROF_ADD(p, 8, t_e);
    if (q == 0) VBSR_TRACE_IT(j, 1);
  }
  VBSR_PROF_ADD(p, 11, t_all);
}

// MMA warp i (0..3): issues the stages k with k % 4 == i into its partial accumulator (TMEM columns
// 256 * buffer + 64 * i): one MMA per group in the row-stacked form, two (S x A, S x A_lo) in the
// column-stacked form.
template <bool CHECK, bool TR, bool RAW, bool DIRECT>
__device__ void tc_mma_warp(const KernelParams& p, const Task& task, uint32_t slots,
                            const CtaBars& cb, uint32_t tmem_base, int i, int lane,
                            volatile int* abort_flag) {
  const int D = task.stages, SF = task.stage_floats;
  ItemWin iw;
  iw.init(p.items + task.item_off, task.item_end - task.item_off, lane);
  int kk = i;      // this warp's next stage
  int ms = i;      // its slot (this warp's slots are i, i + 4, ...)
  uint32_t mph = 0;
  int j = 0;       // items started
  const bool math = !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH);
  bool ok = true;
  VBSR_PROF_T0(t_all);
  while (ok && !iw.done()) {
    const Item it = iw.get();
    iw.advance(lane);
    const int buf = j & 1;
    // the buffer's previous item (j-2) must have been read out by every split warp
    VBSR_PROF_T0(t_f);
    if (j >= 2 && !wait_phase(cb.accfree0 + 8u * buf, uint32_t(((j - 2) >> 1) & 1), p,
                              abort_flag, lane))
      break;
    VBSR_PROF_ADD(p, 5, t_f);
    if (i == 0) VBSR_TRACE_IT(j, 2);
    tc_fence_after();
    const int M = stack_m(it.nw()), h = it.h(), G = stage_groups(h, p.rhs, RAW);
    const uint32_t T = uint32_t(stack_tile_bytes(p.rhs, RAW));
    const uint32_t tmem_d = tmem_base + uint32_t(256 * buf + 64 * i);
    // row-stacked: M = the group's interleaved A / A_lo rows (64 covers h <= 32), N = S's 2 rhs
    // rows; column-stacked: M = S's rows, N = the group's h rows of A (then of A_lo)
    const uint32_t idesc = TR ? tf32_idesc(h <= kTrM64MaxH ? 64 : 128, 2 * p.rhs)
                              : tf32_idesc(RAW ? p.rhs : M, h);
    uint32_t started = 0;
    for (const int kend = int(it.k0 + it.n); kk < kend; kk += kTcMmaWarps) {
      const int groups = it.stage_groups(kk - int(it.k0), G);
      const int s = ms;
      const uint32_t par = mph;
      if ((ms += kTcMmaWarps) >= D) {
        ms -= D;
        mph ^= 1u;
      }
      VBSR_PROF_T0(t_w);
      if (!wait_phase(cb.split0 + 8u * s, par, p, abort_flag, lane)) {
        ok = false;
        break;
      }
      VBSR_PROF_ADD(p, 3, t_w);
      VBSR_TRACE_ST(kk, 4);
      VBSR_PROF_T0(t_i);
      if (lane == 0) {
        if (math) {
          if (DIRECT) fence_proxy_async_smem();  // cp.async data, read by the tensor core
          tc_fence_after();
          const uint32_t sa = slots + 4u * uint32_t(s * SF);
          const uint32_t ss = sa + uint32_t(slot_stack_bytes(h, groups));
          if (TR) {
            for (int g = 0; g < groups; ++g) {  // [A | A_lo] x S^T
              tc_mma_tf32(tmem_d, sw32_desc(sa + 64u * h * g), sw32_desc(ss + T * g), idesc,
                          started);
              started = 1u;
            }
          } else {
            for (int g = 0; g < groups; ++g) {
              const uint64_t sdesc = sw32_desc(ss + T * g);
              const uint32_t ag = sa + 32u * h * g, lo_off = 32u * h * groups;  // A_lo region
              tc_mma_tf32(tmem_d, sdesc, sw32_desc(ag), idesc, started);          // S x A
              tc_mma_tf32(tmem_d, sdesc, sw32_desc(ag + lo_off), idesc, 1u);      // S x A_lo
              if (RAW)  // B_lo x A, into the same rows: S's lo rows follow all groups' raw rows
                tc_mma_tf32(tmem_d, sw32_desc(ss + T * (groups + g)), sw32_desc(ag), idesc, 1u);
              started = 1u;
            }
          }
        }
        tc_commit(cb.empty0 + 8u * s);  // the slot is free once these MMAs have read it
      }
      __syncwarp();
      VBSR_PROF_ADD(p, 10, t_i);
      VBSR_TRACE_ST(kk, 5);
    }
    if (!ok) break;
    if (lane == 0) tc_commit(cb.acc0 + 8u * buf);  // this warp's part of the item is issued
    __syncwarp();
    ++j;
  }
  VBSR_PROF_ADD(p, 9, t_all);
  // Every MMA this warp issued has completed before the CTA releases its tensor memory (bounded).
  if (lane == 0) tc_commit(cb.drain0 + 8u * i);
  __syncwarp();
  {
    const long long t0 = clock64();
    while (!mbar_try(cb.drain0 + 8u * i, 0) && clock64() - t0 < p.wait_limit) {
    }
  }
}

// Short block rows on the CUDA cores. Rows of height 8 or 16 waste most of a tcgen05 MMA (its M
// side is 64 rows) and pay a full pipeline stage per few hundred bytes of A, while their arithmetic
// is small; for RHS <= 32 the plan takes them out of the tensor-core schedule and the pre-pass
// launch computes them here in plain fp32 FMA (no operand splitting needed), one CTA of 8 warps per
// block row. A warp owns 8 rows of the tile (a 16-row block row has two row halves of 4 warps
// each) and a share of the row's blocks (every 8th, or every 4th for a row half), and walks them
// in 8-column groups: the group's B values are staged transposed, bs[k][c] (row stride RHS + 1:
// conflict-free), and its A values as as[k][r] in the warp's shared memory, while the next group's
// global loads are already in flight. Lane (c, row set) accumulates its column over its rows (per
// group a fresh fp32 partial of 8 FMAs, added into the accumulator). At the end the warps' partial
// tiles are summed in warp order through shared memory and the CTA stores the row's h x RHS tile
// of C once (no atomics, no global workspace).
struct CcParams {
  const CcItem* items;
  int count;
  const float* values;
  const uint32_t* blk_desc;
  const int64_t* value_off;  // each block's first value (the device format keeps the offsets)
  float* C;
  long long M;
};
constexpr int kCcWarps = 8;  // warps per block row

// smem floats per warp: bs (8 x (RHS + 1)) + as (8 x 8); the partial tile (8 x RHS) as well
template <int RHS>
__host__ __device__ constexpr int cc_warp_floats() {
  return 8 * (RHS + 1) + 64 > 8 * RHS ? 8 * (RHS + 1) + 64 : 8 * RHS;
}

// One 8-column group's global values in registers: lane i < 2 RHS holds float4 i of B (column
// i / 2, half i % 2; RHS 32: columns 16 + i / 2 in b1 as well), lane i < 16 float4 i of the
// warp's 8 A rows (row i / 2, storage half i % 2).
struct CcGroup {
  float4 b0, b1, a;
};

template <int RHS>
__device__ __forceinline__ void cc_load(CcGroup& x, const float* bcol, const float* ag,
                                        long long K, int lane) {
  const int cl = lane >> 1;
  if (lane < 2 * (RHS == 32 ? 16 : RHS))
    x.b0 = __ldg(reinterpret_cast<const float4*>(bcol + (long long)cl * K) + (lane & 1));
  if (RHS == 32)
    x.b1 = __ldg(reinterpret_cast<const float4*>(bcol + (long long)(16 + cl) * K) + (lane & 1));
  if (lane < 16) x.a = __ldg(reinterpret_cast<const float4*>(ag) + lane);
}

template <int RHS>
__device__ __forceinline__ void cc_stage(const CcGroup& x, float* bs, float* as, int lane) {
  if (lane < 2 * (RHS == 32 ? 16 : RHS)) {
    float* d = bs + (4 * (lane & 1)) * (RHS + 1) + (lane >> 1);
    d[0] = x.b0.x;
    d[RHS + 1] = x.b0.y;
    d[2 * (RHS + 1)] = x.b0.z;
    d[3 * (RHS + 1)] = x.b0.w;
  }
  if (RHS == 32) {
    float* d = bs + (4 * (lane & 1)) * (RHS + 1) + 16 + (lane >> 1);
    d[0] = x.b1.x;
    d[RHS + 1] = x.b1.y;
    d[2 * (RHS + 1)] = x.b1.z;
    d[3 * (RHS + 1)] = x.b1.w;
  }
  if (lane < 16) {
    // device format: row r's 8 values at 8 r, its 16-byte halves exchanged when bit 2 of r is set
    const int r = lane >> 1, kq = 4 * ((lane & 1) ^ ((r >> 2) & 1));
    as[(kq + 0) * 8 + r] = x.a.x;
    as[(kq + 1) * 8 + r] = x.a.y;
    as[(kq + 2) * 8 + r] = x.a.z;
    as[(kq + 3) * 8 + r] = x.a.w;
  }
}

template <int RHS>
__device__ void cc_row_cta(const CcParams& q, const CcItem& it, const float* __restrict__ B,
                           long long K, float* smem) {
  constexpr int L = 32 / RHS;  // lanes per column (row sets)
  constexpr int RPL = 8 / L;   // rows per lane (of the warp's 8)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = int(it.h);
  const int halves = H / 8, stride = kCcWarps / halves;  // warps per row half = block stride
  const int half = warp / stride, first = warp % stride;
  float* bs = smem + warp * cc_warp_floats<RHS>();
  float* as = bs + 8 * (RHS + 1);
  const int c = lane % RHS, r0 = (lane / RHS) * RPL;
  float acc[RPL];
#pragma unroll
  for (int r = 0; r < RPL; ++r) acc[r] = 0.0f;
  // this warp's groups: blocks b0 + first + stride j, each w / 8 groups; A of group g of a block at
  // (block start) + 8 H g floats, the warp's rows 8 half ... 8 half + 7 at + 64 half
  uint32_t b = it.b0 + uint32_t(first);
  const float* a = q.values;
  int g = 0, ngr = 0;
  const float* bcol = B;
  if (b < it.b1) {
    const uint32_t desc = __ldg(q.blk_desc + b);
    ngr = int((desc & 7u) + 1u);
    bcol = B + (long long)(desc & ~7u);
    a = q.values + __ldg(q.value_off + b);
  }
  CcGroup cur, nxt;
  if (b < it.b1) cc_load<RHS>(cur, bcol, a + 64 * half, K, lane);
  while (b < it.b1) {
    // the next group of this warp: the next one of this block, or the first of its next block
    uint32_t nb = b;
    int ng = g + 1, nngr = ngr;
    const float* na = a;
    const float* nbcol = bcol;
    if (ng == ngr) {
      nb = b + uint32_t(stride);
      ng = 0;
      if (nb < it.b1) {
        const uint32_t desc = __ldg(q.blk_desc + nb);
        nngr = int((desc & 7u) + 1u);
        nbcol = B + (long long)(desc & ~7u);
        na = q.values + __ldg(q.value_off + nb);
      }
    }
    if (nb < it.b1)
      cc_load<RHS>(nxt, nbcol + 8 * ng, na + (long long)H * 8 * ng + 64 * half, K, lane);
    cc_stage<RHS>(cur, bs, as, lane);
    __syncwarp();
    float part[RPL];
#pragma unroll
    for (int r = 0; r < RPL; ++r) part[r] = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float bv = bs[k * (RHS + 1) + c];
#pragma unroll
      for (int r = 0; r < RPL; ++r) part[r] = fmaf(as[k * 8 + r0 + r], bv, part[r]);
    }
#pragma unroll
    for (int r = 0; r < RPL; ++r) acc[r] += part[r];
    __syncwarp();
    b = nb;
    g = ng;
    ngr = nngr;
    a = na;
    bcol = nbcol;
    cur = nxt;
  }
  // partial tiles (8 rows x RHS) -> each warp's staging area; summed per row half in warp order
  float* part = smem + warp * cc_warp_floats<RHS>();
#pragma unroll
  for (int r = 0; r < RPL; ++r) part[(r0 + r) * RHS + c] = acc[r];
  __syncthreads();
  for (int e = threadIdx.x; e < H * RHS; e += blockDim.x) {
    const int r = e % H, cc = e / H;  // consecutive threads: consecutive rows of one column
    const int hh = r >> 3;
    float sum = 0.0f;
    for (int v = hh * stride; v < (hh + 1) * stride; ++v)
      sum += smem[v * cc_warp_floats<RHS>() + (r & 7) * RHS + cc];
    q.C[(long long)cc * q.M + it.c_row + r] = sum;
  }
  __syncthreads();
}

template <int RHS>
__device__ void cc_rows(const CcParams& q, const float* __restrict__ B, long long K, int item,
                        float* smem) {
  cc_row_cta<RHS>(q, q.items[item], B, K, smem);
}

// Pre-pass: the operand stacks S of all 8-column groups of B (K x rhs, column-major), one tile of
// stack_rows(rhs) rows x 8 floats per group (kg = k / 8) in the layout the MMA reads. Row-stacked
// form (rhs <= 32): row c holds the 8 values of RHS column c (raw, i.e. hi), row rhs + c their lo
// parts. Column-stacked form (rhs = 64, M = 128, half = 16): row 2*half*q + j holds column
// c = half*q + j, row 2*half*q + half + j its lo parts. The two 16-byte halves of row r are
// exchanged when bit 2 of r is set (32-byte swizzle). A block transposes kBsGroups consecutive
// groups through shared memory: it reads each RHS column's 8 * kBsGroups consecutive values
// (coalesced), then writes the kBsGroups tiles (contiguous) with 16-byte stores. Blocks from
// `stack_blocks` on compute the plan's short block rows on the CUDA cores instead (cc_rows).
constexpr int kBsGroupsWide = 16;    // groups per block iteration, rhs = 64 (at DRAM bandwidth)
constexpr int kBsGroupsNarrow = 32;  // rhs <= 32: more loads in flight per thread (latency-bound)
constexpr int kBsBlocksPerSm = 8;    // stacking blocks per SM of the pre-pass grid
__host__ __device__ constexpr int bs_groups(int rhs) {
  return rhs <= 32 ? kBsGroupsNarrow : kBsGroupsWide;
}
template <int RHS, bool RAW>
__global__ void __launch_bounds__(256, 4) bstack_kernel(const float* __restrict__ B, long long K,
                                                     float* __restrict__ out, int stack_blocks,
                                                     const CcParams cc) {
  constexpr int M = stack_m(RHS), half = M / 8, rows = stack_rows(RHS, RAW);
  constexpr int kBsGroups = bs_groups(RHS);
  constexpr int per_col = 2 * kBsGroups;  // float4s per column run
  constexpr int kCcFloat4s =
      RHS <= 32 ? kCcWarps * cc_warp_floats<(RHS <= 32 ? RHS : 32)>() / 4 : 0;
  // [c][kg][2 x float4] for stacking (up to 32 KB), or the CUDA-core warps' staging
  __shared__ float4 buf[RHS * per_col > kCcFloat4s ? RHS * per_col : kCcFloat4s];
  griddep_launch_dependents();  // the SpMM may start its prologue now (it waits before reading)
  if (RHS <= 32 && int(blockIdx.x) >= stack_blocks) {
    cc_rows<(RHS <= 32 ? RHS : 32)>(cc, B, K, int(blockIdx.x) - stack_blocks,
                                    reinterpret_cast<float*>(buf));
    return;
  }
  const long long ngroups = K >> 3;
  for (long long kg0 = (long long)blockIdx.x * kBsGroups; kg0 < ngroups;
       kg0 += (long long)stack_blocks * kBsGroups) {
    const int ng = int(ngroups - kg0 < kBsGroups ? ngroups - kg0 : kBsGroups);
    // read: each RHS column's run of 8 * kBsGroups values (coalesced)
    const float* src = B + 8 * kg0;
#pragma unroll 8
    for (int i = threadIdx.x; i < RHS * per_col; i += blockDim.x) {
      const int c = i / per_col, r = i % per_col;  // powers of two: shifts
      if (r < 2 * ng) buf[i] = __ldg(reinterpret_cast<const float4*>(src + (long long)c * K) + r);
    }
    __syncthreads();
    // write: tile g, row `row`, 16-byte piece `up` (2M float4s per tile, contiguous)
    float4* dst = reinterpret_cast<float4*>(out) + kg0 * (2 * rows);
#pragma unroll 4
    for (int i = threadIdx.x; i < ng * 2 * rows; i += blockDim.x) {
      const int g = i / (2 * rows), rem = i % (2 * rows);
      const int row = rem >> 1, up = rem & 1;
      int c;
      bool lo;
      if (row_stacked(RHS)) {  // rows c: raw B of column c; rows RHS + c: its lo part
        c = row % RHS;
        lo = row >= RHS;
      } else if (RAW) {  // raw rows only: row c is column c
        c = row;
        lo = false;
      } else {  // per quadrant q: rows of hi, then rows of lo, of columns half*q ...
        const int q = row / (2 * half), jj = row % (2 * half);
        c = q * half + jj % half;
        lo = jj >= half;
      }
      if (c < RHS) {
        const int u = up ^ ((row >> 2) & 1);
        float4 v = buf[c * per_col + 2 * g + u];
        if (lo) v = lo_part4(v);
        dst[i] = v;
      }
    }
    __syncthreads();
  }
}

// TR: row-stacked form (rhs <= 32); RAW: column-stacked form with raw-B stacks; DIRECT: those
// stacks' raw rows read from B itself (no pre-pass).
template <bool CHECK, bool TR, bool RAW, bool DIRECT>
__global__ void __launch_bounds__(32 * Roles<TR>::warps, 1) spmm_tc_kernel(const __grid_constant__ KernelParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t slots = (smem_addr(smem_raw) + 1023u) & ~1023u;  // 1024-aligned ring
  __shared__ __align__(8) uint64_t bars[3][kMaxStages];  // full, split, empty
  __shared__ __align__(8) uint64_t accbars[2][2];        // acc done, acc free
  __shared__ __align__(8) uint64_t drainbars[kTcMmaWarps];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ uint32_t stack_sense;
  const Task task = p.tasks[blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tc_alloc(smem_addr(&tmem_slot), kTmemAlloc);
    tc_relinquish();
  }
  if (threadIdx.x == 32) {
    if (p.timing) p.timing[2 * blockIdx.x] = global_ns();
    for (int s = 0; s < task.stages; ++s) {
      // TMA: one arrival + transaction bytes (DIRECT: + one cp.async arrival per feeder lane)
      mbar_init(smem_addr(&bars[0][s]), DIRECT ? 33u : 1u);
      mbar_init(smem_addr(&bars[1][s]), TR ? 1u : uint32_t(kCsSplitTeam));  // the split team
      mbar_init(smem_addr(&bars[2][s]), 1u);  // the MMA warp's tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&accbars[0][b]), uint32_t(kTcMmaWarps));
      mbar_init(smem_addr(&accbars[1][b]), 4u);  // the four warps of the buffer's epilogue set
    }
    for (int i = 0; i < kTcMmaWarps; ++i) mbar_init(smem_addr(&drainbars[i]), 1u);

    abort_flag = 0;
    mbar_fence_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  CtaBars cb;
  cb.full0 = smem_addr(&bars[0][0]);
  cb.split0 = smem_addr(&bars[1][0]);
  cb.empty0 = smem_addr(&bars[2][0]);
  cb.acc0 = smem_addr(&accbars[0][0]);
  cb.accfree0 = smem_addr(&accbars[1][0]);
  cb.drain0 = smem_addr(&drainbars[0]);

  if (!DIRECT && p.stack_flag != nullptr) {  // fused pre-pass: every warp stacks its share of B
    if (!(p.diag & VBSR_PLAN_DIAG_SKIP_PREPASS))
      stack_fused<TR, RAW>(p, (long long)blockIdx.x * Roles<TR>::warps + warp,
                           (long long)gridDim.x * Roles<TR>::warps, lane);
    fence_proxy_async_global();
    __syncthreads();
    if (threadIdx.x == 0) stack_sense = stack_arrive(p);
    __syncthreads();
  }

  using RL = Roles<TR>;
  if (warp < RL::mma0)
    tc_split_warp<CHECK, TR, RAW>(p, task, slots, cb, tmem_base, warp, lane, &abort_flag);
  else if (warp < RL::feeder0)
    tc_mma_warp<CHECK, TR, RAW, DIRECT>(p, task, slots, cb, tmem_base, warp - RL::mma0, lane,
                                        &abort_flag);
  else if (warp < RL::epi0)
    tc_feeder<CHECK, RAW, DIRECT>(p, task, slots, cb, warp - RL::feeder0, lane, &abort_flag,
                                  stack_sense);
  else  // the epilogue warps: TMEM quadrant warp % 4
    tc_epi_warp<CHECK, TR, RAW>(p, task, cb, tmem_base, warp & 3, (warp - RL::epi0) >> 2, lane,
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
