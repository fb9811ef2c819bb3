// vbsr_kernels.cuh — the sm_100a SpMM kernel: C = A * B for one plan's schedule.
//
// CTA = kConsumerWarps warps, one CTA per SM, each CTA executing one Task of the plan. The warps
// form teams of 1, 2 or 4 warps (fixed per task); each team walks its own instruction stream (item
// headers and k-chunks, compiled by the planner; see vbsr_internal.h) and owns a private ring of
// D shared-memory stages guarded by "full" and "empty" mbarriers. Streams are read through
// lane-distributed register windows of 32 entries with the next window already in flight, so no
// descriptor load sits on the critical path.
//
// The team's leader warp is also its producer: it keeps a second stream cursor D-1 chunks ahead
// and, each time the team starts a chunk, waits for the stage freed by the previous chunk and
// issues the chunk D-1 ahead as TMA copies into it:
//   * the chunk's A values (one cp.async.bulk of h*kc floats, contiguous in the device format;
//     A streams from HBM once, with an L2 evict-first hint), and
//   * the chunk's B rows (kc/8 2-D tensor copies cp.async.bulk.tensor of an 8-column x nw-row
//     box, with an L2 evict-last hint because B is re-read by every block of the same block column),
// arming the stage's full barrier with the byte count. Issuing costs a handful of instructions
// per chunk, so no separate producer warps are needed and every warp of the CTA computes (with up
// to 255 registers per thread).
//
// Teams compute with fp32 FMA on CUDA cores from shared memory into a TM x TN register tile per
// thread, software-pipelined over k-quads, keep a per-block partial sum (so no single fp32 chain
// is longer than one block width), and store their tile of C straight from registers with 16-byte
// stores. Every C element is written by exactly one thread: no atomics, no workspace, and C needs
// no prior clearing.
//
// Every wait is bounded: a wait that exceeds the plan's cycle limit records VBSR_TIMEOUT in the
// plan's status word, raises a CTA-wide abort flag and unwinds; before the CTA exits after an
// abort, each leader waits (again bounded) for every copy it issued.
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

// Issues the next chunk of the team's stream into the next ring slot (waiting until every warp of
// the team has released that slot). Warp-collective. Returns false on abort.
template <bool CHECK>
__device__ __forceinline__ bool issue_next(const KernelParams& p, Issuer& is, float* team_stages,
                                           int sf, int D, int cols, uint32_t full0,
                                           uint32_t empty0, int team, int lane,
                                           volatile int* abort_flag) {
  while (!is.win.done()) {
    const u64 e = is.win.peek();
    if (!is_header(e)) break;
    is.h = hdr_h(e);
    is.n0 = hdr_n0(e);
    is.nw = hdr_nw(e);
    is.win.advance(p.stream, lane);
  }
  if (is.win.done()) return true;
  const int s = is.slot;
  const uint32_t full_bar = full0 + 8u * s;
  if (!wait_phase(empty0 + 8u * s, is.ph ^ 1u, p, abort_flag, lane)) return false;
  const int h = is.h, nw = is.nw, n0 = is.n0;
  const bool drop = (team == 0 && is.issued == p.drop_stage);
  ++is.issued;
  float* st = team_stages + s * sf;
  const CUtensorMap* map = (nw == p.rhs) ? &p.b_full : &p.b_half;
  const bool copy = !drop && !(p.diag & VBSR_PLAN_DIAG_SKIP_COPIES);
  bool in_bounds = true;
  int c0 = 0;
  while (!is.win.done()) {  // the stage's chunks (ends at a stage-end mark)
    const u64 e = is.win.peek();
    is.win.advance(p.stream, lane);
    const long long val = chk_val(e), colk = chk_colk(e);
    const int w = chk_w(e), k0 = chk_k0(e), kc = chk_kc(e);
    bool ok = true;
    if (CHECK)
      ok = val + (long long)h * w <= p.nvalues && colk - k0 + w <= p.K && n0 + nw <= p.rhs &&
           c0 + kc <= cols;
    in_bounds = in_bounds && ok;
    if (copy && ok) {
      if (lane == 0) {
        mbar_expect_tx(full_bar, uint32_t((h + nw) * 4 * kc));
        bulk_g2s(smem_addr(st + h * c0), p.values + val + (long long)h * k0, uint32_t(h * 4 * kc),
                 full_bar, policy_evict_first());
      } else if (lane <= (kc >> 3)) {
        const int g = lane - 1;
        tensor2d_g2s(smem_addr(st + stage_b_offset(h, cols) + ((c0 >> 3) + g) * nw * 8), map,
                     int(colk) + 8 * g, n0, full_bar, policy_evict_last());
      }
    }
    c0 += kc;
    if (chk_stage_end(e)) break;
  }
  if (!drop) {
    if (lane == 0) {
      if (!in_bounds) record_status(p.status, VBSR_BOUNDS_VIOLATION, int(blockIdx.x));
      mbar_arrive(full_bar);  // the stage's bytes were announced chunk by chunk
    }
    if (copy) {
      is.filled |= 1u << s;
      is.lastpar = (is.lastpar & ~(1u << s)) | (is.ph << s);
    }
  }
  if (++is.slot == D) {
    is.slot = 0;
    is.ph ^= 1u;
  }
  return true;
}

// ---- consumer side -------------------------------------------------------------------------------

// Operands of one k-quad (4 block columns) for a TM x TN thread tile.
template <int TM, int TN>
struct Frag {
  float a[4][TM];
  float4 b[TN];
};

// Loads quad q of the stage: A from the XOR-swizzled panel chunk (offa = per-thread unit offsets),
// B from the 8-column boxes (column n of box g at g*nw*8 + n*8).
template <int TM, int TN, int NG>
__device__ __forceinline__ void load_frag(Frag<TM, TN>& f, const float* As, const float* Bs, int q,
                                          const int (&offa)[4][2], int nw) {
  const float* ap = As + q * 32;                          // 8 units of 16 B per quad
  const float* bp = Bs + (q >> 1) * nw * 8 + (q & 1) * 4;  // box q/2, half q%2
#pragma unroll
  for (int j = 0; j < TN; ++j) f.b[j] = *reinterpret_cast<const float4*>(bp + j * NG * 8);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    if constexpr (TM == 8) {
      const float4 x = *reinterpret_cast<const float4*>(ap + offa[kk][0]);
      const float4 y = *reinterpret_cast<const float4*>(ap + offa[kk][1]);
      f.a[kk][0] = x.x; f.a[kk][1] = x.y; f.a[kk][2] = x.z; f.a[kk][3] = x.w;
      f.a[kk][4] = y.x; f.a[kk][5] = y.y; f.a[kk][6] = y.z; f.a[kk][7] = y.w;
    } else if constexpr (TM == 4) {
      const float4 x = *reinterpret_cast<const float4*>(ap + offa[kk][0]);
      f.a[kk][0] = x.x; f.a[kk][1] = x.y; f.a[kk][2] = x.z; f.a[kk][3] = x.w;
    } else {
      const float2 x = *reinterpret_cast<const float2*>(ap + offa[kk][0]);
      f.a[kk][0] = x.x; f.a[kk][1] = x.y;
    }
  }
}

template <int TM, int TN>
__device__ __forceinline__ void fma_frag(float (&part)[TM][TN], const Frag<TM, TN>& f) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const float bk = kk == 0 ? f.b[j].x : kk == 1 ? f.b[j].y : kk == 2 ? f.b[j].z : f.b[j].w;
#pragma unroll
      for (int i = 0; i < TM; ++i) part[i][j] = fmaf(f.a[kk][i], bk, part[i][j]);
    }
}

// Per-team context shared by the item routines.
struct TeamCtx {
  float* stages;       // the team's ring
  int sf, D, cols;     // floats per stage, ring depth, block columns per stage
  uint32_t full0, empty0;
  int team, tt, lane;
  bool leader;         // this warp issues the team's copies
};

// Runs one item (an h x nw tile, header already consumed): every chunk up to the next header or
// the end of the stream, then stores the tile. Returns false on abort.
template <int H, int NW, bool CHECK>
__device__ __forceinline__ bool consume_item(const KernelParams& p, u64 hdr, StreamWin& win,
                                             Issuer& is, const TeamCtx& c, int& s, uint32_t& ph,
                                             volatile int* abort_flag) {
  constexpr TileCfg cfg = tile_cfg(H, NW);
  constexpr int TM = cfg.tm, TN = cfg.tn, RG = H / TM, NG = NW / TN;
  const int tt = c.tt, lane = c.lane;
  const bool active = tt < cfg.threads;
  const int rg = tt % RG, ng = tt / RG;
  const int r0 = rg * TM, pnl = r0 >> 3, xf = panel_xor(pnl);
  // A: offsets (floats) of the thread's 16-byte units for the 4 columns of a k-quad, relative to
  // the quad's first unit (panel format: unit q = 2k + (row/4 & 1), stored at q ^ xf).
  int offa[4][2];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int h2 = (TM == 8) ? hh : ((r0 >> 2) & 1);
      offa[kk][hh] = (((2 * kk + h2) ^ xf) << 2) + ((TM == 2) ? (r0 & 3) : 0);
    }

  float acc[TM][TN], part[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = part[i][j] = 0.0f;

  while (!win.done()) {
    if (is_header(win.peek())) break;
    if (!wait_phase(c.full0 + 8u * s, ph, p, abort_flag, lane)) return false;
    // keep the ring D-1 stages ahead: the slot freed by the previous stage gets the next copies
    if (c.leader && !issue_next<CHECK>(p, is, c.stages, c.sf, c.D, c.cols, c.full0, c.empty0,
                                       c.team, lane, abort_flag))
      return false;
    const float* stage = c.stages + s * c.sf;
    int c0 = 0;
    while (!win.done()) {  // the stage's chunks
      const u64 e = win.peek();
      win.advance(p.stream, lane);
      const int kc = chk_kc(e);
      if (active && !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH)) {
        const float* As = stage + H * c0 + pnl * 8 * kc;
        const float* Bs = stage + stage_b_offset(H, c.cols) + (c0 >> 3) * NW * 8 + ng * 8;
        // Software-pipelined over k-quads: the operands of quad q+1 are loaded from shared
        // memory while the FMAs of quad q run (two register fragments, alternating).
        Frag<TM, TN> f0, f1;
        const int nq = kc >> 2;  // even: kc is a multiple of 8
        load_frag<TM, TN, NG>(f0, As, Bs, 0, offa, NW);
#pragma unroll 1
        for (int q = 0; q < nq; q += 2) {
          load_frag<TM, TN, NG>(f1, As, Bs, q + 1, offa, NW);
          fma_frag<TM, TN>(part, f0);
          if (q + 2 < nq) load_frag<TM, TN, NG>(f0, As, Bs, q + 2, offa, NW);
          fma_frag<TM, TN>(part, f1);
        }
      }
      c0 += kc;
      if (chk_k0(e) + kc == chk_w(e)) {  // block done: fold its partial sums in
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            acc[i][j] += part[i][j];
            part[i][j] = 0.0f;
          }
      }
      if (chk_stage_end(e)) break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(c.empty0 + 8u * s);
    if (++s == c.D) {
      s = 0;
      ph ^= 1u;
    }
  }

  const int c_row = hdr_crow(hdr), n0 = hdr_n0(hdr);
  if (CHECK && ((long long)c_row + H > p.M || n0 + NW > p.rhs)) {
    if (tt == 0) record_status(p.status, VBSR_BOUNDS_VIOLATION, c_row);
    return true;
  }
  if (active) {
    float* cb = p.C + (long long)c_row + r0;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      float* dst = cb + (long long)(n0 + ng + j * NG) * p.M;
      if constexpr (TM == 8) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0][j], acc[1][j], acc[2][j], acc[3][j]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4][j], acc[5][j], acc[6][j], acc[7][j]);
      } else if constexpr (TM == 4) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0][j], acc[1][j], acc[2][j], acc[3][j]);
      } else {
        reinterpret_cast<float2*>(dst)[0] = make_float2(acc[0][j], acc[1][j]);
      }
    }
  }
  return true;
}

template <int RHS, int H, bool CHECK>
__device__ __forceinline__ bool consume_h(const KernelParams& p, u64 hdr, StreamWin& win,
                                          Issuer& is, const TeamCtx& c, int& s, uint32_t& ph,
                                          volatile int* abort_flag) {
  constexpr int HALF = RHS > 8 ? RHS / 2 : RHS;
  if (hdr_nw(hdr) == RHS) return consume_item<H, RHS, CHECK>(p, hdr, win, is, c, s, ph, abort_flag);
  return consume_item<H, HALF, CHECK>(p, hdr, win, is, c, s, ph, abort_flag);
}

template <int RHS, bool CHECK>
__device__ void run_team(const KernelParams& p, const Task& task, float* stages, uint32_t full_base,
                         uint32_t empty_base, int warp, int lane, volatile int* abort_flag) {
  const int tw = task.team_warps;
  TeamCtx c;
  c.team = warp / tw;
  c.tt = (warp % tw) * 32 + lane;
  c.lane = lane;
  c.leader = (warp % tw) == 0;
  c.D = task.stages;
  c.sf = task.stage_floats;
  c.cols = task.stage_cols;
  c.full0 = full_base + 8u * (c.team * kMaxStages);
  c.empty0 = empty_base + 8u * (c.team * kMaxStages);
  c.stages = stages + c.team * c.D * c.sf;
  const int b = task.team_off[c.team], e = task.team_off[c.team + 1];
  StreamWin win;
  win.init(p.stream, b, e, lane);
  Issuer is;
  is.h = 8;
  is.n0 = 0;
  is.nw = 8;
  is.slot = 0;
  is.ph = 0;
  is.filled = is.lastpar = 0;
  is.issued = 0;
  bool ok = true;
  if (c.leader) {
    is.win.init(p.stream, b, e, lane);
    for (int i = 0; i < c.D - 1 && ok; ++i)
      ok = issue_next<CHECK>(p, is, c.stages, c.sf, c.D, c.cols, c.full0, c.empty0, c.team, lane,
                             abort_flag);
  }
  int s = 0;
  uint32_t ph = 0;
  while (ok && !win.done()) {
    const u64 hdr = win.peek();
    win.advance(p.stream, lane);
    if (!is_header(hdr)) {  // malformed stream: a chunk without a header
      if (lane == 0) record_status(p.status, VBSR_BOUNDS_VIOLATION, win.pos);
      break;
    }
    switch (hdr_h(hdr)) {
#define VBSR_CASE_H(HH)                                                \
  case HH:                                                             \
    ok = consume_h<RHS, HH, CHECK>(p, hdr, win, is, c, s, ph, abort_flag); \
    break;
      VBSR_CASE_H(8)
      VBSR_CASE_H(16)
      VBSR_CASE_H(24)
      VBSR_CASE_H(32)
      VBSR_CASE_H(40)
      VBSR_CASE_H(48)
      VBSR_CASE_H(56)
      VBSR_CASE_H(64)
#undef VBSR_CASE_H
    }
  }
  // After an abort, wait (bounded) for the last fill of every slot this leader issued so that no
  // bulk copy is still writing the CTA's shared memory when it exits.
  if (c.leader && __shfl_sync(0xffffffffu, *abort_flag, 0)) {
    for (int sl = 0; sl < c.D; ++sl) {
      if (!(is.filled & (1u << sl))) continue;
      const uint32_t bar = c.full0 + 8u * sl;
      const uint32_t par = (is.lastpar >> sl) & 1u;
      const long long t0 = clock64();
      while (!mbar_try(bar, par) && clock64() - t0 < p.wait_limit) {
      }
    }
  }
}

__device__ __forceinline__ u64 global_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- kernel --------------------------------------------------------------------------------------

template <int RHS, bool CHECK>
__global__ void __launch_bounds__(kThreads, 1) spmm_kernel(const __grid_constant__ KernelParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1 KB-aligned stage base (the host adds 1 KB of slack to the dynamic allocation)
  float* stages = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[2][kConsumerWarps][kMaxStages];
  __shared__ int abort_flag;
  const Task task = p.tasks[blockIdx.x];
  const int tw = task.team_warps;
  const int nt = kConsumerWarps / tw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full_base = smem_addr(&bars[0][0][0]);
  const uint32_t empty_base = smem_addr(&bars[1][0][0]);
  if (threadIdx.x == 0) {
    if (p.timing) p.timing[2 * blockIdx.x] = global_ns();
    for (int j = 0; j < nt; ++j)
      for (int s = 0; s < task.stages; ++s) {
        mbar_init(full_base + 8u * (j * kMaxStages + s), 1u);
        mbar_init(empty_base + 8u * (j * kMaxStages + s), uint32_t(tw));
      }
    abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  run_team<RHS, CHECK>(p, task, stages, full_base, empty_base, warp, lane, &abort_flag);
  __syncthreads();
  if (threadIdx.x == 0 && p.timing) p.timing[2 * blockIdx.x + 1] = global_ns();
}

}  // namespace vbsr_b200
