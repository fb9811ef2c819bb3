// vbsr_kernels.cuh — the sm_100a SpMM kernel: C = A * B for one plan's schedule.
//
// CTA = one producer warpgroup (4 warps; setmaxnreg lowers them to kProducerRegs registers) and two
// consumer warpgroups (8 compute warps raised to kConsumerRegs registers), one CTA per SM, each
// CTA executing one Task of the plan. The compute warps form teams of 1, 2 or 4 warps (fixed per task); each team
// walks its own instruction stream (item headers and k-chunks, compiled by the planner; see
// vbsr_internal.h) and owns a private ring of shared-memory stages guarded by "full" and "empty"
// mbarriers. Streams are read through lane-distributed register windows of 32 entries with the
// next window already in flight, so no descriptor load sits on the critical path. Producer warp w
// walks the streams of teams w, w+4, ... and, for each k-chunk (at most 32 block columns of one block),
// issues 1-D TMA bulk copies (cp.async.bulk) of
//   * the chunk's A values (one bulk copy of h*kc floats, contiguous in the device format; A streams
//     from HBM once, with an L2 evict-first hint), and
//   * the chunk's B rows (kc/8 2-D tensor copies of an 8-column x nw-row box, with an L2
//     evict-last hint because B is re-read by every block of the same block column),
// into a free stage, and arms the stage's full barrier with the byte count. Teams compute with
// fp32 FMA on CUDA cores from shared memory into a TM x TN register tile per thread, keep a
// per-block partial sum (so no single fp32 chain is longer than one block width), and store
// their tile of C straight from registers with 16-byte stores. Every C element is written by
// exactly one thread: no atomics, no workspace, and C needs no prior clearing.
//
// Every wait is bounded: a wait that exceeds the plan's cycle limit records VBSR_TIMEOUT in the
// plan's status word, raises a CTA-wide abort flag and unwinds; before the CTA exits after an
// abort, the producer waits (again bounded) for every copy it issued.
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
__device__ __forceinline__ bool chk_last(u64 e) { return ((e >> 62) & 1u) != 0; }

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

// ---- consumer ------------------------------------------------------------------------------------

// Runs one item (an h x nw tile, header already consumed): every chunk up to the next header or
// the end of the stream, then stores the tile. Returns false on abort.
template <int H, int NW, bool CHECK>
__device__ __forceinline__ bool consume_item(const KernelParams& p, u64 hdr, StreamWin& win,
                                             const float* stages, int stage_floats, int D,
                                             uint32_t full0, uint32_t empty0, int& s, uint32_t& ph,
                                             int tt, int lane, volatile int* abort_flag) {
  constexpr TileCfg cfg = tile_cfg(H, NW);
  constexpr int TM = cfg.tm, TN = cfg.tn, RG = H / TM, NG = NW / TN;
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
    const u64 e = win.peek();
    if (is_header(e)) break;
    win.advance(p.stream, lane);
    const int kc = chk_kc(e);
    if (!wait_phase(full0 + 8u * s, ph, p, abort_flag, lane)) return false;
    if (active && !(p.diag & VBSR_PLAN_DIAG_SKIP_MATH)) {
      const float* As = stages + s * stage_floats + pnl * 8 * kc;
      const float* Bs = stages + s * stage_floats + stage_b_offset(H) + ng * 8;
#pragma unroll 1
      for (int k8 = 0; k8 < kc; k8 += 8) {
        const float* Ak = As + k8 * 8;
        const float* Bk = Bs + k8 * NW;
#pragma unroll
        for (int kq = 0; kq < 8; kq += 4) {
          float4 bv[TN];
#pragma unroll
          for (int j = 0; j < TN; ++j)
            bv[j] = *reinterpret_cast<const float4*>(Bk + j * NG * 8 + kq);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            float a[TM];
            const float* ap = Ak + kq * 8;
            if constexpr (TM == 8) {
              const float4 x = *reinterpret_cast<const float4*>(ap + offa[kk][0]);
              const float4 y = *reinterpret_cast<const float4*>(ap + offa[kk][1]);
              a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w;
              a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
            } else if constexpr (TM == 4) {
              const float4 x = *reinterpret_cast<const float4*>(ap + offa[kk][0]);
              a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w;
            } else {
              const float2 x = *reinterpret_cast<const float2*>(ap + offa[kk][0]);
              a[0] = x.x; a[1] = x.y;
            }
#pragma unroll
            for (int j = 0; j < TN; ++j) {
              const float bk = kk == 0 ? bv[j].x : kk == 1 ? bv[j].y : kk == 2 ? bv[j].z : bv[j].w;
#pragma unroll
              for (int i = 0; i < TM; ++i) part[i][j] = fmaf(a[i], bk, part[i][j]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * s);
    if (++s == D) {
      s = 0;
      ph ^= 1u;
    }
    if (chk_last(e)) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          acc[i][j] += part[i][j];
          part[i][j] = 0.0f;
        }
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
                                          const float* stages, int sf, int D, uint32_t full0,
                                          uint32_t empty0, int& s, uint32_t& ph, int tt, int lane,
                                          volatile int* abort_flag) {
  constexpr int HALF = RHS > 8 ? RHS / 2 : RHS;
  if (hdr_nw(hdr) == RHS)
    return consume_item<H, RHS, CHECK>(p, hdr, win, stages, sf, D, full0, empty0, s, ph, tt, lane,
                                       abort_flag);
  return consume_item<H, HALF, CHECK>(p, hdr, win, stages, sf, D, full0, empty0, s, ph, tt, lane,
                                      abort_flag);
}

template <int RHS, bool CHECK>
__device__ void consumer(const KernelParams& p, const Task& task, const float* stages,
                         uint32_t full_base, uint32_t empty_base, int warp, int lane,
                         volatile int* abort_flag) {
  const int tw = task.team_warps;
  const int team = warp / tw;
  const int tt = (warp % tw) * 32 + lane;
  const uint32_t full0 = full_base + 8u * (team * kMaxStages);
  const uint32_t empty0 = empty_base + 8u * (team * kMaxStages);
  const float* my_stages = stages + team * task.stages * task.stage_floats;
  StreamWin win;
  win.init(p.stream, task.team_off[team], task.team_off[team + 1], lane);
  int s = 0;
  uint32_t ph = 0;
  while (!win.done()) {
    const u64 hdr = win.peek();
    win.advance(p.stream, lane);
    if (!is_header(hdr)) {  // malformed stream: a chunk without a header
      if (lane == 0) record_status(p.status, VBSR_BOUNDS_VIOLATION, win.pos);
      break;
    }
    bool ok = true;
    switch (hdr_h(hdr)) {
#define VBSR_CASE_H(HH)                                                                          \
  case HH:                                                                                       \
    ok = consume_h<RHS, HH, CHECK>(p, hdr, win, my_stages, task.stage_floats, task.stages, full0, \
                                   empty0, s, ph, tt, lane, abort_flag);                         \
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
    if (!ok) break;
  }
}

// ---- producer ------------------------------------------------------------------------------------

// Current item of a team as seen by the producer.
struct ProdItem {
  int h, n0, nw;
};

// Producer warp `pw` serves teams pw, pw + kProducerWarps, ... (NT of them).
template <int NT, bool CHECK>
__device__ void producer(const KernelParams& p, const Task& task, float* stages, uint32_t full_base,
                         uint32_t empty_base, int pw, int lane, volatile int* abort_flag) {
  const int D = task.stages;
  const int sf = task.stage_floats;
  const uint64_t pol_a = policy_evict_first();
  const uint64_t pol_b = policy_evict_last();
  StreamWin win[NT];
  ProdItem it[NT];
  int slot[NT];
  uint32_t phase[NT], filled[NT], lastpar[NT];
  uint32_t live = 0;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int team = pw + j * kProducerWarps;
    win[j].init(p.stream, task.team_off[team], task.team_off[team + 1], lane);
    it[j] = ProdItem{8, 0, 8};
    slot[j] = 0;
    phase[j] = filled[j] = lastpar[j] = 0;
    if (!win[j].done()) live |= 1u << j;
  }
  int issued0 = 0;  // chunks issued for team 0 (debug drop hook)
  int j = 0;
  while (live) {
    // next live team, round robin
    while (!(live & (1u << j))) j = (j + 1 == NT) ? 0 : j + 1;
    bool stop = false;
#pragma unroll
    for (int jj = 0; jj < NT; ++jj) {
      if (jj != j) continue;  // static indexing of the per-team registers
      // Headers need no stage: take them as they come.
      u64 e = win[jj].peek();
      while (is_header(e)) {
        it[jj].h = hdr_h(e);
        it[jj].n0 = hdr_n0(e);
        it[jj].nw = hdr_nw(e);
        win[jj].advance(p.stream, lane);
        if (win[jj].done()) break;
        e = win[jj].peek();
      }
      if (win[jj].done()) {
        live &= ~(1u << jj);
        break;
      }
      const int s = slot[jj];
      const int team = pw + jj * kProducerWarps;
      const uint32_t empty_bar = empty_base + 8u * (team * kMaxStages + s);
      const uint32_t full_bar = full_base + 8u * (team * kMaxStages + s);
      if (!wait_phase(empty_bar, phase[jj] ^ 1u, p, abort_flag, lane)) {
        stop = true;
        break;
      }
      const long long val = chk_val(e), colk = chk_colk(e);
      const int w = chk_w(e), k0 = chk_k0(e), kc = chk_kc(e);
      const int h = it[jj].h, nw = it[jj].nw, n0 = it[jj].n0;
      const bool drop = (team == 0 && issued0 == p.drop_stage);
      if (team == 0) ++issued0;
      bool in_bounds = true;
      if (CHECK)
        in_bounds = val + (long long)h * w <= p.nvalues && colk - k0 + w <= p.K &&
                    n0 + nw <= p.rhs;
      if (drop) {
        // withhold the stage entirely (debug): no arrival, no copies
      } else if (p.diag & VBSR_PLAN_DIAG_SKIP_COPIES) {
        if (lane == 0) mbar_arrive(full_bar);
      } else if (!in_bounds) {
        if (lane == 0) {
          record_status(p.status, VBSR_BOUNDS_VIOLATION, int(blockIdx.x));
          mbar_arrive(full_bar);  // release the consumers without touching memory
        }
      } else {
        float* st = stages + (team * D + s) * sf;
        if (lane == 0) {
          mbar_arrive_expect_tx(full_bar, uint32_t((h + nw) * 4 * kc));
          bulk_g2s(smem_addr(st), p.values + val + (long long)h * k0, uint32_t(h * 4 * kc),
                   full_bar, pol_a);
        } else if (lane <= (kc >> 3)) {
          const int g = lane - 1;
          const CUtensorMap* map = (nw == p.rhs) ? &p.b_full : &p.b_half;
          tensor2d_g2s(smem_addr(st + stage_b_offset(h) + g * nw * 8), map, int(colk) + 8 * g, n0,
                       full_bar, pol_b);
        }
        filled[jj] |= 1u << s;
        lastpar[jj] = (lastpar[jj] & ~(1u << s)) | (phase[jj] << s);
      }
      if (++slot[jj] == D) {
        slot[jj] = 0;
        phase[jj] ^= 1u;
      }
      win[jj].advance(p.stream, lane);
      if (win[jj].done()) live &= ~(1u << jj);
    }
    if (stop) break;
    j = (j + 1 == NT) ? 0 : j + 1;
  }
  __syncwarp();
  // After an abort, wait (bounded) for the last fill of every slot so that no bulk copy is still
  // writing this CTA's shared memory when it exits.
  if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      for (int s = 0; s < D; ++s) {
        if (!(filled[j] & (1u << s))) continue;
        const uint32_t bar = full_base + 8u * ((pw + j * kProducerWarps) * kMaxStages + s);
        const uint32_t par = (lastpar[j] >> s) & 1u;
        const long long t0 = clock64();
        while (!mbar_try(bar, par) && clock64() - t0 < p.wait_limit) {
        }
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
  volatile int* abort_v = &abort_flag;

  if (warp < kProducerWarps) {
    regs_dec<kProducerRegs>();
    if (tw == 1)
      producer<2, CHECK>(p, task, stages, full_base, empty_base, warp, lane, abort_v);
    else if (tw == 2)
      producer<1, CHECK>(p, task, stages, full_base, empty_base, warp, lane, abort_v);
    else if (warp < 2)
      producer<1, CHECK>(p, task, stages, full_base, empty_base, warp, lane, abort_v);
  } else {
    regs_inc<kConsumerRegs>();
    consumer<RHS, CHECK>(p, task, stages, full_base, empty_base, warp - kProducerWarps, lane,
                         abort_v);
  }
  __syncthreads();
  if (threadIdx.x == 0 && p.timing) p.timing[2 * blockIdx.x + 1] = global_ns();
}

}  // namespace vbsr_b200
