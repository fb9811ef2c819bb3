// vbsr_kernels.cuh — the sm_100a SpMM kernel: C = A * B for one plan's schedule.
//
// CTA = kConsumerWarps compute warps + 1 producer warp, one CTA per SM, each CTA executing one
// Task of the plan. The compute warps form teams of 1, 2 or 4 warps (fixed per task); each team
// owns a list of work items (block rows or RHS-column halves of heavy block rows) and a private
// ring of shared-memory stages guarded by "full" and "empty" mbarriers. The producer warp walks
// every team's items in the same order as the team, and for each k-chunk of each block (at most
// 32 block columns) issues 1-D TMA bulk copies (cp.async.bulk) of
//   * the chunk's A row panels (h/8 copies of 8*kc floats; A values stream from HBM once, with an
//     L2 evict-first hint), and
//   * the chunk's B rows (nw copies of kc floats, with an L2 evict-last hint because every B row
//     is re-read by every block of the same block column),
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
#include <cstdint>

#include "vbsr_internal.h"
#include "vbsr_ptx.cuh"
#include "vbsr_tiles.h"

namespace vbsr_b200 {

struct KernelParams {
  const Item* items;
  const Task* tasks;
  const uint32_t* blk;  // per-block descriptors
  const float* values;  // re-laid-out values
  const float* B;
  float* C;
  long long M, K, nvalues;
  int rhs;
  int* status;
  int drop_stage;       // debug: stage number (per CTA, team 0) the producer withholds; < 0 off
  long long wait_limit; // SM clocks a single wait may take before it is declared stalled
};

__device__ __forceinline__ void record_status(int* status, int code, int info) {
  if (atomicCAS(status + kStatusCode, 0, code) == 0) status[kStatusInfo] = info;
}

// Bounds check of one item against the matrix (used by the checked kernel build only). Producer
// and consumers evaluate it identically, so both skip a bad item.
__device__ __forceinline__ bool item_in_bounds(const KernelParams& p, const Item& it) {
  if (it.h < 8 || it.h > 64 || (it.h & 7) || it.n0 < 0 || it.nw < 8 || it.n0 + it.nw > p.rhs ||
      it.c_row < 0 || (long long)it.c_row + it.h > p.M || it.val_off < 0 || it.nblk < 0)
    return false;
  long long v = it.val_off;
  for (int b = 0; b < it.nblk; ++b) {
    const uint32_t d = p.blk[it.blk_begin + b];
    const int w = int((d & 7u) + 1u) * 8;
    const long long col = (long long)(d & ~7u);
    if (col + w > p.K) return false;
    v += (long long)it.h * w;
    if (v > p.nvalues) return false;
  }
  return true;
}

// Warp-collective wait for phase `parity` of `bar`; every lane polls the barrier itself (so each
// lane gets the barrier's acquire ordering), and every decision is made uniformly by the warp.
// Returns false if the CTA aborted or the wait exceeded p.wait_limit SM clocks.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, const KernelParams& p,
                                           volatile int* abort_flag, int lane) {
  const long long t0 = clock64();
  while (true) {
    const bool ok = mbar_try(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
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

template <int H, int NW>
__device__ __forceinline__ bool consume_item(const KernelParams& p, const Item& item,
                                             const float* stages, int stage_floats, int D,
                                             uint32_t full0, uint32_t empty0, int& s, uint32_t& ph,
                                             int tt, int lane, volatile int* abort_flag) {
  constexpr TileCfg cfg = tile_cfg(H, NW);
  constexpr int TM = cfg.tm, TN = cfg.tn, RG = H / TM;
  constexpr int PS = a_panel_stride(TM);
  const bool active = tt < cfg.threads;
  const int rg = tt % RG, ng = tt / RG;
  const int a_off = ((rg * TM) / 8) * PS + (rg * TM) % 8;
  const int b_off = stage_b_offset(H, TM) + b_row_offset(ng * TN, TN);

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  for (int b = 0; b < item.nblk; ++b) {
    const uint32_t d = __ldg(p.blk + item.blk_begin + b);
    const int w = int((d & 7u) + 1u) * 8;
    float part[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) part[i][j] = 0.0f;

    for (int k0 = 0; k0 < w; k0 += kChunk) {
      const int kc = min(kChunk, w - k0);
      if (!wait_phase(full0 + 8u * s, ph, p, abort_flag, lane)) return false;
      if (active) {
        const float* As = stages + s * stage_floats + a_off;
        const float* Bs = stages + s * stage_floats + b_off;
#pragma unroll 1
        for (int k = 0; k < kc; k += 8) {
#pragma unroll
          for (int kq = 0; kq < 8; kq += 4) {
            float4 bv[TN];
#pragma unroll
            for (int j = 0; j < TN; ++j)
              bv[j] = *reinterpret_cast<const float4*>(Bs + j * kBRow + k + kq);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              float a[TM];
              const float* ap = As + (k + kq + kk) * 8;
              if constexpr (TM == 8) {
                const float4 x = *reinterpret_cast<const float4*>(ap);
                const float4 y = *reinterpret_cast<const float4*>(ap + 4);
                a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w;
                a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
              } else if constexpr (TM == 4) {
                const float4 x = *reinterpret_cast<const float4*>(ap);
                a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w;
              } else {
                const float2 x = *reinterpret_cast<const float2*>(ap);
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
    }
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] += part[i][j];
  }

  if (active) {
    float* cb = p.C + (long long)item.c_row + rg * TM;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      float* dst = cb + (long long)(item.n0 + ng * TN + j) * p.M;
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

template <int RHS, int H>
__device__ __forceinline__ bool consume_h(const KernelParams& p, const Item& item,
                                          const float* stages, int sf, int D, uint32_t full0,
                                          uint32_t empty0, int& s, uint32_t& ph, int tt, int lane,
                                          volatile int* abort_flag) {
  constexpr int HALF = RHS > 8 ? RHS / 2 : RHS;
  if (item.nw == RHS)
    return consume_item<H, RHS>(p, item, stages, sf, D, full0, empty0, s, ph, tt, lane, abort_flag);
  return consume_item<H, HALF>(p, item, stages, sf, D, full0, empty0, s, ph, tt, lane, abort_flag);
}

// ---- producer ------------------------------------------------------------------------------------

struct TeamCursor {
  int it, ie;        // next item, end of the team's item list
  int b, be;         // current block, end of the item's blocks
  int k0, w;         // chunk start within the block, block width
  long long val;     // value offset of the current block
  long long col;     // scalar column offset of the current block
  int h, n0, nw, tm, tn;
  int s;             // next ring slot
  uint32_t ph;       // ring phase
  uint32_t filled;   // bit s: slot s has been filled at least once
  uint32_t lastpar;  // bit s: parity of the last fill of slot s
};

template <bool CHECK>
__device__ __forceinline__ bool cursor_load_item(const KernelParams& p, TeamCursor& q) {
  while (q.it < q.ie) {
    const Item item = p.items[q.it];
    if (item.nblk == 0 || (CHECK && !item_in_bounds(p, item))) {
      ++q.it;
      continue;
    }
    q.h = item.h;
    q.n0 = item.n0;
    q.nw = item.nw;
    const TileCfg c = tile_cfg(item.h, item.nw);
    q.tm = c.tm;
    q.tn = c.tn;
    q.b = item.blk_begin;
    q.be = item.blk_begin + item.nblk;
    q.val = item.val_off;
    const uint32_t d = __ldg(p.blk + q.b);
    q.w = int((d & 7u) + 1u) * 8;
    q.col = (long long)(d & ~7u);
    q.k0 = 0;
    return true;
  }
  return false;
}

// Advances past the chunk just issued; false when the team has no chunk left.
template <bool CHECK>
__device__ __forceinline__ bool cursor_advance(const KernelParams& p, TeamCursor& q) {
  q.k0 += kChunk;
  if (q.k0 < q.w) return true;
  q.val += (long long)q.h * q.w;
  if (++q.b < q.be) {
    const uint32_t d = __ldg(p.blk + q.b);
    q.w = int((d & 7u) + 1u) * 8;
    q.col = (long long)(d & ~7u);
    q.k0 = 0;
    return true;
  }
  ++q.it;
  return cursor_load_item<CHECK>(p, q);
}

template <bool CHECK>
__device__ void producer(const KernelParams& p, const Task& task, float* stages, uint32_t full_base,
                         uint32_t empty_base, int lane, volatile int* abort_flag) {
  const int nt = kConsumerWarps / task.team_warps;
  const int D = task.stages;
  const int sf = task.stage_floats;
  const uint64_t pol_a = policy_evict_first();
  const uint64_t pol_b = policy_evict_last();
  TeamCursor cur[kConsumerWarps];
  uint32_t live = 0;
  for (int j = 0; j < nt; ++j) {
    TeamCursor& q = cur[j];
    q.it = task.team_off[j];
    q.ie = task.team_off[j + 1];
    q.s = 0;
    q.ph = 0;
    q.filled = 0;
    q.lastpar = 0;
    if (cursor_load_item<CHECK>(p, q)) live |= 1u << j;
  }
  int issued0 = 0;  // stages issued for team 0 (debug drop hook)
  long long t_stall = clock64();
  while (live) {
    bool progressed = false;
    for (int j = 0; j < nt; ++j) {
      if (!(live & (1u << j))) continue;
      TeamCursor& q = cur[j];
      const uint32_t empty_bar = empty_base + 8u * (j * kMaxStages + q.s);
      const uint32_t full_bar = full_base + 8u * (j * kMaxStages + q.s);
      // every lane probes (each gets the barrier's acquire ordering); act only when all agree
      if (!__all_sync(0xffffffffu, mbar_test(empty_bar, q.ph ^ 1u))) continue;
      progressed = true;
      const int kc = min(kChunk, q.w - q.k0);
      const bool drop = (j == 0 && issued0 == p.drop_stage);
      if (j == 0) ++issued0;
      if (!drop) {
        const int ps = a_panel_stride(q.tm);
        const int panels = q.h / 8;
        const uint32_t a_bytes = uint32_t(panels * 32 * kc);
        const uint32_t b_bytes = uint32_t(q.nw * 4 * kc);
        float* st = stages + (j * D + q.s) * sf;
        if (lane == 0) mbar_arrive_expect_tx(full_bar, a_bytes + b_bytes);
        __syncwarp();
        if (lane < panels) {
          const float* src = p.values + q.val + (long long)lane * 8 * q.w + q.k0 * 8;
          bulk_g2s(smem_addr(st + lane * ps), src, uint32_t(32 * kc), full_bar, pol_a);
        }
        const int boff = panels * ps;
        for (int n = lane; n < q.nw; n += 32) {
          const float* src = p.B + q.col + q.k0 + (long long)(q.n0 + n) * p.K;
          bulk_g2s(smem_addr(st + boff + b_row_offset(n, q.tn)), src, uint32_t(4 * kc), full_bar,
                   pol_b);
        }
        q.filled |= 1u << q.s;
        q.lastpar = (q.lastpar & ~(1u << q.s)) | (q.ph << q.s);
      }
      if (++q.s == D) {
        q.s = 0;
        q.ph ^= 1u;
      }
      if (!cursor_advance<CHECK>(p, q)) live &= ~(1u << j);
    }
    if (progressed) {
      t_stall = clock64();
    } else {
      int stop = 0;
      if (lane == 0) {
        if (*abort_flag) {
          stop = 1;
        } else if (clock64() - t_stall > p.wait_limit) {
          record_status(p.status, VBSR_TIMEOUT, int(blockIdx.x));
          *abort_flag = 1;
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) break;
      __nanosleep(32);
    }
  }
  __syncwarp();
  // After an abort, wait (bounded) for the last fill of every slot so that no bulk copy is still
  // writing this CTA's shared memory when it exits.
  if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
    for (int j = 0; j < nt; ++j) {
      for (int s = 0; s < D; ++s) {
        if (!(cur[j].filled & (1u << s))) continue;
        const uint32_t bar = full_base + 8u * (j * kMaxStages + s);
        const uint32_t par = (cur[j].lastpar >> s) & 1u;
        const long long t0 = clock64();
        bool done = false;
        while (!(done = mbar_try(bar, par)) && clock64() - t0 < p.wait_limit) {
        }
        (void)done;
      }
    }
  }
}

// ---- kernel --------------------------------------------------------------------------------------

template <int RHS, bool CHECK>
__global__ void __launch_bounds__(kThreads, 1) spmm_kernel(const __grid_constant__ KernelParams p) {
  extern __shared__ __align__(128) float stages[];
  __shared__ __align__(8) uint64_t bars[2][kConsumerWarps][kMaxStages];
  __shared__ int abort_flag;
  const Task task = p.tasks[blockIdx.x];
  const int tw = task.team_warps;
  const int nt = kConsumerWarps / tw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full_base = smem_addr(&bars[0][0][0]);
  const uint32_t empty_base = smem_addr(&bars[1][0][0]);
  if (threadIdx.x == 0) {
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

  if (warp == kConsumerWarps) {
    producer<CHECK>(p, task, stages, full_base, empty_base, lane, abort_v);
  } else {
    const int team = warp / tw;
    const int tt = (warp % tw) * 32 + lane;
    const uint32_t full0 = full_base + 8u * (team * kMaxStages);
    const uint32_t empty0 = empty_base + 8u * (team * kMaxStages);
    const float* my_stages = stages + team * task.stages * task.stage_floats;
    int s = 0;
    uint32_t ph = 0;
    for (int it = task.team_off[team]; it < task.team_off[team + 1]; ++it) {
      const Item item = p.items[it];
      if (CHECK && !item_in_bounds(p, item)) {
        if (tt == 0) record_status(p.status, VBSR_BOUNDS_VIOLATION, it);
        continue;
      }
      bool ok = true;
      switch (item.h) {
#define VBSR_CASE_H(HH)                                                                       \
  case HH:                                                                                    \
    ok = consume_h<RHS, HH>(p, item, my_stages, task.stage_floats, task.stages, full0, empty0, \
                            s, ph, tt, lane, abort_v);                                        \
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
        default:
          break;
      }
      if (!ok) break;
    }
  }
  __syncthreads();
}

}  // namespace vbsr_b200
