// vbsr_tiles.h — tile geometry shared by the host planner and the sm_100a kernels.
//
// One work item is one block row (or one RHS-column half of a heavy block row): an h x nw tile of C,
// h in {8,...,64}, nw in {8,16,32,64}. A "team" of 1, 2 or 4 warps owns one item at a time; each
// thread of the team keeps a TM x TN register tile of C (TM consecutive rows; TN RHS columns
// strided by the number of column groups).
//
// Device value format. Every h x w block keeps its reference position and size in the value array
// (value_off is unchanged), but inside the block the values are re-laid-out for the kernels: the
// block is cut into k-chunks of 32 block columns (the last one may be narrower, kc = 8..32), each
// chunk is one contiguous run of h*kc floats, and inside a chunk the rows form h/8 panels of 8
// rows, panel p holding its 8 x kc values column-major in 16-byte units whose index is XOR-ed
// with f(p) = ((p&3)<<1) | ((p>>2)&1). One TMA bulk copy moves a whole chunk into shared memory,
// and the XOR makes the consumers' 16-byte reads of different panels at the same column fall into
// different shared-memory bank groups (for both 8-row and 4-row thread tiles).
//
// Pipeline stage: consecutive k-chunks of one item, packed up to `cols` (32 or 64) block columns.
// A chunk starting at stage column c0 keeps its stored layout at offset h*c0 floats; the B part
// starts at h*cols floats and holds one box per 8 stage columns (box c0/8 + g at (c0/8+g)*nw*8),
// each box nw rows of 8 consecutive floats of one RHS column (2-D tensor TMA, no swizzle).
#pragma once

#if defined(__CUDACC__)
#define VBSR_HD __host__ __device__ constexpr
#else
#define VBSR_HD constexpr
#endif

namespace vbsr_b200 {

constexpr int kConsumerWarps = 8;                 // warps per CTA (all compute; team leaders
constexpr int kThreads = 32 * kConsumerWarps;     // also issue their team's TMA copies)
constexpr int kChunk = 32;                        // block columns per device k-chunk
constexpr int kMaxStageCols = 64;                 // block columns per pipeline stage (max)
constexpr int kMaxStages = 4;

struct TileCfg {
  int tm, tn;    // register tile per thread
  int threads;   // active threads in the team = (h/tm) * (nw/tn)
  int warps;     // team size in warps
};

VBSR_HD TileCfg tile_cfg(int h, int nw) {
  // First candidate that keeps at least 24 threads busy; ordered by decreasing register tile so
  // that large tiles (fewest shared-memory loads per FMA) win whenever the output is big enough.
  const int cand_tm[6] = {8, 4, 4, 4, 2, 2};
  const int cand_tn[6] = {4, 4, 2, 1, 1, 1};
  TileCfg c{2, 1, 0, 1};
  for (int i = 0; i < 6; ++i) {
    const int t = (h / cand_tm[i]) * (nw / cand_tn[i]);
    c.tm = cand_tm[i];
    c.tn = cand_tn[i];
    c.threads = t;
    if (t >= 24) break;
  }
  c.warps = (c.threads + 31) / 32;
  return c;
}

// 16-byte-unit XOR of panel p (see the format description above).
VBSR_HD int panel_xor(int p) { return ((p & 3) << 1) | ((p >> 2) & 1); }

// Position of element (r, k) of an h x w block inside the block's device storage.
VBSR_HD int blk_pos(int h, int w, int r, int k) {
  const int k0 = k & ~31;
  const int kc = (w - k0) < 32 ? (w - k0) : 32;
  const int p = r >> 3;
  const int q = ((k - k0) << 1) | ((r >> 2) & 1);
  return h * k0 + p * 8 * kc + ((q ^ panel_xor(p)) << 2) + (r & 3);
}

// Floats of one stage of `cols` block columns for an (h, nw) item, rounded to 1 KB.
VBSR_HD int stage_floats(int h, int nw, int cols) { return ((h + nw) * cols + 255) / 256 * 256; }

// Offset (floats) of the B boxes inside a stage of `cols` columns.
VBSR_HD int stage_b_offset(int h, int cols) { return h * cols; }

}  // namespace vbsr_b200
