// vbsr_tiles.h — tile geometry shared by the host planner and the sm_100a kernels.
//
// One work item is one block row (or one RHS-column half of a heavy block row): an h x nw tile
// of C, h in {8,...,64}, nw in {8,16,32,64}. A "team" of 1, 2 or 4 warps owns one item at a time;
// each thread of the team keeps a TM x TN register tile of C (TM rows, TN RHS columns).
//
// The item's A and B operands are streamed through a shared-memory ring, one k-chunk of at most
// 32 block columns per stage:
//   A part: h/8 row panels, each 8 rows x kc columns column-major (8*kc floats, exactly the bytes
//           of that panel's columns [k0, k0+kc) in the device value format), placed at a panel
//           stride of 256 + pad floats so that lanes reading different panels at the same k hit
//           different 16-byte bank groups;
//   B part: nw rows (one per RHS column n), row n holding B[col_off+k0 .. +kc, n0+n], placed at
//           36 floats per row plus 4 floats after every TN rows, for the same reason.
#pragma once

#if defined(__CUDACC__)
#define VBSR_HD __host__ __device__ constexpr
#else
#define VBSR_HD constexpr
#endif

namespace vbsr_b200 {

constexpr int kConsumerWarps = 8;                 // compute warps per CTA
constexpr int kThreads = 32 * (kConsumerWarps + 1); // + one producer warp
constexpr int kChunk = 32;                        // block columns per pipeline stage
constexpr int kMaxStages = 4;
constexpr int kBRow = 36;                         // floats per staged B row (32 + 4 pad)

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

// Panel stride (floats) of the staged A chunk for a thread tile of TM rows.
VBSR_HD int a_panel_stride(int tm) { return 256 + (tm == 8 ? 4 : (tm == 4 ? 8 : 16)); }

// Offset (floats) of staged B row n for a thread tile of TN columns.
VBSR_HD int b_row_offset(int n, int tn) { return n * kBRow + (tn > 1 ? (n / tn) * 4 : 0); }

// Floats of one stage for an (h, nw) item: A panels followed by B rows, rounded to 32 floats.
VBSR_HD int stage_floats(int h, int nw) {
  const TileCfg c = tile_cfg(h, nw);
  const int a = (h / 8) * a_panel_stride(c.tm);
  const int b = b_row_offset(nw, c.tn);
  return ((a + b) + 31) / 32 * 32;
}

// Offset (floats) of the B rows inside a stage.
VBSR_HD int stage_b_offset(int h, int tm) { return (h / 8) * a_panel_stride(tm); }

}  // namespace vbsr_b200
