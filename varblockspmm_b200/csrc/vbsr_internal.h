// vbsr_internal.h — types shared by the host code (vbsr_host.cpp) and the CUDA code
// (vbsr_device.cu). Not part of the public ABI.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "vbsr_b200.h"

namespace vbsr_b200 {

// ---- per-thread last error ---------------------------------------------------------------------
vbsr_status set_error(vbsr_status s, const std::string& msg);
void clear_error();

// ---- work schedule ---------------------------------------------------------------------------
// The plan compiles the matrix into, per CTA, a list of work items (one block row each, or one row
// part of a heavy block row: an h x nw tile of C) and the list of their pipeline stages. A stage covers up to twelve consecutive
// 8-column groups of one item (as many as fit one shared-memory slot at the item's h), possibly
// from several blocks. Because a block row's blocks are contiguous in
// the value array and each block stores its groups in order (h x 8 floats each), the A values of a
// stage are one contiguous range; B is fetched per 8-column group. A block row with no blocks is an
// item without stages (its C rows are stored as zeros).
// Stage descriptor, 8 x 64 bits:
//   w0: bits  0..27 A start / 64 (offsets of blocks and groups are multiples of 64 floats)
//       bits 28..31 groups - 1 (a stage holds 1..12 groups of 8 block columns)
//       bits 32..34 h/8 - 1         bits 36..38 n0/8   bits 39..40 log2(nw/8)
//       bits 41..43 H/8 - 1: the height of the block row; H > h for a row part of a split block
//                   row (rows [r0, r0 + h) of H, A start then points at row r0 of the first group)
//   w1: the item's index in the CTA's item list
//   w2..w7: the groups' scalar columns / 8, two per word (group 2i in bits 0..27 of w[2+i],
//           group 2i+1 in bits 32..59)
struct alignas(64) StageDesc {
  uint64_t w[8];
};
static_assert(sizeof(StageDesc) == 64, "StageDesc layout");
namespace stage {
constexpr int64_t kMaxVal = (int64_t(1) << 28) * 64;  // value offsets must stay below this
constexpr int64_t kMaxCol = (int64_t(1) << 28) * 8;   // scalar columns must stay below this
inline int nw_code(int nw) {
  int lg = 0;
  while ((8 << lg) < nw) ++lg;
  return lg;
}
}  // namespace stage

// Item descriptor, 4 x 32 bits:
//   x: c_row (first scalar row of the tile in C)
//   y: bits 0..2 h/8 - 1, bits 3..5 n0/8, bits 6..7 log2(nw/8), bits 8..31 the item's number of
//      8-column groups (its stages hold stage_groups(h, rhs) groups each, the last one the rest)
//   z: index of the item's first stage in the CTA's stage list
//   w: number of stages of the item (0 for a block row without blocks)
struct alignas(16) ItemDesc {
  uint32_t c_row, shape, k0, n;
};
static_assert(sizeof(ItemDesc) == 16, "ItemDesc layout");

// A block row computed on the CUDA cores (short rows, h <= 16, RHS <= 32; see cc_rows in
// vbsr_tc.cuh): its C rows, height, device-format A start and block range.
struct alignas(16) CcItem {
  uint32_t c_row, h;
  uint32_t b0, b1;  // blocks [b0, b1) of the matrix (their descriptors in d_blk_desc)
  uint64_t a_off;   // first A value of the row in the device format (blocks: value_off)
  uint64_t pad;
};
static_assert(sizeof(CcItem) == 32, "CcItem layout");

// One CTA task: items [item_off, item_end) and stages [stage_off, stage_end) of the plan's lists.
struct alignas(16) Task {
  int item_off, item_end, stage_off, stage_end;
  int team_warps;     // warps per CTA
  int stages;         // ring depth (slots)
  int stage_floats;   // floats per slot
  int stage_cols;     // block columns one stage holds at most (any h)
  int pad[8];
};
static_assert(sizeof(Task) == 64, "Task layout");

// Per-block descriptor: col_scalar_off | (w/8 - 1); col_scalar_off is a multiple of 8 so its low
// three bits are free.
inline uint32_t pack_block(int64_t col_off, int w) { return uint32_t(col_off) | uint32_t(w / 8 - 1); }

// Device status word layout.
enum { kStatusCode = 0, kStatusInfo = 1, kStatusWords = 4 };

// ---- owning matrix -------------------------------------------------------------------------
struct MatrixData {
  int device = 0;
  int32_t block_rows = 0, block_cols = 0, row_begin = 0, row_end = 0;
  int64_t nnzb = 0, M = 0, K = 0, nvalues = 0, device_bytes = 0;
  // host copies of the row structure (the planner reads these)
  std::vector<int32_t> h_row_ptr, h_row_size;
  std::vector<int64_t> h_row_off, h_val_off_row, h_sum_w;
  std::vector<uint32_t> h_blk_desc;  // per block: col_scalar_off | (w/8 - 1)
  // device arrays in the reference layout (device_view) ...
  int32_t *d_row_ptr = nullptr, *d_block_col = nullptr, *d_row_size = nullptr,
          *d_col_size = nullptr;
  int64_t *d_row_off = nullptr, *d_col_off = nullptr, *d_value_off = nullptr;
  float* d_values = nullptr;  // re-laid-out value array
  // ... and the kernels' descriptors
  uint32_t* d_blk_desc = nullptr;
};

}  // namespace vbsr_b200

struct vbsr_matrix {
  vbsr_b200::MatrixData d;
};

struct vbsr_host_matrix {
  int32_t block_rows = 0, block_cols = 0;
  std::vector<int32_t> row_ptr, block_col, row_size, col_size;
  std::vector<int64_t> row_scalar_off, col_scalar_off, value_off;
  std::vector<float> values;
};
