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

// ---- work schedule -----------------------------------------------------------------------------
// One work item: an h x nw tile of C (block row, RHS columns [n0, n0+nw)).
struct alignas(16) Item {
  long long val_off;  // offset (floats) of the row's first block in the device value array
  int blk_begin;      // first block (index into the block descriptor array)
  int nblk;           // blocks in the row
  int c_row;          // first scalar row of the tile in C (matrix-local)
  int h;              // block-row height
  int n0;             // first RHS column
  int nw;             // RHS columns
};
static_assert(sizeof(Item) == 32, "Item layout");

// One CTA task: up to kConsumerWarps / team_warps teams, team t owning items
// [team_off[t], team_off[t+1]).
struct alignas(16) Task {
  int team_off[9];
  int team_warps;     // 1, 2 or 4
  int stages;         // ring depth per team
  int stage_floats;   // floats per stage
};
static_assert(sizeof(Task) == 48, "Task layout");

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
