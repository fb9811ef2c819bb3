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
// The plan compiles the matrix into one instruction stream per team: a sequence of 64-bit entries,
// an item header followed by that item's k-chunks (one chunk = at most kChunk block columns of one
// block), then the next header, and so on. Producer and consumers of a team walk the same stream.
//
// Header (bit 63 = 1): an h x nw tile of C starting at scalar row c_row, RHS columns [n0, n0+nw)
//   bits  0..30 c_row       bits 31..33 h/8 - 1      bits 34..36 n0/8     bits 37..38 log2(nw/8)
// Chunk  (bit 63 = 0): block columns [k0, k0+kc) of one block of that item (one contiguous k-chunk
// of the device value format, kc <= 32). Consecutive chunks of an item are packed into one
// pipeline stage of up to Task::stage_cols columns; bit 62 marks the last chunk of a stage.
//   bits  0..27 val/64  (value offset of the block; blocks start at multiples of 64 floats)
//   bits 28..55 (col + k0)/8   (first scalar column of the chunk in B)
//   bits 56..58 w/8 - 1        bit 59 k0/32     bits 60..61 kc/8 - 1     bit 62 last chunk of stage
namespace entry {
constexpr uint64_t kHeader = 1ull << 63;
constexpr uint64_t kLastOfStage = 1ull << 62;
inline uint64_t header(int64_t c_row, int h, int n0, int nw) {
  int lg = 0;
  while ((8 << lg) < nw) ++lg;
  return kHeader | uint64_t(c_row) | (uint64_t(h / 8 - 1) << 31) | (uint64_t(n0 / 8) << 34) |
         (uint64_t(lg) << 37);
}
inline uint64_t chunk(int64_t val, int64_t col, int w, int k0, int kc, bool last) {
  return uint64_t(val / 64) | (uint64_t((col + k0) / 8) << 28) | (uint64_t(w / 8 - 1) << 56) |
         (uint64_t(k0 / 32) << 59) | (uint64_t(kc / 8 - 1) << 60) | (last ? kLastOfStage : 0);
}
constexpr int64_t kMaxVal = (int64_t(1) << 28) * 64;  // value offsets must stay below this
constexpr int64_t kMaxCol = (int64_t(1) << 28) * 8;
}  // namespace entry

// One CTA task: kConsumerWarps / team_warps teams; team t walks stream entries
// [team_off[t], team_off[t+1]).
struct alignas(16) Task {
  int team_off[9];
  int team_warps;     // 1, 2 or 4
  int stages;         // ring depth per team
  int stage_floats;   // floats per stage
  int stage_cols;     // block columns one stage holds (32 or 64)
  int pad[3];
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
