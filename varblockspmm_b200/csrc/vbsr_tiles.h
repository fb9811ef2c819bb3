// vbsr_tiles.h — tile geometry shared by the host planner and the sm_100a kernels.
//
// One work item is one block row (or one RHS-column half of a heavy block row): an h x nw tile of
// C, h in {8,...,64}, nw in {8,16,32,64}.
//
// Device value format. Every h x w block keeps its reference position and size in the value array
// (value_off is unchanged), but inside the block the values are re-laid-out for the tensor-core
// kernel: the block is cut into k-chunks of 32 block columns (the last one may be narrower,
// kc = 8..32), each chunk is one contiguous run of h*kc floats, and a chunk is a sequence of kc/8
// groups of 8 columns. A group holds its h rows one after another, 8 floats (32 bytes) per row,
// i.e. the K-major operand tile of one tcgen05.mma (K = 8 tf32), with the 32-byte swizzle of the
// MMA's shared-memory layout applied in advance: the two 16-byte halves of row r are exchanged
// when bit 2 of r is set. One TMA bulk copy then lands a whole chunk in shared memory exactly as
// the MMA reads it.
#pragma once

#if defined(__CUDACC__)
#define VBSR_HD __host__ __device__ constexpr
#else
#define VBSR_HD constexpr
#endif

namespace vbsr_b200 {

constexpr int kChunk = 32;                        // block columns per device k-chunk
constexpr int kMaxStages = 12;                    // pipeline depth limit per CTA

// Position of element (r, k) of an h x w block inside the block's device storage.
VBSR_HD int blk_pos(int h, int w, int r, int k) {
  const int k0 = k & ~31;
  const int g = (k - k0) >> 3, kk = k & 7;
  const int unit = (kk >> 2) ^ ((r >> 2) & 1);
  (void)w;
  return h * k0 + g * h * 8 + r * 8 + unit * 4 + (kk & 3);
}

}  // namespace vbsr_b200
