// Device weight descriptor shared by the layout kernels, the decode GEMV and
// the host-side QLinear object.
//
// Quantized weights are re-laid out at load time into "mma tiles": 16 output
// rows x KCH input columns per chunk, one 16-byte piece per lane so that a
// warp reads 512 contiguous bytes per row half and every lane's bytes feed
// its own m16n8k16 A-fragment registers directly (no shared-memory transpose).
#pragma once

#include <cstdint>

namespace dialb200 {

// Weight formats (values are part of the C ABI, see include/dial_b200.h).
enum WeightFormat : int {
  kFmtW8A16Row = 0,    // int8 symmetric, one f32 scale per output row
  kFmtFp8Block128 = 1, // e4m3, one f32 scale per 128x128 block
  kFmtFp8Row = 2,      // e4m3, one f32 scale per output row (or per tensor)
  kFmtNvfp4G16 = 3,    // e2m1 pairs, e4m3 scale per 16 inputs, f32 global
  kFmtDense = 4,       // activation-dtype dense weight (lm_head)
};

// Columns covered by one chunk, and bytes per chunk.
__host__ __device__ constexpr int fmt_kch(int fmt) {
  return fmt == kFmtNvfp4G16 ? 128 : (fmt == kFmtDense ? 32 : 64);
}
__host__ __device__ constexpr int fmt_chunk_bytes(int fmt) {
  return fmt == kFmtNvfp4G16 ? 1152 : 1024;
}

struct DevQLinear {
  const uint8_t* tiles;      // [T][C][chunk_bytes]
  const float* row_scale;    // [T*16] in tile-row order (W8A16 / FP8 row), else null
  const float* blk_scale;    // [ceil(N/128)][blk_ld] (FP8 block-128), else null
  int blk_ld;                // floats per block-scale row (multiple of 4)
  float global_scale;        // NVFP4 dequant multiplier
  int fmt;
  int N;                     // logical output rows (gate+up for SwiGLU)
  int K;                     // logical input columns
  int K_pad;                 // K rounded up to the chunk width
  int T;                     // row tiles
  int C;                     // chunks per tile
  int swiglu;                // 1: tile rows 0-7 = gate rows 8t.., rows 8-15 = up rows I+8t..
};

}  // namespace dialb200
