// Host interface of the prefill W8A16 GEMM on the 5th-generation tensor cores (gemm.cu).
#pragma once

#include <cstddef>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "qlinear.h"

namespace dialb200 {

struct GemmArgs {
  DevQLinear w;         // W8A16 tiles (int8 ^ 0x80) + f32 row scales
  const void* x;        // [M][x_ld] activations (bf16 or f16)
  int x_ld;
  const void* norm_w;   // RMSNorm weight [K] applied to x first, or null
  float eps;
  void* out;            // [M][out_ld]
  int out_ld;
  int M;
  __half* xh;           // scratch [M][w.K_pad]: staged f16 activations
  int* xexp;            // scratch [M]: per-row power-of-two pre-scale
  int* status;
  // Optional split-K workspace (f32): when given and a launch would leave
  // most SMs idle, K is cut into splits whose partial sums land here
  // ([split][M][N]) and a second kernel adds them in split order and applies
  // the epilogue.  Null: one pass over K.
  float* part;
  size_t part_bytes;
  int couple;  // diagnostic: weight slots also wait for the MMAs of their k-step
};

// True when the weight can take the tensor-core path: W8A16, FP8 (row or
// 128x128 block scales) or NVFP4 (e4m3 scale per 16 inputs, f32 global
// scale), 128-row blocks (N % 128 == 0, or 64 gate + 64 up rows for the
// fused gate/up layout), K <= 24576.
bool gemm_w8a16_supported(const DevQLinear& w);

// Scratch bytes for `rows` rows (xh + xexp), 256-byte aligned pieces.
size_t gemm_scratch_bytes(int rows, int k_pad);

// act: 0 = bf16, 1 = f16; epi: GemvEpilogue (store, residual, swiglu).
cudaError_t gemm_w8a16_launch(const GemmArgs& a, int act, int epi, cudaStream_t s);

}  // namespace dialb200
