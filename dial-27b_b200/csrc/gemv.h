// Host interface of the decode GEMV (gemv.cu).
#pragma once

#include <algorithm>
#include <cuda_runtime.h>
#include <type_traits>

#include "qlinear.h"

namespace dialb200 {

enum GemvEpilogue : int {
  kEpiStore = 0,     // out = act(acc * scale)
  kEpiResidual = 1,  // out = act(out + act(acc * scale))      (in-place residual)
  kEpiSwiglu = 2,    // out[:, j] = act(silu(gate_j) * up_j)   (fused gate/up rows)
  kEpiArgmax = 3,    // store (when out != null) + greedy argmax per row -> amax_tok
};

struct GemvArgs {
  DevQLinear w;
  const void* x;       // [M][x_ld] activations (bf16 or f16)
  int x_ld;
  const void* norm_w;  // RMSNorm weight [K] when the prologue normalizes x
  float eps;
  void* out;           // [M][out_ld]
  int out_ld;
  int M;
  int* status;         // device status word (first error code wins)
  // kEpiArgmax: per-row packed (value, index) keys and a CTA arrival counter,
  // both zero on entry and left zero on exit; amax_tok [M] receives the ids.
  unsigned long long* amax_key;
  int* amax_count;
  int32_t* amax_tok;
  unsigned long long* trace;  // opt-in timeline records (common.cuh), null = off
  int trace_tag;
};

struct GemvTuning {
  int slots = 0;   // ring stages (0 = as many as fit)
  int grid = 0;    // CTAs (0 = one per SM)
  bool pdl = true; // programmatic dependent launch
  int nvfp4_stage = 0;  // NVFP4 GEMV chunks per ring stage (0: chosen per linear)
  int gemm_min_rows = 16;    // rows from which linears take the tcgen05 GEMM (0 = never)
  int attn_min_split = 0;    // decode attention: context tokens per split at least (0 = 16)
  bool attn_tc = true;       // prefill attention on the tensor cores when supported
  bool attn_ring = false;    // decode attention pages through a shared-memory ring (opt-in)
  int attn_tok_split = 1;  // decode attention: warps split each page's tokens (AttnDecodeArgs)
  bool attn_mma = true;     // decode attention for many rows on the tensor cores
  int attn_mma_min_split = 256;  // ... its context tokens per split at least (0: attn_min_split)
  int attn_mma_ring = 2;       // ... its page slots per warp (2 or 3)
};

// act: 0 = bf16, 1 = f16.  Launches ceil(M/8) kernels on `stream`.
cudaError_t gemv_launch(const GemvArgs& args, int act, int epi, bool norm, cudaStream_t stream,
                        const GemvTuning& tune);
int gemv_smem_bytes(const DevQLinear& w, int M, int grid, int slots);

}  // namespace dialb200
