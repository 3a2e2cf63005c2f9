// Small kernels around the layer stack: embedding gather, greedy argmax and
// the on-device step-state update of the graph-captured decode loop.
//
// Reference: Embedding::forward (qwen3_vl.rs:3302), device argmax
// (qwen3_vl.rs:138-143; candle keeps the first index among equal maxima).
#include "common.cuh"
#include "misc.h"

namespace dialb200 {
namespace {

__global__ void embed_kernel(const uint16_t* __restrict__ table, const int32_t* __restrict__ tokens,
                             int vocab, int H, uint16_t* __restrict__ out, int out_ld, int* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  int tok = tokens[m];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) set_status(status, kStatusBadArgs);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(tok) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * out_ld);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

template <typename Act>
__global__ void argmax_kernel(const Act* __restrict__ logits, int ld, int V,
                              int32_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const Act* row = logits + static_cast<size_t>(blockIdx.x) * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = ActTraits<Act>::to_f(row[i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

// next step: tokens <- sampled (when a stage samples), pos += 1
__global__ void advance_kernel(const int32_t* __restrict__ sampled, int32_t* __restrict__ tokens,
                               int32_t* __restrict__ pos, int M) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = threadIdx.x;
  if (i < M) {
    if (sampled) tokens[i] = sampled[i];
    pos[i] += 1;
  }
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t s, bool pdl,
                           cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

cudaError_t embed_launch(const void* table, const int32_t* tokens, int M, int vocab, int H,
                         void* out, int out_ld, int* status, cudaStream_t s, bool pdl) {
  if (H % 8) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(M), dim3(256), s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, embed_kernel, static_cast<const uint16_t*>(table), tokens, vocab,
                            H, static_cast<uint16_t*>(out), out_ld, status);
}

cudaError_t argmax_launch(const void* logits, int ld, int V, int rows, int act, int32_t* out,
                          cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(1024), s, pdl, attr);
  if (act == 0)
    return cudaLaunchKernelEx(&cfg, argmax_kernel<__nv_bfloat16>,
                              static_cast<const __nv_bfloat16*>(logits), ld, V, out);
  return cudaLaunchKernelEx(&cfg, argmax_kernel<__half>, static_cast<const __half*>(logits), ld, V,
                            out);
}

cudaError_t advance_launch(const int32_t* sampled, int32_t* tokens, int32_t* pos, int M,
                           cudaStream_t s, bool pdl) {
  if (M > 1024) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(1024), s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, advance_kernel, sampled, tokens, pos, M);
}

}  // namespace dialb200
