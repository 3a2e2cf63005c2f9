// Host interface of the load-time kernels (layout.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <type_traits>

#include "qlinear.h"

namespace dialb200 {

enum SrcDtype : int { kSrcBf16 = 0, kSrcF16 = 1, kSrcF32 = 2 };

uint64_t synth_base(uint64_t seed, uint64_t stream);

cudaError_t quantize_rows(const void* w, int src_dtype, int N, int K, int8_t* q, float* scale,
                          cudaStream_t s);
cudaError_t tile_codes(const uint8_t* src, int64_t src_ld_bytes, const DevQLinear& w, uint8_t* dst,
                       cudaStream_t s);
cudaError_t tile_nvfp4_scales(const uint8_t* sc, int64_t sc_ld, const DevQLinear& w, uint8_t* dst,
                              cudaStream_t s);
cudaError_t tile_row_scales(const float* scale, const DevQLinear& w, float* dst, cudaStream_t s);
cudaError_t synth_table_fill(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream,
                             int64_t offset, const uint16_t* table_dev, cudaStream_t s);
cudaError_t synth_tokens(int32_t* out, int64_t n, uint64_t seed, uint32_t vocab, cudaStream_t s);
cudaError_t fill_u16(uint16_t* out, int64_t n, uint16_t v, cudaStream_t s);

// Synthetic-weight quantizers on the device (bf16 [N][K] in, the rules of
// the CPU oracle's quantize_fp8_block128 / quantize_nvfp4):
//  * FP8 e4m3 codes [N][K] + f32 scales [ceil(N/128)][ld] of blockmax/448;
//  * NVFP4: e2m1 pairs [n/2] + e4m3 group scales [n/16]; the f32 global scale
//    amax/6/448 is derived from *amax_bits (written here, read back by the host).
cudaError_t quantize_fp8_block128_dev(const uint16_t* w_bf16, int N, int K, uint8_t* codes,
                                      float* scales, int ld, cudaStream_t s);
cudaError_t quantize_nvfp4_dev(const uint16_t* w_bf16, int64_t n, uint8_t* packed, uint8_t* sc,
                               unsigned* amax_bits, cudaStream_t s);

}  // namespace dialb200
