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

}  // namespace dialb200
