// Host interface of the small kernels (misc.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dialb200 {

cudaError_t embed_launch(const void* table, const int32_t* tokens, int M, int vocab, int H,
                         void* out, int out_ld, int* status, cudaStream_t s, bool pdl);
cudaError_t argmax_launch(const void* logits, int ld, int V, int rows, int act, int32_t* out,
                          cudaStream_t s, bool pdl);
cudaError_t advance_launch(const int32_t* sampled, int32_t* tokens, int32_t* pos, int M,
                           cudaStream_t s, bool pdl);

}  // namespace dialb200
