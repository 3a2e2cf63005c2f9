// Load-time kernels: W8A16 row quantization, re-layout of quantized or dense
// weights into the decode GEMV's mma tiles, and the seeded synthetic
// generators used for benchmark weights.
#include <cstdint>

#include <cuda_fp8.h>

#include "common.cuh"
#include "layout.h"

namespace dialb200 {
namespace {

// ---------------------------------------------------------------- a1
// Row-wise symmetric int8 quantization, bit-identical to
// CudaW8A16Linear::from_linear (worker_w8a16.rs:330-341):
//   scale = max|w| / 127 (1.0 for an all-zero row), inv = 1 / scale,
//   q = clamp(round_half_away(w * inv), -127, 127).
template <typename T>
__device__ __forceinline__ float load_f(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
  else return __bfloat162float(*p);
}

template <typename T>
__global__ void quantize_rows_kernel(const T* __restrict__ w, int N, int K, int8_t* __restrict__ q,
                                     float* __restrict__ scale) {
  const int row = blockIdx.x;
  if (row >= N) return;
  const T* wr = w + static_cast<size_t>(row) * K;
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(load_f(wr + k)));
  __shared__ float red[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  m = red[0];
  const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
  const float inv = __fdiv_rn(1.f, s);
  if (threadIdx.x == 0) scale[row] = s;
  int8_t* qr = q + static_cast<size_t>(row) * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = roundf(__fmul_rn(load_f(wr + k), inv));
    v = fminf(fmaxf(v, -127.f), 127.f);
    qr[k] = static_cast<int8_t>(v);
  }
}

__device__ __forceinline__ int src_row(int t, int r, int N, int swiglu, bool& valid) {
  if (swiglu) {
    const int I = N / 2;
    const int j = 8 * t + (r & 7);
    valid = j < I;
    return r < 8 ? j : I + j;
  }
  const int n = 16 * t + r;
  valid = n < N;
  return n;
}

// One thread per 16-byte piece of a chunk.
__global__ void tile_codes_kernel(const uint8_t* __restrict__ src, int64_t src_ld_bytes, int fmt,
                                  int N, int K, int T, int C, int swiglu, uint8_t* __restrict__ dst) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(T) * C * 64;
  if (p >= total) return;
  const int piece = static_cast<int>(p & 63);
  const int64_t chunk = p >> 6;
  const int kc = static_cast<int>(chunk % C);
  const int t = static_cast<int>(chunk / C);
  const int h = piece >> 5, l = piece & 31;
  const int r = (l >> 2) + 8 * h, c = l & 3;
  bool valid;
  const int row = src_row(t, r, N, swiglu, valid);
  uint8_t out[16];
  const int kch = fmt_kch(fmt);
  const int cb = fmt_chunk_bytes(fmt);
  if (fmt == kFmtDense) {
    const int k0 = kc * kch + c * 8;  // 8 elements x 2 bytes
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      uint16_t v = 0;
      if (valid && k < K)
        v = reinterpret_cast<const uint16_t*>(src + static_cast<int64_t>(row) * src_ld_bytes)[k];
      out[2 * e] = static_cast<uint8_t>(v & 0xff);
      out[2 * e + 1] = static_cast<uint8_t>(v >> 8);
    }
  } else if (fmt == kFmtNvfp4G16) {
    const int k0 = kc * kch + c * 32;  // 32 nibbles
    for (int e = 0; e < 16; ++e) {
      const int k = k0 + 2 * e;
      uint8_t v = 0;
      if (valid && k < K) v = src[static_cast<int64_t>(row) * src_ld_bytes + k / 2];
      out[e] = v;
    }
  } else {
    const int k0 = kc * kch + c * 16;
    for (int e = 0; e < 16; ++e) {
      const int k = k0 + e;
      uint8_t v = 0;
      if (valid && k < K) v = src[static_cast<int64_t>(row) * src_ld_bytes + k];
      if (fmt == kFmtW8A16Row) {
        v ^= 0x80u;  // stored as q + 128
      } else if ((v & 0x7fu) == 0x7fu) {
        v = 0;  // e4m3 NaN codes decode to 0 (cuda_quant.rs:34-35)
      }
      out[e] = v;
    }
  }
  uint8_t* d = dst + chunk * cb + h * 512 + l * 16;
  *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(out);
}

// NVFP4 group-scale area: 128 bytes after each chunk's 1024 code bytes.
__global__ void tile_nvfp4_scales_kernel(const uint8_t* __restrict__ sc, int64_t sc_ld, int N, int K,
                                         int T, int C, int swiglu, uint8_t* __restrict__ dst) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(T) * C * 128;
  if (p >= total) return;
  const int b = static_cast<int>(p & 127);
  const int64_t chunk = p >> 7;
  const int kc = static_cast<int>(chunk % C);
  const int t = static_cast<int>(chunk / C);
  const int h = b >> 6, l = (b & 63) >> 1, j = b & 1;
  const int r = (l >> 2) + 8 * h, c = l & 3;
  bool valid;
  const int row = src_row(t, r, N, swiglu, valid);
  const int group = (kc * 128 + c * 32) / 16 + j;
  uint8_t v = 0;
  if (valid && group * 16 < K) {
    v = sc[static_cast<int64_t>(row) * sc_ld + group];
    if ((v & 0x7fu) == 0x7fu) v = 0;
  }
  dst[chunk * 1152 + 1024 + b] = v;
}

__global__ void tile_row_scales_kernel(const float* __restrict__ s, int N, int T, int swiglu,
                                       float* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * 16) return;
  bool valid;
  const int row = src_row(i >> 4, i & 15, N, swiglu, valid);
  dst[i] = valid ? s[row] : 0.f;
}

// ---------------------------------------------------------- synthetic data
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_table_kernel(uint16_t* __restrict__ out, int64_t n, uint64_t base,
                                   int64_t offset, const uint16_t* __restrict__ table) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t h = mix64(static_cast<uint64_t>(i + offset) + base);
  out[i] = table[h & 0xffffu];
}

__global__ void synth_tokens_kernel(int32_t* __restrict__ out, int64_t n, uint64_t base,
                                    uint32_t vocab) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = static_cast<int32_t>(mix64(static_cast<uint64_t>(i) + base) % vocab);
}

__global__ void fill_u16_kernel(uint16_t* out, int64_t n, uint16_t v) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = v;
}

// ------------------------------------------------- synthetic FP8 / NVFP4
// e4m3 code of v: round to nearest even, saturating at 448, +0 for zero.
__device__ __forceinline__ uint8_t to_e4m3(float v) {
  const uint8_t c = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
  return c == 0x80 ? 0 : c;
}
__device__ __forceinline__ float e4m3_value(uint8_t c) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(c), __NV_E4M3);
  return __half2float(__half(h));
}
// e2m1 code of v: the nearest of {0, .5, 1, 1.5, 2, 3, 4, 6} (|v| clamped to 6),
// ties to the smaller magnitude, sign bit 0x8 unless the code is zero.
__device__ __forceinline__ uint8_t to_e2m1(float v) {
  const float vals[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float mag = fminf(fabsf(v), 6.f);
  uint8_t best = 0;
  float bd = fabsf(mag - vals[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(mag - vals[i]);
    if (d < bd) {
      bd = d;
      best = static_cast<uint8_t>(i);
    }
  }
  return (v < 0.f && best != 0) ? static_cast<uint8_t>(best | 0x8) : best;
}

__device__ __forceinline__ float bf16_at(const uint16_t* w, int64_t i) {
  return __uint_as_float(static_cast<uint32_t>(w[i]) << 16);
}

// One CTA per 128x128 block: scale = blockmax / 448 (1 when zero), codes = e4m3(w / scale).
__global__ void fp8_block_quant_kernel(const uint16_t* __restrict__ w, int N, int K,
                                       uint8_t* __restrict__ codes, float* __restrict__ scales,
                                       int ld) {
  __shared__ float red[8];
  const int r0 = blockIdx.y * 128, c0 = blockIdx.x * 128;
  const int rows = min(128, N - r0), cols = min(128, K - c0);
  float am = 0.f;
  for (int i = threadIdx.x; i < rows * cols; i += blockDim.x)
    am = fmaxf(am, fabsf(bf16_at(w, static_cast<int64_t>(r0 + i / cols) * K + c0 + i % cols)));
  am = warp_max(am);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  am = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) am = fmaxf(am, red[i]);
  const float sc = am > 0.f ? __fdiv_rn(am, 448.f) : 1.f;
  if (threadIdx.x == 0) scales[static_cast<size_t>(blockIdx.y) * ld + blockIdx.x] = sc;
  for (int i = threadIdx.x; i < rows * cols; i += blockDim.x) {
    const int64_t idx = static_cast<int64_t>(r0 + i / cols) * K + c0 + i % cols;
    codes[idx] = to_e4m3(__fdiv_rn(bf16_at(w, idx), sc));
  }
}

__global__ void absmax_kernel(const uint16_t* __restrict__ w, int64_t n, unsigned* out) {
  float am = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    am = fmaxf(am, fabsf(bf16_at(w, i)));
  am = warp_max(am);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(am));  // non-negative floats
}

// One thread per 16-element group: e4m3 group scale of groupmax / 6 / global,
// e2m1 codes of w / (scale * global), two per byte (low nibble first).
__global__ void nvfp4_quant_kernel(const uint16_t* __restrict__ w, int64_t groups,
                                   const unsigned* __restrict__ amax_bits, uint8_t* __restrict__ packed,
                                   uint8_t* __restrict__ sc) {
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const float amax = __uint_as_float(*amax_bits);
  // amax / 6 / 448 in double, rounded once to f32 (the oracle computes it in Python floats)
  const float gs = amax > 0.f ? static_cast<float>(static_cast<double>(amax) / 6.0 / 448.0) : 1.f;
  float v[16], gm = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    v[e] = bf16_at(w, g * 16 + e);
    gm = fmaxf(gm, fabsf(v[e]));
  }
  const uint8_t code = to_e4m3(__fdiv_rn(__fdiv_rn(gm, 6.f), gs));
  sc[g] = code;
  float sdec = e4m3_value(code) * gs;
  if (sdec == 0.f) sdec = 1.f;
#pragma unroll
  for (int e = 0; e < 16; e += 2)
    packed[g * 8 + e / 2] = static_cast<uint8_t>(to_e2m1(__fdiv_rn(v[e], sdec)) |
                                                 (to_e2m1(__fdiv_rn(v[e + 1], sdec)) << 4));
}

inline unsigned blocks_for(int64_t n, int bs) { return static_cast<unsigned>((n + bs - 1) / bs); }

}  // namespace

uint64_t synth_base(uint64_t seed, uint64_t stream) {
  return (seed * 0x9E3779B97F4A7C15ull) ^ (stream * 0xD1B54A32D192ED03ull);
}

cudaError_t quantize_rows(const void* w, int src_dtype, int N, int K, int8_t* q, float* scale,
                          cudaStream_t s) {
  if (src_dtype == kSrcBf16)
    quantize_rows_kernel<<<N, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), N, K, q, scale);
  else if (src_dtype == kSrcF16)
    quantize_rows_kernel<<<N, 256, 0, s>>>(static_cast<const __half*>(w), N, K, q, scale);
  else
    quantize_rows_kernel<<<N, 256, 0, s>>>(static_cast<const float*>(w), N, K, q, scale);
  return cudaGetLastError();
}

cudaError_t tile_codes(const uint8_t* src, int64_t src_ld_bytes, const DevQLinear& w, uint8_t* dst,
                       cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(w.T) * w.C * 64;
  tile_codes_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src, src_ld_bytes, w.fmt, w.N, w.K, w.T,
                                                           w.C, w.swiglu, dst);
  return cudaGetLastError();
}

cudaError_t tile_nvfp4_scales(const uint8_t* sc, int64_t sc_ld, const DevQLinear& w, uint8_t* dst,
                              cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(w.T) * w.C * 128;
  tile_nvfp4_scales_kernel<<<blocks_for(total, 256), 256, 0, s>>>(sc, sc_ld, w.N, w.K, w.T, w.C,
                                                                  w.swiglu, dst);
  return cudaGetLastError();
}

cudaError_t tile_row_scales(const float* scale, const DevQLinear& w, float* dst, cudaStream_t s) {
  tile_row_scales_kernel<<<blocks_for(w.T * 16, 256), 256, 0, s>>>(scale, w.N, w.T, w.swiglu, dst);
  return cudaGetLastError();
}

cudaError_t synth_table_fill(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream,
                             int64_t offset, const uint16_t* table_dev, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  synth_table_kernel<<<blocks_for(n, 256), 256, 0, s>>>(out, n, synth_base(seed, stream), offset,
                                                        table_dev);
  return cudaGetLastError();
}

cudaError_t synth_tokens(int32_t* out, int64_t n, uint64_t seed, uint32_t vocab, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  synth_tokens_kernel<<<blocks_for(n, 256), 256, 0, s>>>(out, n, synth_base(seed, 0x70CE), vocab);
  return cudaGetLastError();
}

cudaError_t fill_u16(uint16_t* out, int64_t n, uint16_t v, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  fill_u16_kernel<<<blocks_for(n, 256), 256, 0, s>>>(out, n, v);
  return cudaGetLastError();
}

cudaError_t quantize_fp8_block128_dev(const uint16_t* w_bf16, int N, int K, uint8_t* codes,
                                      float* scales, int ld, cudaStream_t s) {
  const dim3 grid((K + 127) / 128, (N + 127) / 128);
  fp8_block_quant_kernel<<<grid, 256, 0, s>>>(w_bf16, N, K, codes, scales, ld);
  return cudaGetLastError();
}

cudaError_t quantize_nvfp4_dev(const uint16_t* w_bf16, int64_t n, uint8_t* packed, uint8_t* sc,
                               unsigned* amax_bits, cudaStream_t s) {
  if (n % 16) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(amax_bits, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  absmax_kernel<<<1184, 256, 0, s>>>(w_bf16, n, amax_bits);
  nvfp4_quant_kernel<<<blocks_for(n / 16, 256), 256, 0, s>>>(w_bf16, n / 16, amax_bits, packed, sc);
  return cudaGetLastError();
}

}  // namespace dialb200
