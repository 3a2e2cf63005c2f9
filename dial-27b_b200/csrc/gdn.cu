// Gated-DeltaNet token mixer of the Qwen3.8 hybrid decoder
// (dial-core/src/models/qwen3_8/text.rs:233-481), between its input
// projections (ordinary quantized linears: in_proj_qkv, in_proj_z, in_proj_b,
// in_proj_a) and out_proj, for one session.
//
//  1. gdn_conv_kernel: the causal depthwise conv1d over time (kernel K) of
//     every channel of mixed = q | k | v, continued from the carried conv
//     state (or zeros at a sequence start), then SiLU; the last K-1 inputs
//     become the new state (GatedDeltaNet::causal_conv, text.rs:301-337).
//  2. gdn_scan_kernel: one CTA per value head.  Its 128 x 128 f32 recurrent
//     state lives in registers (thread (ib, j) holds rows 32*ib .. 32*ib+31 of
//     column j) for the whole call.  Per token: q and k of the head's key head
//     L2-normalised (q also / sqrt(dk)), beta = sigmoid(b), g = -softplus(a +
//     dt_bias) * exp(A_log), state *= exp(g), pred = k . state, state += k (x)
//     (v - pred) * beta, out = q . state (text.rs:339-459); the output is
//     rounded to the activation dtype and goes through the gated RMSNorm
//     (x / rms * w * silu(z), text.rs:240-250, 460-466).
//
// Rounding points (candle-owned ops, not pinned by a reference test): conv
// sums in f32 and rounds once; SiLU / sigmoid round each step to the
// activation dtype; the recurrence is f32 (text.rs:459 states it); the gated
// norm is f32 with one final rounding.  The tokens of a call are scanned in
// order by each CTA (the recurrence is sequential); heads run in parallel.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/dial_b200.h"
#include "common.cuh"

namespace dialb200 {
namespace {

constexpr int kGdnDim = 128;   // key and value head dims this kernel handles
constexpr int kGdnThreads = 512;

template <typename Act>
__device__ __forceinline__ float silu_act(float v) {
  using AT = ActTraits<Act>;
  const float e = AT::round(expf(-v));
  return AT::round(__fdiv_rn(v, AT::round(1.f + e)));
}

template <typename Act>
__device__ __forceinline__ float sigmoid_act(float v) {
  using AT = ActTraits<Act>;
  const float e = AT::round(expf(-v));
  return AT::round(__fdiv_rn(1.f, AT::round(1.f + e)));
}

// One thread per channel: conv_out[t][c] = silu(act(sum_j w[c][j] * in[t + j]))
// over in = state[c] (K-1 values, zeros when fresh) ++ mixed[0..S)[c].
template <typename Act>
__global__ void gdn_conv_kernel(const Act* __restrict__ mixed, const Act* __restrict__ w,
                                Act* __restrict__ state, Act* __restrict__ out, int S, int C, int K,
                                int fresh) {
  using AT = ActTraits<Act>;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float win[8];  // K <= 8: the last K-1 inputs
  float wc[8];
  for (int j = 0; j < K; ++j) wc[j] = AT::to_f(w[static_cast<size_t>(c) * K + j]);
  for (int j = 0; j < K - 1; ++j)
    win[j] = fresh ? 0.f : AT::to_f(state[static_cast<size_t>(c) * (K - 1) + j]);
  for (int t = 0; t < S; ++t) {
    const float x = AT::to_f(mixed[static_cast<size_t>(t) * C + c]);
    float acc = 0.f;
    for (int j = 0; j < K - 1; ++j) acc = fmaf(wc[j], win[j], acc);
    acc = fmaf(wc[K - 1], x, acc);
    out[static_cast<size_t>(t) * C + c] = AT::from_f(silu_act<Act>(AT::round(acc)));
    for (int j = 0; j + 1 < K - 1; ++j) win[j] = win[j + 1];
    if (K > 1) win[K - 2] = x;
  }
  for (int j = 0; j < K - 1; ++j)
    state[static_cast<size_t>(c) * (K - 1) + j] = AT::from_f(win[j]);
}

struct GdnScanArgs {
  const void* conv_out;  // [S][C] activation: q | k | v after conv + SiLU
  const void* z;         // [S][hv * dv]
  const void* b;         // [S][hv]
  const void* a;         // [S][hv]
  const float* dt_bias;  // [hv]
  const float* a_log;    // [hv]
  const float* norm_w;   // [dv]
  float* rec;            // [hv][dk][dv] recurrent state
  void* out;             // [S][hv * dv]
  int S, C, hk, hv;
  float eps;
  int fresh;
};

__device__ __forceinline__ float block_sum_128(float v, float* red, int tid) {
  // sum over threads 0..127 (4 warps); every thread of the block calls it
  v = warp_sum(v);
  if ((tid & 31) == 0 && tid < 128) red[tid >> 5] = v;
  __syncthreads();
  const float s = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();
  return s;
}

template <typename Act>
__global__ void __launch_bounds__(kGdnThreads, 1) gdn_scan_kernel(const GdnScanArgs g) {
  using AT = ActTraits<Act>;
  __shared__ float qs[kGdnDim], ks[kGdnDim], vs[kGdnDim];
  __shared__ float part[4][kGdnDim];
  __shared__ float red[8];
  __shared__ float gb[2];  // decay exp(g), beta
  const int h = blockIdx.x, tid = threadIdx.x;
  const int ib = tid >> 7, j = tid & 127;
  const int kh = h / (g.hv / g.hk);
  float s[32];
  float* rec = g.rec + static_cast<size_t>(h) * kGdnDim * kGdnDim;
#pragma unroll
  for (int r = 0; r < 32; ++r)
    s[r] = g.fresh ? 0.f : rec[static_cast<size_t>(ib * 32 + r) * kGdnDim + j];
  const float qscale = rsqrtf(static_cast<float>(kGdnDim));
  const Act* cv = reinterpret_cast<const Act*>(g.conv_out);
  const int ksz = g.hk * kGdnDim;
  for (int t = 0; t < g.S; ++t) {
    const Act* row = cv + static_cast<size_t>(t) * g.C;
    // q (threads 0..127) and k (128..255) of the key head, v (256..383)
    float x = 0.f;
    if (tid < 128) x = AT::to_f(row[kh * kGdnDim + j]);
    else if (tid < 256) x = AT::to_f(row[ksz + kh * kGdnDim + j]);
    else if (tid < 384) vs[j] = AT::to_f(row[2 * ksz + h * kGdnDim + j]);
    if (tid == 0) {
      const float bv = AT::to_f(reinterpret_cast<const Act*>(g.b)[static_cast<size_t>(t) * g.hv + h]);
      const float av = AT::to_f(reinterpret_cast<const Act*>(g.a)[static_cast<size_t>(t) * g.hv + h]);
      const float sp = logf(expf(av + g.dt_bias[h]) + 1.f);
      gb[0] = expf(-(sp * expf(g.a_log[h])));
      gb[1] = sigmoid_act<Act>(bv);
    }
    // l2 norms of q and k: warps 0-3 hold q, 4-7 hold k
    float ss = warp_sum(x * x);
    if ((tid & 31) == 0 && tid < 256) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 256) {
      const int base = tid < 128 ? 0 : 4;
      const float tot = (red[base] + red[base + 1]) + (red[base + 2] + red[base + 3]);
      const float nx = __fdiv_rn(x, sqrtf(tot + 1e-6f));
      if (tid < 128) qs[j] = nx * qscale;
      else ks[j] = nx;
    }
    __syncthreads();
    const float decay = gb[0], beta = gb[1];
    float pp = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      s[r] *= decay;
      pp = fmaf(s[r], ks[ib * 32 + r], pp);
    }
    part[ib][j] = pp;
    __syncthreads();
    const float pred = (part[0][j] + part[1][j]) + (part[2][j] + part[3][j]);
    const float delta = (vs[j] - pred) * beta;
    float po = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      s[r] = fmaf(ks[ib * 32 + r], delta, s[r]);
      po = fmaf(s[r], qs[ib * 32 + r], po);
    }
    __syncthreads();  // every thread has read part[] for pred
    part[ib][j] = po;
    __syncthreads();
    // gated RMSNorm of the head's output (threads 0..127 own one column each)
    float o = 0.f;
    if (tid < 128) o = AT::round((part[0][j] + part[1][j]) + (part[2][j] + part[3][j]));
    const float msum = block_sum_128(tid < 128 ? o * o : 0.f, red, tid);
    if (tid < 128) {
      const float y = __fdiv_rn(o, sqrtf(__fdiv_rn(msum, static_cast<float>(kGdnDim)) + g.eps));
      const float zv = AT::to_f(reinterpret_cast<const Act*>(g.z)[static_cast<size_t>(t) * g.hv *
                                                                  kGdnDim + h * kGdnDim + j]);
      const float sz = __fdiv_rn(zv, 1.f + expf(-zv));
      reinterpret_cast<Act*>(g.out)[static_cast<size_t>(t) * g.hv * kGdnDim + h * kGdnDim + j] =
          AT::from_f(y * g.norm_w[j] * sz);
    }
    __syncthreads();  // qs/ks/vs/part are rewritten by the next token
  }
#pragma unroll
  for (int r = 0; r < 32; ++r) rec[static_cast<size_t>(ib * 32 + r) * kGdnDim + j] = s[r];
}

int fail(char* err, size_t n, int code, const char* f, ...) {
  if (err && n) {
    va_list ap;
    va_start(ap, f);
    std::vsnprintf(err, n, f, ap);
    va_end(ap);
  }
  return code;
}

template <typename Act>
cudaError_t launch_gdn(const dial_b200_gdn_shape* sh, const void* mixed, const void* z,
                       const void* b, const void* a, const void* conv_w, const float* dt_bias,
                       const float* a_log, const float* norm_w, void* conv_state, float* rec,
                       int S, int fresh, void* scratch, void* out, cudaStream_t s) {
  const int C = 2 * sh->k_heads * kGdnDim + sh->v_heads * kGdnDim;
  gdn_conv_kernel<Act><<<(C + 127) / 128, 128, 0, s>>>(
      static_cast<const Act*>(mixed), static_cast<const Act*>(conv_w),
      static_cast<Act*>(conv_state), static_cast<Act*>(scratch), S, C, sh->conv_kernel, fresh);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GdnScanArgs g{};
  g.conv_out = scratch;
  g.z = z;
  g.b = b;
  g.a = a;
  g.dt_bias = dt_bias;
  g.a_log = a_log;
  g.norm_w = norm_w;
  g.rec = rec;
  g.out = out;
  g.S = S;
  g.C = C;
  g.hk = sh->k_heads;
  g.hv = sh->v_heads;
  g.eps = sh->eps;
  g.fresh = fresh;
  gdn_scan_kernel<Act><<<sh->v_heads, kGdnThreads, 0, s>>>(g);
  return cudaGetLastError();
}

}  // namespace
}  // namespace dialb200

using namespace dialb200;

extern "C" int64_t dial_b200_gdn_scratch_bytes(const dial_b200_gdn_shape* sh, int64_t seq_len) {
  if (!sh || seq_len < 1) return -1;
  return seq_len * (2LL * sh->k_heads * sh->k_head_dim + 1LL * sh->v_heads * sh->v_head_dim) * 2;
}

extern "C" int dial_b200_gdn_forward(const dial_b200_gdn_shape* sh, const void* mixed,
                                     const void* z, const void* b, const void* a,
                                     const void* conv_weight, const float* dt_bias,
                                     const float* a_log, const float* norm_weight,
                                     void* conv_state, float* recurrent_state, int64_t seq_len,
                                     int64_t index_pos, void* scratch, void* core_out,
                                     void* stream, char* err, size_t n) {
  if (!(sh && mixed && z && b && a && conv_weight && dt_bias && a_log && norm_weight &&
        conv_state && recurrent_state && scratch && core_out))
    return fail(err, n, DIAL_ERR_INVALID, "null pointer argument");
  if (sh->k_head_dim != kGdnDim || sh->v_head_dim != kGdnDim)
    return fail(err, n, DIAL_ERR_INVALID, "key and value head dims must be %d (got %d, %d)",
                kGdnDim, sh->k_head_dim, sh->v_head_dim);
  if (sh->k_heads < 1 || sh->v_heads < 1 || sh->v_heads % sh->k_heads != 0)
    return fail(err, n, DIAL_ERR_INVALID,
                "linear_num_value_heads %d is not a multiple of linear_num_key_heads %d",
                sh->v_heads, sh->k_heads);
  if (sh->conv_kernel < 1 || sh->conv_kernel > 8)
    return fail(err, n, DIAL_ERR_INVALID, "conv kernel %d outside [1, 8]", sh->conv_kernel);
  if (sh->act != DIAL_ACT_BF16 && sh->act != DIAL_ACT_F16)
    return fail(err, n, DIAL_ERR_INVALID, "act must be BF16 or F16");
  if (seq_len < 1 || seq_len > (1 << 20) || index_pos < 0)
    return fail(err, n, DIAL_ERR_INVALID, "seq_len %lld / index_pos %lld out of range",
                (long long)seq_len, (long long)index_pos);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fresh = index_pos == 0 ? 1 : 0;
  const cudaError_t e =
      sh->act == DIAL_ACT_BF16
          ? launch_gdn<__nv_bfloat16>(sh, mixed, z, b, a, conv_weight, dt_bias, a_log, norm_weight,
                                      conv_state, recurrent_state, static_cast<int>(seq_len),
                                      fresh, scratch, core_out, s)
          : launch_gdn<__half>(sh, mixed, z, b, a, conv_weight, dt_bias, a_log, norm_weight,
                               conv_state, recurrent_state, static_cast<int>(seq_len), fresh,
                               scratch, core_out, s);
  if (e != cudaSuccess)
    return fail(err, n, DIAL_ERR_CUDA, "gated-deltanet launch failed: %s", cudaGetErrorString(e));
  return DIAL_OK;
}
