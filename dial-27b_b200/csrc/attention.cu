// GQA attention over the paged per-session KV cache.
//
// Reference path (lisa301/DIAL-27B, dial-core/src/models/qwen3_vl/text.rs):
//   q/k RMSNorm per head ........ 1466-1467, 1513-1514
//   RoPE (half-split) ........... 1143-1153 with tables llama3/cache.rs:37-67
//   KV append ................... llama3/cache.rs:117-160 (prefill), 169-237 (decode)
//   grouped decode attention .... 1258-1281
//   grouped prefill attention ... 1283-1327 (causal mask cache.rs:102-113)
//
// The decode kernel fuses q/k-norm, RoPE and the KV append of the new token
// with a split-KV flash pass: CTA (kv_head, split, row) runs one warp per
// query head of the group, so the 4 (or 5) query heads share every K/V load.
// Scores follow the reference's rounding: act(act(q.k) * act(1/sqrt(d))),
// then an f32 online softmax.  With more than one split, partials go to a
// scratch buffer and the last CTA of each (row, kv head) combines them
// (arrival counter, self-resetting to zero).
#include <cmath>

#include "attention.h"
#include "common.cuh"

namespace dialb200 {
namespace {

constexpr int kD = 128;  // head_dim supported by these kernels

template <typename Act>
__device__ __forceinline__ void load4(const Act* p, float (&v)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const Act* h = reinterpret_cast<const Act*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = ActTraits<Act>::to_f(h[e]);
}

template <typename Act>
__device__ __forceinline__ void store4(Act* p, const float (&v)[4]) {
  uint2 raw;
  Act* h = reinterpret_cast<Act*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = ActTraits<Act>::from_f(v[e]);
  *reinterpret_cast<uint2*>(p) = raw;
}

// Per-head RMSNorm + RoPE of one 128-wide head held 4 dims per lane
// (lane l: dims 4l..4l+3); values are activation-rounded floats.
template <typename Act, bool NORM, bool ROPE>
__device__ __forceinline__ void norm_rope(float (&x)[4], const Act* norm_w, float eps,
                                          const Act* cos_row, const Act* sin_row, int lane) {
  using AT = ActTraits<Act>;
  if constexpr (NORM) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = fmaf(x[e], x[e], ss);
    ss = warp_sum(ss);
    const float m = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(kD)) + eps));
    float w[4];
    load4(norm_w + lane * 4, w);
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = AT::round(AT::round(__fdiv_rn(x[e], m)) * w[e]);
  }
  if constexpr (ROPE) {
    float partner[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const int i0 = (lane & 15) * 4;
    float c[4], s[4];
    load4(cos_row + i0, c);
    load4(sin_row + i0, s);
    const bool first = lane < 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x1 = first ? x[e] : partner[e];
      const float x2 = first ? partner[e] : x[e];
      x[e] = first ? AT::round(AT::round(x1 * c[e]) - AT::round(x2 * s[e]))
                   : AT::round(AT::round(x1 * s[e]) + AT::round(x2 * c[e]));
    }
  }
}

__device__ __forceinline__ int lane_of_token(int t) {
  return (((t >> 3) & 1) << 4) | (((t >> 2) & 1) << 3) | (((t >> 1) & 1) << 2) | ((t & 1) << 1);
}

template <typename Act, int NREP>
__global__ void __launch_bounds__(NREP * 32) attn_decode_kernel(const AttnDecodeArgs a) {
  using AT = ActTraits<Act>;
  const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int QH = a.sh.q_heads, KVH = a.sh.kv_heads;
  const int h = kvh * NREP + warp;

  pdl_launch_dependents();
  pdl_wait();

  __shared__ float kn_s[kD], vn_s[kD];
  __shared__ int last_flag;

  const int sid = a.sid[m];
  int pos = a.pos[m];
  const bool bad = pos < 0 || pos >= a.sh.max_pos || pos / kPageTokens >= a.sh.max_blocks;
  if (bad) {
    set_status(a.status, kStatusBadArgs);
    pos = 0;
  }
  const int ctx = pos + 1;
  const int32_t* bt = a.block_table + static_cast<size_t>(sid) * a.sh.max_blocks;
  const int span = ((ctx + a.splits - 1) / a.splits + kPageTokens - 1) / kPageTokens * kPageTokens;
  const int tok0 = split * span;
  const int tok1 = min(ctx, tok0 + span);
  const bool owner = tok0 <= pos && pos < tok1;

  const Act* qkv = reinterpret_cast<const Act*>(a.qkv) + static_cast<size_t>(m) * a.qkv_ld;
  const Act* cos_row = reinterpret_cast<const Act*>(a.cos) + static_cast<size_t>(pos) * (kD / 2);
  const Act* sin_row = reinterpret_cast<const Act*>(a.sin) + static_cast<size_t>(pos) * (kD / 2);
  Act* kpool = reinterpret_cast<Act*>(a.kv.k);
  Act* vpool = reinterpret_cast<Act*>(a.kv.v);

  float q[4];
  load4(qkv + h * kD + lane * 4, q);
  norm_rope<Act, true, true>(q, reinterpret_cast<const Act*>(a.q_norm_w), a.sh.eps, cos_row,
                             sin_row, lane);

  if (owner && warp == 0 && !bad) {
    float k[4], v[4];
    load4(qkv + (QH + kvh) * kD + lane * 4, k);
    load4(qkv + (QH + KVH + kvh) * kD + lane * 4, v);
    norm_rope<Act, true, true>(k, reinterpret_cast<const Act*>(a.k_norm_w), a.sh.eps, cos_row,
                               sin_row, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      kn_s[lane * 4 + e] = k[e];
      vn_s[lane * 4 + e] = v[e];
    }
    const int blk = bt[pos / kPageTokens];
    const size_t off =
        ((static_cast<size_t>(blk) * KVH + kvh) * kPageTokens + (pos % kPageTokens)) * kD + lane * 4;
    store4(kpool + off, k);
    store4(vpool + off, v);
  }
  __syncthreads();

  const float scale = AT::round(1.0f / sqrtf(static_cast<float>(kD)));
  float mrun = -INFINITY, lrun = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int my_tok = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                     ((lane >> 1) & 1);

  for (int b0 = tok0; b0 < tok1; b0 += kPageTokens) {
    const int blk = bt[b0 / kPageTokens];
    const size_t base = (static_cast<size_t>(blk) * KVH + kvh) * kPageTokens * kD + lane * 4;
    uint2 kr[kPageTokens], vr[kPageTokens];
#pragma unroll
    for (int j = 0; j < kPageTokens; ++j) {
      kr[j] = *reinterpret_cast<const uint2*>(kpool + base + j * kD);
      vr[j] = *reinterpret_cast<const uint2*>(vpool + base + j * kD);
    }
    float v16[kPageTokens];
#pragma unroll
    for (int j = 0; j < kPageTokens; ++j) {
      const Act* kh = reinterpret_cast<const Act*>(&kr[j]);
      float d = 0.f;
      if (owner && b0 + j == pos) {
#pragma unroll
        for (int e = 0; e < 4; ++e) d = fmaf(q[e], kn_s[lane * 4 + e], d);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) d = fmaf(q[e], AT::to_f(kh[e]), d);
      }
      v16[j] = d;
    }
    // reduce-scatter: afterwards lane holds the full dot of token my_tok
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = (lane & 16) ? v16[i] : v16[i + 8];
      const float keep = (lane & 16) ? v16[i + 8] : v16[i];
      v16[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = (lane & 8) ? v16[i] : v16[i + 4];
      const float keep = (lane & 8) ? v16[i + 4] : v16[i];
      v16[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = (lane & 4) ? v16[i] : v16[i + 2];
      const float keep = (lane & 4) ? v16[i + 2] : v16[i];
      v16[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
      const float send = (lane & 2) ? v16[0] : v16[1];
      const float keep = (lane & 2) ? v16[1] : v16[0];
      v16[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    float s = v16[0] + __shfl_xor_sync(0xffffffffu, v16[0], 1);
    const bool valid = b0 + my_tok < tok1;
    s = valid ? AT::round(AT::round(s) * scale) : -INFINITY;
    const float bm = warp_max(s);
    const float mnew = fmaxf(mrun, bm);
    const float p = valid ? expf(s - mnew) : 0.f;
    const float alpha = expf(mrun - mnew);
    const float lsum = warp_sum((lane & 1) ? 0.f : p);
    lrun = lrun * alpha + lsum;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] *= alpha;
#pragma unroll
    for (int j = 0; j < kPageTokens; ++j) {
      const float pj = __shfl_sync(0xffffffffu, p, lane_of_token(j));
      const Act* vh = reinterpret_cast<const Act*>(&vr[j]);
      if (owner && b0 + j == pos) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = fmaf(pj, vn_s[lane * 4 + e], acc[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = fmaf(pj, AT::to_f(vh[e]), acc[e]);
      }
    }
    mrun = mnew;
  }

  Act* out = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(m) * a.out_ld + h * kD + lane * 4;
  if (a.splits == 1) {
    float o[4];
    const float inv = lrun > 0.f ? 1.f / lrun : 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = acc[e] * inv;
    store4(out, o);
    return;
  }

  const int S = a.splits;
  const size_t prow = (static_cast<size_t>(m) * QH + h) * S;
  *reinterpret_cast<float4*>(a.part_o + (prow + split) * kD + lane * 4) =
      make_float4(acc[0], acc[1], acc[2], acc[3]);
  if (lane == 0) {
    a.part_ml[(prow + split) * 2] = mrun;
    a.part_ml[(prow + split) * 2 + 1] = lrun;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(a.counters + m * KVH + kvh, 1);
    last_flag = (old == S - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  float M = -INFINITY;
  for (int s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, __ldcg(a.part_ml + (prow + s2) * 2));
  M = warp_max(M);
  float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s2 = 0; s2 < S; ++s2) {
    const float ms = __ldcg(a.part_ml + (prow + s2) * 2);
    const float ls = __ldcg(a.part_ml + (prow + s2) * 2 + 1);
    const float w = ms == -INFINITY ? 0.f : expf(ms - M);
    L = fmaf(w, ls, L);
    const float4 po = __ldcg(reinterpret_cast<const float4*>(a.part_o + (prow + s2) * kD + lane * 4));
    o[0] = fmaf(w, po.x, o[0]);
    o[1] = fmaf(w, po.y, o[1]);
    o[2] = fmaf(w, po.z, o[2]);
    o[3] = fmaf(w, po.w, o[3]);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e] *= inv;
  store4(out, o);
  __syncthreads();
  if (threadIdx.x == 0) a.counters[m * KVH + kvh] = 0;
}

// Prefill KV append: token t of the session at position p0+t.  One warp per
// (token, kv head) writes the normed+roped K and the raw V into the pages.
template <typename Act>
__global__ void kv_append_kernel(const AttnPrefillArgs a) {
  const int t = blockIdx.x;
  const int kvh = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();
  if (kvh >= a.sh.kv_heads) return;
  const int pos = a.p0 + t;
  if (pos < 0 || pos >= a.sh.max_pos || pos / kPageTokens >= a.sh.max_blocks) {
    set_status(a.status, kStatusBadArgs);
    return;
  }
  const int QH = a.sh.q_heads, KVH = a.sh.kv_heads;
  const Act* qkv = reinterpret_cast<const Act*>(a.qkv) + static_cast<size_t>(t) * a.qkv_ld;
  const Act* cos_row = reinterpret_cast<const Act*>(a.cos) + static_cast<size_t>(pos) * (kD / 2);
  const Act* sin_row = reinterpret_cast<const Act*>(a.sin) + static_cast<size_t>(pos) * (kD / 2);
  float k[4], v[4];
  load4(qkv + (QH + kvh) * kD + lane * 4, k);
  load4(qkv + (QH + KVH + kvh) * kD + lane * 4, v);
  norm_rope<Act, true, true>(k, reinterpret_cast<const Act*>(a.k_norm_w), a.sh.eps, cos_row,
                             sin_row, lane);
  const int blk = a.block_table[pos / kPageTokens];
  const size_t off =
      ((static_cast<size_t>(blk) * KVH + kvh) * kPageTokens + (pos % kPageTokens)) * kD + lane * 4;
  store4(reinterpret_cast<Act*>(a.kv.k) + off, k);
  store4(reinterpret_cast<Act*>(a.kv.v) + off, v);
}

__global__ void iota_pos_kernel(int32_t* pos, int32_t* sid, int M, int p0) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < M) {
    pos[i] = p0 + i;
    sid[i] = 0;
  }
}

template <typename Act, int NREP>
cudaError_t launch_decode_t(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.sh.kv_heads, a.splits, a.M);
  cfg.blockDim = dim3(NREP * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<Act, NREP>, a);
}

template <typename Act>
cudaError_t launch_decode_act(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  switch (a.sh.q_heads / a.sh.kv_heads) {
    case 1: return launch_decode_t<Act, 1>(a, s, pdl);
    case 2: return launch_decode_t<Act, 2>(a, s, pdl);
    case 4: return launch_decode_t<Act, 4>(a, s, pdl);
    case 5: return launch_decode_t<Act, 5>(a, s, pdl);
    case 8: return launch_decode_t<Act, 8>(a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t attn_decode_scratch_bytes(const AttnShape& sh, int M, int splits) {
  if (splits <= 1) return 0;
  const size_t rows = static_cast<size_t>(M) * sh.q_heads * splits;
  return rows * kD * 4 + rows * 2 * 4 + static_cast<size_t>(M) * sh.kv_heads * 4;
}

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, int act, cudaStream_t s, bool pdl) {
  if (a.sh.head_dim != kD || a.M < 1 || a.splits < 1 ||
      a.sh.q_heads % a.sh.kv_heads != 0)
    return cudaErrorInvalidValue;
  if (a.splits > 1 && (!a.part_o || !a.part_ml || !a.counters)) return cudaErrorInvalidValue;
  return act == 0 ? launch_decode_act<__nv_bfloat16>(a, s, pdl)
                  : launch_decode_act<__half>(a, s, pdl);
}

cudaError_t attn_prefill_launch(const AttnPrefillArgs& a, int act, cudaStream_t s, bool pdl) {
  if (a.sh.head_dim != kD || a.M < 1 || a.sh.kv_heads > 32) return cudaErrorInvalidValue;
  {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.M);
    cfg.blockDim = dim3(32 * a.sh.kv_heads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = act == 0 ? cudaLaunchKernelEx(&cfg, kv_append_kernel<__nv_bfloat16>, a)
                             : cudaLaunchKernelEx(&cfg, kv_append_kernel<__half>, a);
    if (e != cudaSuccess) return e;
  }
  // Causal attention: row t attends to positions <= p0+t.
  int32_t* pos = a.rows_scratch;
  int32_t* sid = pos + a.M;
  iota_pos_kernel<<<(a.M + 255) / 256, 256, 0, s>>>(pos, sid, a.M, a.p0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  AttnDecodeArgs d{};
  d.sh = a.sh;
  d.qkv = a.qkv;
  d.qkv_ld = a.qkv_ld;
  d.q_norm_w = a.q_norm_w;
  d.k_norm_w = a.k_norm_w;
  d.cos = a.cos;
  d.sin = a.sin;
  d.kv = a.kv;
  d.block_table = a.block_table;
  d.sid = sid;
  d.pos = pos;
  d.out = a.out;
  d.out_ld = a.out_ld;
  d.M = a.M;
  d.splits = 1;
  d.status = a.status;
  return attn_decode_launch(d, act, s, false);
}

}  // namespace dialb200
