// Device-side pieces of the decode GEMV (chunk conversion + MMA, SwiGLU).
//
// Chunk layout (built by layout.cu): 16 weight rows x KCH inputs per chunk;
// lane l = (g, c) = (l / 4, l % 4) owns bytes [16l, 16l+16) (row g) and
// [512 + 16l, ...) (row g+8).  Within its 16 bytes the lane's inputs are in
// natural order; the m16n8k16 K index is permuted identically for the
// activation fragment, so no shuffle is needed.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "gemv.h"
#include "qlinear.h"

namespace dialb200 {

// ---------------------------------------------------------- chunk compute
// acc: 16 rows x 8 tokens C fragment.  xrow: this lane's token row in smem.
template <int FMT, typename XT>
__device__ __forceinline__ void chunk_mma(const uint8_t* st, int kc, const XT* xrow, int lane,
                                          float (&acc)[4]) {
  const int c = lane & 3;
  if constexpr (FMT == kFmtW8A16Row || FMT == kFmtFp8Row || FMT == kFmtFp8Block128) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(st + lane * 16);
    const uint4 w1 = *reinterpret_cast<const uint4*>(st + 512 + lane * 16);
    const XT* xp = xrow + kc * 64 + c * 16;
    const uint4 xa = *reinterpret_cast<const uint4*>(xp);
    const uint4 xb = *reinterpret_cast<const uint4*>(xp + 8);
    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
    const uint32_t wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t A[4];
      if constexpr (FMT == kFmtW8A16Row) {
        A[0] = i8_lo_pair(wa[s]);
        A[1] = i8_lo_pair(wb[s]);
        A[2] = i8_hi_pair(wa[s]);
        A[3] = i8_hi_pair(wb[s]);
      } else {
        A[0] = e4m3x2_to_f16x2(static_cast<uint16_t>(wa[s] & 0xffffu));
        A[1] = e4m3x2_to_f16x2(static_cast<uint16_t>(wb[s] & 0xffffu));
        A[2] = e4m3x2_to_f16x2(static_cast<uint16_t>(wa[s] >> 16));
        A[3] = e4m3x2_to_f16x2(static_cast<uint16_t>(wb[s] >> 16));
      }
      mma_f16(acc, A, xw[2 * s], xw[2 * s + 1]);
    }
  } else if constexpr (FMT == kFmtNvfp4G16) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(st + lane * 16);
    const uint4 w1 = *reinterpret_cast<const uint4*>(st + 512 + lane * 16);
    const uint16_t s0 = *reinterpret_cast<const uint16_t*>(st + 1024 + lane * 2);
    const uint16_t s1 = *reinterpret_cast<const uint16_t*>(st + 1024 + 64 + lane * 2);
    const uint32_t sg0 = e4m3x2_to_f16x2(s0);  // row g   : groups (2c, 2c+1)
    const uint32_t sg1 = e4m3x2_to_f16x2(s1);  // row g+8
    const __half2 sc0[2] = {__low2half2(*reinterpret_cast<const __half2*>(&sg0)),
                            __high2half2(*reinterpret_cast<const __half2*>(&sg0))};
    const __half2 sc1[2] = {__low2half2(*reinterpret_cast<const __half2*>(&sg1)),
                            __high2half2(*reinterpret_cast<const __half2*>(&sg1))};
    const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
    const uint32_t wb[4] = {w1.x, w1.y, w1.z, w1.w};
    const XT* xp = xrow + kc * 128 + c * 32;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t oa[4], ob[4];
      e2m1x8_to_f16x2x4(wa[s], oa);
      e2m1x8_to_f16x2x4(wb[s], ob);
      const int gj = s >> 1;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 ha = __hmul2(*reinterpret_cast<__half2*>(&oa[q]), sc0[gj]);
        __half2 hb = __hmul2(*reinterpret_cast<__half2*>(&ob[q]), sc1[gj]);
        oa[q] = *reinterpret_cast<uint32_t*>(&ha);
        ob[q] = *reinterpret_cast<uint32_t*>(&hb);
      }
      const uint4 xv = *reinterpret_cast<const uint4*>(xp + 8 * s);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t A[4] = {oa[2 * h], ob[2 * h], oa[2 * h + 1], ob[2 * h + 1]};
        const uint32_t b0 = h ? xv.z : xv.x;
        const uint32_t b1 = h ? xv.w : xv.y;
        mma_f16(acc, A, b0, b1);
      }
    }
  } else {  // dense act-dtype weights
    const uint4 w0 = *reinterpret_cast<const uint4*>(st + lane * 16);
    const uint4 w1 = *reinterpret_cast<const uint4*>(st + 512 + lane * 16);
    const XT* xp = xrow + kc * 32 + c * 8;
    const uint4 xv = *reinterpret_cast<const uint4*>(xp);
    const uint32_t A0[4] = {w0.x, w1.x, w0.y, w1.y};
    const uint32_t A1[4] = {w0.z, w1.z, w0.w, w1.w};
    if constexpr (std::is_same<XT, __nv_bfloat16>::value) {
      mma_bf16(acc, A0, xv.x, xv.y);
      mma_bf16(acc, A1, xv.z, xv.w);
    } else {
      mma_f16(acc, A0, xv.x, xv.y);
      mma_f16(acc, A1, xv.z, xv.w);
    }
  }
}

// Two neighbouring int8 / e4m3 chunks of one stage with their MMAs
// interleaved into four independent accumulator chains (chunk 0 -> acc[0..1],
// chunk 1 -> acc[2..3], even/odd k16 steps alternating), so the tensor pipe's
// dependent-issue latency is hidden within one warp.
template <int FMT, typename XT>
__device__ __forceinline__ void chunk_pair_mma(const uint8_t* st, int kc, const XT* xrow, int lane,
                                               float (&acc)[4][4]) {
  static_assert(FMT == kFmtW8A16Row || FMT == kFmtFp8Row || FMT == kFmtFp8Block128, "int8/e4m3");
  const int c = lane & 3;
  uint4 w[2][2];
  uint32_t xw[2][8];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    w[h][0] = *reinterpret_cast<const uint4*>(st + h * 1024 + lane * 16);
    w[h][1] = *reinterpret_cast<const uint4*>(st + h * 1024 + 512 + lane * 16);
    const XT* xp = xrow + (kc + h) * 64 + c * 16;
    const uint4 xa = *reinterpret_cast<const uint4*>(xp);
    const uint4 xb = *reinterpret_cast<const uint4*>(xp + 8);
    xw[h][0] = xa.x; xw[h][1] = xa.y; xw[h][2] = xa.z; xw[h][3] = xa.w;
    xw[h][4] = xb.x; xw[h][5] = xb.y; xw[h][6] = xb.z; xw[h][7] = xb.w;
  }
#pragma unroll
  for (int s = 0; s < 4; ++s) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wa = (&w[h][0].x)[s], wb = (&w[h][1].x)[s];
      uint32_t A[4];
      if constexpr (FMT == kFmtW8A16Row) {
        A[0] = i8_lo_pair(wa);
        A[1] = i8_lo_pair(wb);
        A[2] = i8_hi_pair(wa);
        A[3] = i8_hi_pair(wb);
      } else {
        A[0] = e4m3x2_to_f16x2(static_cast<uint16_t>(wa & 0xffffu));
        A[1] = e4m3x2_to_f16x2(static_cast<uint16_t>(wb & 0xffffu));
        A[2] = e4m3x2_to_f16x2(static_cast<uint16_t>(wa >> 16));
        A[3] = e4m3x2_to_f16x2(static_cast<uint16_t>(wb >> 16));
      }
      mma_f16(acc[2 * h + (s & 1)], A, xw[h][2 * s], xw[h][2 * s + 1]);
    }
  }
}

// Two NVFP4 chunks of one stage (anywhere in it) with their MMAs interleaved
// into four independent accumulator chains (chunk h -> acc[2h], acc[2h + 1]
// for the two MMAs of each 32-input step), as chunk_pair_mma does for int8.
template <typename XT>
__device__ __forceinline__ void chunk_pair_nvfp4(const uint8_t* st0, int kc0, const uint8_t* st1,
                                                 int kc1, const XT* xrow, int lane,
                                                 float (&acc)[4][4]) {
  const int c = lane & 3;
  const uint8_t* st[2] = {st0, st1};
  const XT* xp[2] = {xrow + kc0 * 128 + c * 32, xrow + kc1 * 128 + c * 32};
  uint4 w0[2], w1[2];
  __half2 sc0[2][2], sc1[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    w0[h] = *reinterpret_cast<const uint4*>(st[h] + lane * 16);
    w1[h] = *reinterpret_cast<const uint4*>(st[h] + 512 + lane * 16);
    const uint32_t sg0 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(st[h] + 1024 + lane * 2));
    const uint32_t sg1 =
        e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(st[h] + 1024 + 64 + lane * 2));
    sc0[h][0] = __low2half2(*reinterpret_cast<const __half2*>(&sg0));
    sc0[h][1] = __high2half2(*reinterpret_cast<const __half2*>(&sg0));
    sc1[h][0] = __low2half2(*reinterpret_cast<const __half2*>(&sg1));
    sc1[h][1] = __high2half2(*reinterpret_cast<const __half2*>(&sg1));
  }
#pragma unroll
  for (int s = 0; s < 4; ++s) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t oa[4], ob[4];
      e2m1x8_to_f16x2x4((&w0[h].x)[s], oa);
      e2m1x8_to_f16x2x4((&w1[h].x)[s], ob);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 ha = __hmul2(*reinterpret_cast<__half2*>(&oa[q]), sc0[h][s >> 1]);
        __half2 hb = __hmul2(*reinterpret_cast<__half2*>(&ob[q]), sc1[h][s >> 1]);
        oa[q] = *reinterpret_cast<uint32_t*>(&ha);
        ob[q] = *reinterpret_cast<uint32_t*>(&hb);
      }
      const uint4 xv = *reinterpret_cast<const uint4*>(xp[h] + 8 * s);
      const uint32_t A0[4] = {oa[0], ob[0], oa[1], ob[1]};
      const uint32_t A1[4] = {oa[2], ob[2], oa[3], ob[3]};
      mma_f16(acc[2 * h], A0, xv.x, xv.y);
      mma_f16(acc[2 * h + 1], A1, xv.z, xv.w);
    }
  }
}

// ------------------------------------------------------------ x staging
// Stage the M activation rows of a GEMV in shared memory (NW consumer warps,
// named barrier 1): optional RMSNorm (text.rs:1620-1626 rounding), then f16
// with a power-of-two pre-scale xexp[r] when the values would overflow f16
// (bf16 inputs), or the activation dtype itself for dense weights.
template <typename Act, typename XT, bool NORM, bool SCALE, int NW>
__device__ void stage_x_scalar(const GemvArgs& a, XT* xs, int xs_stride, int* xexp,
                               float* scratch) {
  using AT = ActTraits<Act>;
  const int tid = threadIdx.x;
  constexpr int NT = NW * 32;
  const int K = a.w.K, Kp = a.w.K_pad;
  const Act* nw = reinterpret_cast<const Act*>(a.norm_w);
  const int warp = tid >> 5, lane = tid & 31;

  float wmax = 1.f;
  if (NORM && SCALE) {
    float m = 0.f;
    for (int k = tid; k < K; k += NT) m = fmaxf(m, fabsf(AT::to_f(nw[k])));
    m = warp_max(m);
    if (lane == 0) scratch[warp] = m;
    named_bar_sync(1, NT);
    m = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) m = fmaxf(m, scratch[i]);
    wmax = m;
    named_bar_sync(1, NT);
  }
  for (int r = 0; r < a.M; ++r) {
    const Act* xr = reinterpret_cast<const Act*>(a.x) + static_cast<size_t>(r) * a.x_ld;
    float ss = 0.f, am = 0.f;
    for (int k = tid; k < K; k += NT) {
      const float v = AT::to_f(xr[k]);
      ss = fmaf(v, v, ss);
      am = fmaxf(am, fabsf(v));
    }
    ss = warp_sum(ss);
    am = warp_max(am);
    if (lane == 0) {
      scratch[warp] = ss;
      scratch[NW + warp] = am;
    }
    named_bar_sync(1, NT);
    ss = 0.f;
    am = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      ss += scratch[i];
      am = fmaxf(am, scratch[NW + i]);
    }
    named_bar_sync(1, NT);
    float rms = 1.f;
    if (NORM) rms = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(K)) + a.eps));
    int e = 0;
    if (SCALE) {
      const float bound = NORM ? __fdiv_rn(am, rms) * wmax * 1.02f : am;
      if (bound >= 16384.f) e = ilogbf(bound) - 13;
    }
    const float sc = exp2i(-e);
    XT* xrow = xs + static_cast<size_t>(r) * xs_stride;
    for (int k = tid; k < Kp; k += NT) {
      float v = 0.f;
      if (k < K) {
        v = AT::to_f(xr[k]);
        if (NORM) {
          v = AT::round(__fdiv_rn(v, rms));
          v = AT::round(v * AT::to_f(nw[k]));
        }
      }
      if constexpr (sizeof(XT) == 2 && std::is_same<XT, __half>::value) {
        xrow[k] = __float2half_rn(v * sc);
      } else {
        xrow[k] = ActTraits<XT>::from_f(v);
      }
    }
    if (tid == 0) xexp[r] = e;
  }
}

// 16-byte vector form of stage_x: every load of a row is issued at once
// (one L2 round trip), the sum of squares and the pre-scale bound come from
// one block reduction, and the converted row is written with 16-byte stores.
// Rows whose length, stride or address do not allow 16-byte access, or that
// exceed kStageVec vectors per thread, take stage_x_scalar.
constexpr int kStageVec = 6;

template <typename Act>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const Act* p = reinterpret_cast<const Act*>(&v);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = ActTraits<Act>::to_f(p[e]);
}

template <typename Act, typename XT, bool NORM, bool SCALE, int NW>
__device__ void stage_x(const GemvArgs& a, XT* xs, int xs_stride, int* xexp, float* scratch) {
  using AT = ActTraits<Act>;
  constexpr int NT = NW * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.w.K, Kp = a.w.K_pad;
  const bool vec = (K % 8) == 0 && (a.x_ld % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                   (!NORM || (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0) &&
                   K <= kStageVec * 8 * NT && (xs_stride % 8) == 0;
  if (!vec) {
    stage_x_scalar<Act, XT, NORM, SCALE, NW>(a, xs, xs_stride, xexp, scratch);
    return;
  }
  const int nv = K / 8;
  const uint4* wr = reinterpret_cast<const uint4*>(a.norm_w);
  for (int r = 0; r < a.M; ++r) {
    const uint4* xr =
        reinterpret_cast<const uint4*>(reinterpret_cast<const Act*>(a.x) + static_cast<size_t>(r) * a.x_ld);
    uint4 xv[kStageVec], wv[kStageVec];
#pragma unroll
    for (int j = 0; j < kStageVec; ++j) {
      const int i = tid + j * NT;
      if (i < nv) {
        xv[j] = __ldcg(xr + i);  // produced by other SMs: read through L2
        if (NORM) wv[j] = __ldg(wr + i);
      }
    }
    float ss = 0.f, am = 0.f;
#pragma unroll
    for (int j = 0; j < kStageVec; ++j) {
      if (tid + j * NT < nv) {
        float xf[8], wf[8];
        unpack8<Act>(xv[j], xf);
        if (NORM) unpack8<Act>(wv[j], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ss = fmaf(xf[e], xf[e], ss);
          am = fmaxf(am, fabsf(NORM ? xf[e] * wf[e] : xf[e]));
        }
      }
    }
    ss = warp_sum(ss);
    am = warp_max(am);
    if (lane == 0) {
      scratch[warp] = ss;
      scratch[NW + warp] = am;
    }
    named_bar_sync(1, NT);
    ss = 0.f;
    am = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      ss += scratch[i];
      am = fmaxf(am, scratch[NW + i]);
    }
    named_bar_sync(1, NT);
    float rms = 1.f;
    if (NORM) rms = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(K)) + a.eps));
    int e = 0;
    if (SCALE) {
      // NORM: staged values are act(act(x/rms)*w) <= |x*w|/rms * (1 + 2^-7)
      const float bound = NORM ? __fdiv_rn(am, rms) * 1.02f : am;
      if (bound >= 16384.f) e = ilogbf(bound) - 13;
    }
    const float sc = exp2i(-e);
    XT* xrow = xs + static_cast<size_t>(r) * xs_stride;
#pragma unroll
    for (int j = 0; j < kStageVec; ++j) {
      const int i = tid + j * NT;
      if (i < nv) {
        float xf[8], wf[8];
        unpack8<Act>(xv[j], xf);
        if (NORM) unpack8<Act>(wv[j], wf);
        uint4 o;
        XT* op = reinterpret_cast<XT*>(&o);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float v = xf[q];
          if (NORM) {
            v = AT::round(__fdiv_rn(v, rms));
            v = AT::round(v * wf[q]);
          }
          if constexpr (std::is_same<XT, __half>::value) {
            op[q] = __float2half_rn(v * sc);
          } else {
            op[q] = ActTraits<XT>::from_f(v);
          }
        }
        *reinterpret_cast<uint4*>(xrow + static_cast<size_t>(i) * 8) = o;
      }
    }
    for (int k = K + tid; k < Kp; k += NT) xrow[k] = ActTraits<XT>::from_f(0.f);
    if (tid == 0) xexp[r] = e;
  }
}

// Greedy-argmax key: larger value wins, then the lower index (the first of
// equal maxima, as candle's argmax over the logits, qwen3_vl.rs:138-143).
// -0 counts as +0.
__device__ __forceinline__ unsigned long long argmax_key(float y, int n) {
  uint32_t b = __float_as_uint(y == 0.f ? 0.f : y);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

template <typename Act>
__device__ __forceinline__ float silu_mul_ref(float g, float u) {
  using AT = ActTraits<Act>;
  // act(act(g / act(1 + act(exp(-g)))) * u)  (text.rs:816-820 via candle silu)
  const float e = AT::round(expf(-g));
  const float d = AT::round(1.f + e);
  const float s = AT::round(__fdiv_rn(g, d));
  return s * u;
}

}  // namespace dialb200
