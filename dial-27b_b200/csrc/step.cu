// Persistent decode-step kernel: one launch runs a whole decode token --
// embedding, every decoder layer (QKV GEMV + q/k norm + RoPE + KV append +
// split-KV attention + o_proj + gate/up SwiGLU + down) and the lm_head with
// the greedy argmax -- as a program of ops over one CTA per SM.
//
// It is the B200 counterpart of the reference's per-token forward
// (qwen3_vl.rs:2018-2177 forward_blocks_from over text.rs:1636-1688 layers,
// then qwen3_vl.rs:2462-2487 head and 138-143 argmax), with the same
// arithmetic as the per-op kernels in gemv.cu / attention.cu.
//
// Why one kernel: a decode token streams 8.2 GB of weights through ~180
// dependent ops; as separate launches each op pays launch latency, pipeline
// fill and a tail.  Here the producer warp of every CTA streams its share of
// the weights of op after op into a shared-memory ring without waiting for
// the activations (weights do not depend on them), so HBM keeps streaming
// while the consumer warps wait at the grid barrier between dependent ops.
//
// Work split: the weight stream of a linear is cut into units of one ring
// stage (16 chunks = 16 rows x 1024 columns of int8), and CTA b takes the
// contiguous unit range [U*b/G, U*(b+1)/G).  A 16-row tile cut by a range
// boundary is finished by the last CTA to arrive on its counter, which adds
// the parts in CTA order (deterministic).  Grid barriers are one monotonic
// counter per launch; every wait is bounded (status code + clean exit).
#include <cmath>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv_dev.cuh"
#include "step.h"

namespace dialb200 {
namespace {

constexpr int kNC = 8;                      // consumer warps
constexpr int kThreads = (kNC + 1) * 32;    // + producer warp
constexpr int kStage = 16;                  // chunks per ring stage
constexpr int kChunk = 1024;                // bytes per chunk (int8, e4m3, dense)
constexpr int kStageBytes = kStage * kChunk;
constexpr int kMaxSlots = 16;
constexpr int kSmemBudget = 232448;
constexpr int kStatusGridWait = 0x301;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Range of units of CTA b, and the CTA that owns unit u.
__device__ __forceinline__ long long unit_lo(long long U, int b, int G) {
  return U * b / G;
}
__device__ __forceinline__ int unit_owner(long long u, long long U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}

struct Smem {
  uint8_t* ring;
  void* xs;
  float* red;
  float* tv;
  int* xexp;
  float* scratch;
  int* flag;         // [0] last-arrival flag, [1] abort
  unsigned long long* skey;
  AttnItemSmem* attn;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* xbar;    // activation-row bulk copy
};

// --------------------------------------------------------------- producer
__device__ void producer(const StepArgs& a, const Smem& sm, int NS) {
  const int G = gridDim.x, b = blockIdx.x;
  int slot = 0;
  uint32_t round = 0;
  long long it = 0;
  bool ok = true;
  for (int k = 0; k < a.n_ops && ok; ++k) {
    const StepOp& op = a.ops[k];
    if (op.kind != kOpGemv) continue;
    const int S = op.S, C = op.w.C;
    const long long U = static_cast<long long>(op.w.T) * S;
    const long long u0 = unit_lo(U, b, G), u1 = unit_lo(U, b + 1, G);
    const uint8_t* tiles = op.w.tiles;
    for (long long u = u0; u < u1; ++u, ++it) {
      const int t = static_cast<int>(u / S), s = static_cast<int>(u % S);
      if (round > 0 &&
          !mbar_wait(&sm.empty[slot], (round - 1) & 1u, a.status, kStatusEmptyWaitTimeout)) {
        ok = false;
        break;
      }
      const int nch = min(kStage, C - s * kStage);
      const uint32_t bytes = static_cast<uint32_t>(nch * kChunk);
      mbar_arrive_expect_tx(&sm.full[slot], bytes);
      bulk_g2s(sm.ring + static_cast<size_t>(slot) * kStageBytes,
               tiles + (static_cast<size_t>(t) * C + static_cast<size_t>(s) * kStage) * kChunk,
               bytes, &sm.full[slot]);
      if (++slot == NS) {
        slot = 0;
        ++round;
      }
    }
  }
  // the most recent NS stages must land before the CTA may retire
  const long long first = it > NS ? it - NS : 0;
  for (long long j = first; j < it; ++j) {
    if (!mbar_wait(&sm.full[j % NS], static_cast<uint32_t>(j / NS) & 1u, a.status,
                   kStatusDrainTimeout))
      break;
  }
}

// ---------------------------------------------------------- grid barrier
__device__ __forceinline__ void grid_arrive(const StepArgs& a) {
  named_bar_sync(1, kNC * 32);
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.bar, 1u);
  }
}

// Wait until `target` arrivals; returns false (status set) on timeout.
__device__ bool grid_wait(const StepArgs& a, unsigned target, const Smem& sm) {
  if (threadIdx.x == 0) {
    int abort = 0;
    if (ld_acquire(a.bar) < target) {
      const unsigned long long t0 = global_ns();
      while (ld_acquire(a.bar) < target) {
        if (global_ns() - t0 > kWaitLimitNs) {
          set_status(a.status, kStatusGridWait);
          abort = 1;
          break;
        }
      }
    }
    sm.flag[1] = abort;
  }
  named_bar_sync(1, kNC * 32);
  return sm.flag[1] == 0;
}

// ------------------------------------------------------------- embedding
__device__ void embed_op(const StepArgs& a) {
  const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
  const int n16 = a.H * 2 / 16;
  const int total = a.M * n16;
  const uint4* table = reinterpret_cast<const uint4*>(a.embed);
  uint4* hid = reinterpret_cast<uint4*>(a.hidden);
  for (int i = b * (kNC * 32) + tid; i < total; i += G * kNC * 32) {
    const int m = i / n16, j = i % n16;
    int tok = a.tok_in[m];
    if (tok < 0 || tok >= a.vocab) {
      set_status(a.status, kStatusBadArgs);
      tok = 0;
    }
    hid[static_cast<size_t>(m) * n16 + j] = table[static_cast<size_t>(tok) * n16 + j];
  }
}

// ------------------------------------------------------------- attention
template <typename Act, int NREP>
__device__ void attn_op(const StepOp& op, int M, const Smem& sm) {
  constexpr int kGroups = kNC / NREP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = warp / NREP, r = warp % NREP;
  if (g >= kGroups) return;
  const AttnDecodeArgs& at = op.attn;
  const int KVH = at.sh.kv_heads, splits = at.splits;
  const int items = M * KVH * splits;
  const int G = gridDim.x;
  for (int i = blockIdx.x + G * g; i < items; i += G * kGroups) {
    const int m = i / (KVH * splits);
    const int rem = i % (KVH * splits);
    attn_item<Act, NREP>(at, m, rem / splits, rem % splits, r, lane, sm.attn[g], 2 + g);
  }
}

// ------------------------------------------------------------------ GEMV
// Epilogue of one finished 16-row tile from the tile sums tv[(row << 3) | tok].
// Row scales and residual inputs of tile t for thread i < 128, loaded when
// the tile starts so that their latency hides behind the tile's stages.
template <typename Act>
__device__ __forceinline__ void tile_prefetch(const StepOp& op, int M, int t, float& pre_a,
                                              float& pre_b, float& pre_o) {
  const int i = threadIdx.x;
  pre_a = pre_b = 1.f;
  pre_o = 0.f;
  if (i >= 128) return;
  const DevQLinear& w = op.w;
  const int rr = i >> 3, tt = i & 7;
  if (op.epi == kEpiSwiglu) {
    if (i < 64 && w.row_scale) {
      pre_a = __ldg(w.row_scale + t * 16 + rr);
      pre_b = __ldg(w.row_scale + t * 16 + 8 + rr);
    }
    return;
  }
  if (w.row_scale) pre_a = __ldg(w.row_scale + t * 16 + rr);
  const int n = t * 16 + rr;
  if (op.epi == kEpiResidual && tt < M && n < w.N) {
    const unsigned short bits = __ldcg(reinterpret_cast<const unsigned short*>(op.out) +
                                       static_cast<size_t>(tt) * op.out_ld + n);
    pre_o = ActTraits<Act>::to_f(*reinterpret_cast<const Act*>(&bits));
  }
}

template <typename Act>
__device__ void tile_epilogue(const StepOp& op, int M, int t, const Smem& sm, float pre_a,
                              float pre_b, float pre_o) {
  using AT = ActTraits<Act>;
  const int i = threadIdx.x;
  const DevQLinear& w = op.w;
  if (op.epi == kEpiSwiglu) {
    if (i < 64) {
      const int rr = i >> 3, tt = i & 7;
      const int I = w.N / 2;
      const int j = t * 8 + rr;
      if (tt < M && j < I) {
        const float mul = exp2i(sm.xexp[tt]);
        const float sg = mul * pre_a, su = mul * pre_b;
        const float gq = AT::round(sm.tv[(rr << 3) | tt] * sg);
        const float uq = AT::round(sm.tv[((rr + 8) << 3) | tt] * su);
        reinterpret_cast<Act*>(op.out)[static_cast<size_t>(tt) * op.out_ld + j] =
            AT::from_f(silu_mul_ref<Act>(gq, uq));
      }
    }
    return;
  }
  if (i < 128) {
    const int rr = i >> 3, tt = i & 7;
    const int n = t * 16 + rr;
    if (tt < M && n < w.N) {
      const float mul = exp2i(sm.xexp[tt]) * pre_a;
      const float y = AT::round(sm.tv[i] * mul);
      if (op.epi == kEpiArgmax) {
        if (op.out)
          reinterpret_cast<Act*>(op.out)[static_cast<size_t>(tt) * op.out_ld + n] = AT::from_f(y);
        atomicMax(&sm.skey[tt], argmax_key(y, n));
      } else {
        Act* o = reinterpret_cast<Act*>(op.out) + static_cast<size_t>(tt) * op.out_ld + n;
        *o = op.epi == kEpiResidual ? AT::from_f(y + pre_o) : AT::from_f(y);
      }
    }
  }
}

// Stage the op's activation rows: one 1-D bulk copy per row into shared
// memory (no registers held), then RMSNorm / pre-scale / conversion in place
// with the same rounding as stage_x in gemv_dev.cuh.  The RMSNorm weights
// (K <= kStepNormVec * 8 * 256) are loaded into registers while the copy
// is in flight.
constexpr int kStepNormVec = 4;

template <typename Act, typename XT, bool NORM, bool SCALE>
__device__ void stage_op_x(const StepArgs& a, const StepOp& op, const Smem& sm, int xs_stride,
                           uint32_t& xphase) {
  using AT = ActTraits<Act>;
  constexpr int NT = kNC * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = op.w.K, Kp = op.w.K_pad, nv = K / 8;
  uint4 wv[kStepNormVec];
  if (NORM) {
    const uint4* wr = reinterpret_cast<const uint4*>(op.norm_w);
#pragma unroll
    for (int j = 0; j < kStepNormVec; ++j)
      if (tid + j * NT < nv) wv[j] = __ldg(wr + tid + j * NT);
  }
  Act* raw = reinterpret_cast<Act*>(sm.xs);
  if (tid == 0) {
    asm volatile("fence.proxy.async;" ::: "memory");
    mbar_arrive_expect_tx(sm.xbar, static_cast<uint32_t>(a.M * K * 2));
    for (int r = 0; r < a.M; ++r)
      bulk_g2s(raw + static_cast<size_t>(r) * xs_stride,
               reinterpret_cast<const Act*>(op.x) + static_cast<size_t>(r) * op.x_ld,
               static_cast<uint32_t>(K * 2), sm.xbar);
  }
  mbar_wait(sm.xbar, xphase, a.status, kStatusFullWaitTimeout);
  xphase ^= 1u;
  // NORM: thread tid owns vectors tid + j*NT (weights held in wv[j]);
  // otherwise any number of vectors per thread.
  auto for_each_vec = [&](auto&& f) {
    if (NORM) {
#pragma unroll
      for (int j = 0; j < kStepNormVec; ++j)
        if (tid + j * NT < nv) f(tid + j * NT, wv[j]);
    } else {
      for (int i = tid; i < nv; i += NT) f(i, wv[0]);
    }
  };
  for (int r = 0; r < a.M; ++r) {
    uint4* row = reinterpret_cast<uint4*>(raw + static_cast<size_t>(r) * xs_stride);
    float ss = 0.f, am = 0.f;
    for_each_vec([&](int i, const uint4& w) {
      float xf[8], wf[8];
      unpack8<Act>(row[i], xf);
      if (NORM) unpack8<Act>(w, wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(xf[e], xf[e], ss);
        am = fmaxf(am, fabsf(NORM ? xf[e] * wf[e] : xf[e]));
      }
    });
    ss = warp_sum(ss);
    am = warp_max(am);
    if (lane == 0) {
      sm.scratch[warp] = ss;
      sm.scratch[kNC + warp] = am;
    }
    named_bar_sync(1, NT);
    ss = 0.f;
    am = 0.f;
#pragma unroll
    for (int i = 0; i < kNC; ++i) {
      ss += sm.scratch[i];
      am = fmaxf(am, sm.scratch[kNC + i]);
    }
    named_bar_sync(1, NT);
    float rms = 1.f;
    if (NORM) rms = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(K)) + a.eps));
    int e = 0;
    if (SCALE) {
      const float bound = NORM ? __fdiv_rn(am, rms) * 1.02f : am;
      if (bound >= 16384.f) e = ilogbf(bound) - 13;
    }
    const float sc = exp2i(-e);
    for_each_vec([&](int i, const uint4& w) {
      float xf[8], wf[8];
      unpack8<Act>(row[i], xf);
      if (NORM) unpack8<Act>(w, wf);
      uint4 o;
      XT* op8 = reinterpret_cast<XT*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float v = xf[q];
        if (NORM) {
          v = AT::round(__fdiv_rn(v, rms));
          v = AT::round(v * wf[q]);
        }
        if constexpr (std::is_same<XT, __half>::value) {
          op8[q] = __float2half_rn(v * sc);
        } else {
          op8[q] = ActTraits<XT>::from_f(v);
        }
      }
      row[i] = o;
    });
    XT* xrow = reinterpret_cast<XT*>(row);
    for (int k = K + tid; k < Kp; k += NT) xrow[k] = ActTraits<XT>::from_f(0.f);
    if (tid == 0) sm.xexp[r] = e;
  }
}

template <typename Act>
__device__ void gemv_op(const StepArgs& a, const StepOp& op, int op_index, const Smem& sm,
                        const StepPlan& p, int& slot, uint32_t& round, int& parity, bool& ok,
                        uint32_t& xphase) {
  const int G = gridDim.x, b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int fmt = op.w.fmt;
  const int S = op.S, C = op.w.C, NS = p.slots;
  const long long U = static_cast<long long>(op.w.T) * S;
  const long long u0 = unit_lo(U, b, G), u1 = unit_lo(U, b + 1, G);
  constexpr bool kScaleX = std::is_same<Act, __nv_bfloat16>::value;

  if (op.epi == kEpiArgmax && tid < kStepMaxM) sm.skey[tid] = 0ull;
  if (fmt == kFmtDense) {
    if (op.norm_w)
      stage_op_x<Act, Act, true, false>(a, op, sm, p.xs_stride, xphase);
    else
      stage_op_x<Act, Act, false, false>(a, op, sm, p.xs_stride, xphase);
  } else {
    if (op.norm_w)
      stage_op_x<Act, __half, true, kScaleX>(a, op, sm, p.xs_stride, xphase);
    else
      stage_op_x<Act, __half, false, kScaleX>(a, op, sm, p.xs_stride, xphase);
  }
  named_bar_sync(1, kNC * 32);
  if (a.trace && tid == 0) atomicMax(a.trace + op_index * kTraceFields + 1, global_ns());

  const int tok = min(lane >> 2, a.M - 1);
  const __half* xh = reinterpret_cast<const __half*>(sm.xs) + static_cast<size_t>(tok) * p.xs_stride;
  const Act* xa = reinterpret_cast<const Act*>(sm.xs) + static_cast<size_t>(tok) * p.xs_stride;
  const int ch0 = warp * 2, ch1 = warp * 2 + 1;

  float acc[4], acc2[4], pacc[4][4];
  float pre_a = 1.f, pre_b = 1.f, pre_o = 0.f;
  int t_next = static_cast<int>(u0 / S), s_next = static_cast<int>(u0 % S);
  for (long long u = u0; u < u1; ++u) {
    const int t = t_next, s = s_next;
    if (++s_next == S) {
      s_next = 0;
      ++t_next;
    }
    if (u == u0 || s == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[q] = acc2[q] = 0.f;
        pacc[0][q] = pacc[1][q] = pacc[2][q] = pacc[3][q] = 0.f;
      }
      tile_prefetch<Act>(op, a.M, t, pre_a, pre_b, pre_o);
    }
    if (ok && !mbar_wait(&sm.full[slot], round & 1u, a.status, kStatusFullWaitTimeout)) ok = false;
    if (ok) {
      const int nch = min(kStage, C - s * kStage);
      const uint8_t* st = sm.ring + static_cast<size_t>(slot) * kStageBytes;
      const int kc = s * kStage;
      if (fmt == kFmtW8A16Row) {
        if (nch == kStage) {
          chunk_pair_mma<kFmtW8A16Row, __half>(st + ch0 * kChunk, kc + ch0, xh, lane, pacc);
        } else {
          if (ch0 < nch) chunk_mma<kFmtW8A16Row, __half>(st + ch0 * kChunk, kc + ch0, xh, lane, acc);
          if (ch1 < nch) chunk_mma<kFmtW8A16Row, __half>(st + ch1 * kChunk, kc + ch1, xh, lane, acc2);
        }
      } else if (fmt == kFmtFp8Row) {
        if (nch == kStage) {
          chunk_pair_mma<kFmtFp8Row, __half>(st + ch0 * kChunk, kc + ch0, xh, lane, pacc);
        } else {
          if (ch0 < nch) chunk_mma<kFmtFp8Row, __half>(st + ch0 * kChunk, kc + ch0, xh, lane, acc);
          if (ch1 < nch) chunk_mma<kFmtFp8Row, __half>(st + ch1 * kChunk, kc + ch1, xh, lane, acc2);
        }
      } else {  // dense activation-dtype weights (lm_head)
        if (ch0 < nch) chunk_mma<kFmtDense, Act>(st + ch0 * kChunk, kc + ch0, xa, lane, acc);
        if (ch1 < nch) chunk_mma<kFmtDense, Act>(st + ch1 * kChunk, kc + ch1, xa, lane, acc2);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    if (++slot == NS) {
      slot = 0;
      ++round;
    }
    if (s != S - 1 && u != u1 - 1) continue;

    // ---- this CTA's part of tile t is done: reduce over warps
    float* rb = sm.red + parity * (kNC * 128);
    parity ^= 1;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      acc[q] += acc2[q] + ((pacc[0][q] + pacc[1][q]) + (pacc[2][q] + pacc[3][q]));
    *reinterpret_cast<float4*>(rb + (warp * 32 + lane) * 4) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
    named_bar_sync(1, kNC * 32);
    const long long tu0 = static_cast<long long>(t) * S, tu1 = tu0 + S - 1;
    const bool complete = tu0 >= u0 && tu1 < u1;
    if (tid < 128) {
      const int rr = tid >> 3, tt = tid & 7;
      const int src_lane = (rr & 7) * 4 + (tt >> 1);
      const int reg = ((rr >> 3) << 1) | (tt & 1);
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kNC; ++w) v += rb[(w * 32 + src_lane) * 4 + reg];
      if (complete) {
        sm.tv[tid] = v;
      } else {
        const int qs = (t == static_cast<int>(u0 / S)) ? 0 : 1;
        __stcg(a.tile_part + (static_cast<size_t>(b) * 2 + qs) * 128 + tid, v);
        __threadfence();
      }
    }
    named_bar_sync(1, kNC * 32);
    if (!complete) {
      const int b0 = unit_owner(tu0, U, G), b1 = unit_owner(tu1, U, G);
      if (tid == 0) {
        __threadfence();
        const int prev = atomicAdd(a.tile_cnt + t, 1);
        sm.flag[0] = prev == b1 - b0;
      }
      named_bar_sync(1, kNC * 32);
      if (!sm.flag[0]) continue;  // another CTA finishes this tile
      __threadfence();
      if (tid < 128) {
        float v = 0.f;
        for (int q = b0; q <= b1; ++q) {
          const int qs = (t == static_cast<int>(unit_lo(U, q, G) / S)) ? 0 : 1;
          v += __ldcg(a.tile_part + (static_cast<size_t>(q) * 2 + qs) * 128 + tid);
        }
        sm.tv[tid] = v;
      }
      if (tid == 0) a.tile_cnt[t] = 0;
      named_bar_sync(1, kNC * 32);
    }
    tile_epilogue<Act>(op, a.M, t, sm, pre_a, pre_b, pre_o);
  }

  if (op.epi == kEpiArgmax) {
    // CTA best -> global keys; the last CTA decodes, resets and (device loop)
    // feeds the token back and advances the position.
    named_bar_sync(1, kNC * 32);
    if (tid < a.M) atomicMax(&a.amax_key[tid], sm.skey[tid]);
    __threadfence();
    named_bar_sync(1, kNC * 32);
    if (tid == 0) {
      const int prev = atomicAdd(a.amax_count, 1);
      sm.flag[0] = prev == G - 1;
    }
    named_bar_sync(1, kNC * 32);
    if (sm.flag[0]) {
      __threadfence();
      if (tid < a.M) {
        const unsigned long long key = atomicExch(&a.amax_key[tid], 0ull);
        const int32_t id = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key));
        a.tok_out[tid] = id;
        if (a.tok_loop) a.tok_loop[tid] = id;
        if (a.pos_loop) a.pos_loop[tid] += 1;
      }
      if (tid == 0) atomicExch(a.amax_count, 0);
    }
  }
}

// ------------------------------------------------------------------ kernel
template <typename Act, int NREP>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const StepArgs a, const StepPlan p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Smem sm;
  sm.ring = smem;
  sm.xs = smem + p.x_off;
  sm.red = reinterpret_cast<float*>(smem + p.red_off);
  sm.tv = reinterpret_cast<float*>(smem + p.tv_off);
  sm.xexp = reinterpret_cast<int*>(smem + p.misc_off);
  sm.scratch = reinterpret_cast<float*>(smem + p.misc_off + 64);
  sm.flag = reinterpret_cast<int*>(smem + p.misc_off + 128);
  sm.skey = reinterpret_cast<unsigned long long*>(smem + p.misc_off + 192);
  sm.attn = reinterpret_cast<AttnItemSmem*>(smem + p.attn_off);
  sm.full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  sm.empty = sm.full + kMaxSlots;
  sm.xbar = sm.empty + kMaxSlots;
  const int NS = p.slots;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kNC);
    }
    mbar_init(sm.xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if ((threadIdx.x >> 5) == kNC) {
    if ((threadIdx.x & 31) == 0) producer(a, sm, NS);
    return;
  }

  const unsigned G = gridDim.x;
  int slot = 0, parity = 0;
  uint32_t round = 0, xphase = 0;
  bool ok = true;
  for (int k = 0; k < a.n_ops; ++k) {
    if (k > 0 && !grid_wait(a, G * static_cast<unsigned>(k), sm)) break;
    const StepOp& op = a.ops[k];
    if (a.trace && threadIdx.x == 0) atomicMax(a.trace + k * kTraceFields, global_ns());
    if (op.kind == kOpEmbed) {
      embed_op(a);
    } else if (op.kind == kOpAttn) {
      attn_op<Act, NREP>(op, a.M, sm);
    } else {
      gemv_op<Act>(a, op, k, sm, p, slot, round, parity, ok, xphase);
    }
    if (a.trace) {
      named_bar_sync(1, kNC * 32);
      if (threadIdx.x == 0) {
        const unsigned long long t = global_ns();
        atomicMax(a.trace + k * kTraceFields + 2, t);
        atomicMax(a.trace + k * kTraceFields + 3, kTraceBig - t);
      }
    }
    grid_arrive(a);
  }
}

template <typename Act, int NREP>
cudaError_t launch_t(const StepArgs& a, const StepPlan& p, int grid, cudaStream_t s) {
  auto kern = step_kernel<Act, NREP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.total);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, p);
}

template <typename Act>
cudaError_t launch_act(const StepArgs& a, const StepPlan& p, int nrep, int grid, cudaStream_t s) {
  switch (nrep) {
    case 1: return launch_t<Act, 1>(a, p, grid, s);
    case 2: return launch_t<Act, 2>(a, p, grid, s);
    case 4: return launch_t<Act, 4>(a, p, grid, s);
    case 5: return launch_t<Act, 5>(a, p, grid, s);
    case 8: return launch_t<Act, 8>(a, p, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

StepPlan step_plan(int k_pad_max, int rows) {
  StepPlan p{};
  p.xs_stride = k_pad_max + 8;
  const int x_bytes = (rows * p.xs_stride * 2 + 127) / 128 * 128;
  const int red_bytes = 2 * kNC * 128 * 4;
  const int tv_bytes = 128 * 4;
  const int misc_bytes = 256;
  const int attn_bytes = (kNC * static_cast<int>(sizeof(AttnItemSmem)) + 127) / 128 * 128;
  const int bar_bytes = (2 * kMaxSlots + 1) * 8;
  const int fixed = x_bytes + red_bytes + tv_bytes + misc_bytes + attn_bytes + bar_bytes + 1024;
  int slots = (kSmemBudget - fixed) / kStageBytes;
  if (slots > kMaxSlots) slots = kMaxSlots;
  p.slots = slots;
  p.x_off = slots * kStageBytes;
  p.red_off = p.x_off + x_bytes;
  p.tv_off = p.red_off + red_bytes;
  p.misc_off = p.tv_off + tv_bytes;
  p.attn_off = p.misc_off + misc_bytes;
  p.bar_off = p.attn_off + attn_bytes;
  p.total = p.bar_off + bar_bytes;
  return p;
}

cudaError_t step_launch(const StepArgs& a, const StepPlan& p, int act, int nrep, int grid,
                        cudaStream_t s) {
  if (a.M < 1 || a.M > kStepMaxM || p.slots < 2 || grid < 1) return cudaErrorInvalidValue;
  return act == 0 ? launch_act<__nv_bfloat16>(a, p, nrep, grid, s)
                  : launch_act<__half>(a, p, nrep, grid, s);
}

}  // namespace dialb200
