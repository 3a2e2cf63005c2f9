// Decode attention for steps of many rows on the tensor cores (mma.sync).
//
// Same contract and reference path as the split-KV kernels of attention.cu
// (dial-core/src/models/qwen3_vl/text.rs:1258-1281 grouped decode attention,
// q/k norm 1466-1467, RoPE 1143-1153, KV append llama3/cache.rs:169-237).
// The CUDA-core forms spend most of their instructions on per-element dot
// products, shuffles and conversions (about 5 bytes of K/V per warp
// instruction, so they cannot reach HBM bandwidth).  Here one CTA of 4 warps
// takes item (row, kv head, split); each warp owns every 4th page of the span
// and streams it through its own shared-memory ring (TMA 2-D copies of the K
// and V halves, 128-byte swizzle), then per 16-token page:
//   S   = Q (group's query heads as rows 0..NREP-1) . K^T   16 mma (ldmatrix)
//   P   = exp(act(act(S) * act(1/sqrt d)) - m) with the running row max m
//   O  += P . V  with P split into act(P) + act(P - act(P)) (two MMAs keep
//         the f32 probabilities of the CUDA-core forms to ~16 bits)
// The 4 warps' (m, l, O) are merged in shared memory; with more than one
// split the last CTA of (row, kv head) combines the partials.  The new token's
// K/V (normed + rotated k, raw v) replace its row in the landed page before
// the MMAs and reach the global page last.
#include <cuda.h>

#include <cmath>
#include <type_traits>

#include "attention.h"
#include "attn_dev.cuh"
#include "common.cuh"

namespace dialb200 {
namespace {

constexpr int kMW = 4;                                // warps per CTA
constexpr int kHalfBytes = kPageTokens * 128;         // 16 rows x 64 dims x 2 B
constexpr int kSlotBytes = 4 * kHalfBytes;            // K lo | K hi | V lo | V hi
constexpr int kQStride = kHeadDim + 8;  // padded query rows: conflict-free fragment loads
constexpr int kMiscBytes = 4096;

struct PageMaps {
  CUtensorMap k, v;
};

// misc area: q rows, fresh k|v, ring barriers, per-warp (m, l), combine flag
static_assert(8 * kQStride * 2 + 2 * kHeadDim * 2 + kMW * 4 * 8 + kMW * 8 * 2 * 4 + 4 <= kMiscBytes,
              "misc area");

template <int RING>
constexpr int mma_smem_bytes() {
  static_assert(RING * kSlotBytes * kMW >= (kMW * 8 * kHeadDim + 8 * 32 * 2) * 4,
                "the idle rings hold the merge buffers");
  return 1024 + kMW * RING * kSlotBytes + kMiscBytes;
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y,
                                       uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D(rows 0-7) += A(rows 0-7) . B for m16n8k16 with rows 8-15 of A zero:
// only c0 / c1 (row g) are kept; rows 8-15 of D go to dead registers.
template <typename Act>
__device__ __forceinline__ void mma_rows8(float& d0, float& d1, uint32_t a0, uint32_t a2,
                                          uint32_t b0, uint32_t b1) {
  float x2, x3;
  if constexpr (std::is_same<Act, __nv_bfloat16>::value) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, {%0,%1,%9,%9};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.f));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, {%0,%1,%9,%9};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.f));
  }
}

// (x0, x1) -> packed act pair hi = act(x), lo = act(x - hi)
template <typename Act>
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  using AT = ActTraits<Act>;
  Act h[2] = {AT::from_f(x0), AT::from_f(x1)};
  Act l[2] = {AT::from_f(x0 - AT::to_f(h[0])), AT::from_f(x1 - AT::to_f(h[1]))};
  hi = *reinterpret_cast<const uint32_t*>(h);
  lo = *reinterpret_cast<const uint32_t*>(l);
}

// Byte offset of (row r, 16-byte unit u) inside one 16 x 128-byte half page
// written by a 128-byte-swizzled TMA copy.
__device__ __forceinline__ uint32_t sw_off(int r, int u) {
  return static_cast<uint32_t>(r * 128 + ((u ^ (r & 7)) << 4));
}

template <int RING>
constexpr int mma_min_ctas() {  // CTAs per SM that the ring's shared memory allows
  return RING <= 2 ? 3 : RING == 3 ? 2 : 1;
}

template <typename Act, int NREP, int RING>
__global__ void __launch_bounds__(kMW * 32, mma_min_ctas<RING>()) attn_decode_mma_kernel(
    const __grid_constant__ PageMaps maps, const AttnDecodeArgs a) {
  static_assert(NREP >= 1 && NREP <= 8, "query heads per kv head: rows 0..7 of the MMA");
  using AT = ActTraits<Act>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* misc = smem + kMW * RING * kSlotBytes;
  Act* qs = reinterpret_cast<Act*>(misc);                 // [8][kQStride], rows >= NREP zero
  Act* kvs = qs + 8 * kQStride;                           // fresh k | v [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(kvs + 2 * kHeadDim);  // [kMW][RING]
  float* mls = reinterpret_cast<float*>(bars + kMW * RING);          // [kMW][8][2]
  int* flag = reinterpret_cast<int*>(mls + kMW * 8 * 2);
  // once every ring is idle: the warps' partials [kMW][NREP][128] and the
  // combine's (m, l) of every split [NREP][32][2]
  float* ow = reinterpret_cast<float*>(ring);
  float* mlc = reinterpret_cast<float*>(ring + kMW * 8 * kHeadDim * 4);

  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int QH = a.sh.q_heads, KVH = a.sh.kv_heads;
  const bool early = a.rows_ready != 0;
  if (!early) pdl_wait();

  const int sid = a.sid[m];
  int pos = a.pos[m];
  const bool bad = pos < 0 || pos >= a.sh.max_pos || pos / kPageTokens >= a.sh.max_blocks;
  if (bad) {
    if (threadIdx.x == 0) set_status(a.status, kStatusBadArgs);
    pos = 0;
  }
  const int ctx = pos + 1;
  const int S = active_splits(ctx, a.splits, a.min_split_tokens);
  if (split >= S) return;
  const int span = ((ctx + S - 1) / S + kPageTokens - 1) / kPageTokens * kPageTokens;
  const int tok0 = split * span;
  const int tok1 = min(ctx, tok0 + span);
  const bool owner = tok0 <= pos && pos < tok1;
  const bool fresh = owner && !bad;
  const int pg_first = tok0 / kPageTokens;
  const int npg = tok1 > tok0 ? (tok1 - tok0 + kPageTokens - 1) / kPageTokens : 0;
  const int mine = npg > warp ? (npg - warp + kMW - 1) / kMW : 0;  // this warp's pages
  const int32_t* bt = a.block_table + static_cast<size_t>(sid) * a.sh.max_blocks;

  uint64_t* full = bars + warp * RING;
  uint8_t* wring = ring + warp * RING * kSlotBytes;
  if (lane == 0) {
    for (int i = 0; i < RING; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // lane l holds the block id of this warp's page (32 * window + l)
  int bt_lane = lane < mine ? checked_block(a, bt[pg_first + warp + kMW * lane]) : 0;
  auto issue = [&](int i) {  // warp-uniform i
    if (i > 0 && (i & 31) == 0)
      bt_lane = i + lane < mine ? checked_block(a, bt[pg_first + warp + kMW * (i + lane)]) : 0;
    const int blk = __shfl_sync(0xffffffffu, bt_lane, i & 31);
    if (lane == 0) {
      uint8_t* dst = wring + (i % RING) * kSlotBytes;
      uint64_t* bar = &full[i % RING];
      mbar_arrive_expect_tx(bar, kSlotBytes);
      const int y = (blk * KVH + kvh) * kPageTokens;
      tma_2d(dst, &maps.k, 0, y, bar);
      tma_2d(dst + kHalfBytes, &maps.k, 64, y, bar);
      tma_2d(dst + 2 * kHalfBytes, &maps.v, 0, y, bar);
      tma_2d(dst + 3 * kHalfBytes, &maps.v, 64, y, bar);
    }
  };
  int issued = 0;
  for (; issued < RING && issued < mine; ++issued) issue(issued);
  const int blk_pos = fresh && warp == 0 ? checked_block(a, bt[pos / kPageTokens]) : 0;

  const Act* cos_row = reinterpret_cast<const Act*>(a.cos) + static_cast<size_t>(pos) * (kHeadDim / 2);
  const Act* sin_row = reinterpret_cast<const Act*>(a.sin) + static_cast<size_t>(pos) * (kHeadDim / 2);
  float qw[4], kw[4], cs[4], sn[4];
  load4(reinterpret_cast<const Act*>(a.q_norm_w) + lane * 4, qw);
  load4(reinterpret_cast<const Act*>(a.k_norm_w) + lane * 4, kw);
  load4(cos_row + (lane & 15) * 4, cs);
  load4(sin_row + (lane & 15) * 4, sn);
  if (early) pdl_wait();

  const Act* qkv = reinterpret_cast<const Act*>(a.qkv) + static_cast<size_t>(m) * a.qkv_ld;
  for (int hh = warp; hh < NREP; hh += kMW) {
    float q[4];
    load4_cg(qkv + (kvh * NREP + hh) * kHeadDim + lane * 4, q);
    norm_rope_pre<Act>(q, qw, a.sh.eps, cs, sn, lane);
    store4(qs + hh * kQStride + lane * 4, q);  // already act values: exact
  }
  for (int e = threadIdx.x; e < (8 - NREP) * kQStride; e += kMW * 32)
    qs[NREP * kQStride + e] = AT::from_f(0.f);
  float kn[4] = {0.f, 0.f, 0.f, 0.f}, vn[4] = {0.f, 0.f, 0.f, 0.f};
  if (fresh && warp == 0) {
    load4_cg(qkv + (QH + kvh) * kHeadDim + lane * 4, kn);
    load4_cg(qkv + (QH + KVH + kvh) * kHeadDim + lane * 4, vn);
    norm_rope_pre<Act>(kn, kw, a.sh.eps, cs, sn, lane);
    store4(kvs + lane * 4, kn);
    store4(kvs + kHeadDim + lane * 4, vn);
  }
  __syncthreads();

  const int g = lane >> 2, c = lane & 3;
  const Act* qrow = qs + g * kQStride + 2 * c;  // rows NREP..7 are zero
  const float scale = AT::round(1.0f / sqrtf(static_cast<float>(kHeadDim)));
  // ldmatrix row addresses: K (plain) lane -> matrix mi: row r_k, unit +(mi & 1);
  // V (transposed) lane -> row r_v, unit +(mi >> 1)
  const int mi = lane >> 3;
  const int r_k = (lane & 7) + ((mi >> 1) << 3), uk = mi & 1;
  const int r_v = (lane & 7) + ((mi & 1) << 3), uv = mi >> 1;
  const int pos_page = fresh ? (pos - tok0) / kPageTokens : -1;

  float o[16][2];
#pragma unroll
  for (int nb = 0; nb < 16; ++nb) o[nb][0] = o[nb][1] = 0.f;
  float mrun = -INFINITY, lrun = 0.f;
  int done = 0;
  for (; done < mine; ++done) {
    const int i = done, slot = i % RING;
    uint8_t* kp = wring + slot * kSlotBytes;
    uint8_t* vp = kp + 2 * kHalfBytes;
    const bool landed = mbar_wait(&full[slot], static_cast<uint32_t>(i / RING) & 1u, a.status,
                                  kStatusAttnRing);
    if (!__all_sync(0xffffffffu, landed)) break;
    const int j = warp + kMW * i;  // page index inside the span
    if (j == pos_page) {
      // the new token's row: lanes 0-15 write K units, 16-31 V units
      const int rr = pos % kPageTokens, u = lane & 15;
      uint8_t* base = (lane < 16 ? kp : vp) + (u >> 3) * kHalfBytes + sw_off(rr, u & 7);
      *reinterpret_cast<uint4*>(base) =
          *reinterpret_cast<const uint4*>(kvs + (lane < 16 ? 0 : kHeadDim) + u * 8);
      fence_proxy_async_smem();
      __syncwarp();
    }
    // S = Q K^T for the page's 16 tokens (n-blocks: tokens 0-7, 8-15)
    // four accumulator chains (token half x k-step parity) of 4 MMAs each
    float sa[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b[4];
      ldsm_x4(smem_u32(kp + (ks >> 2) * kHalfBytes + sw_off(r_k, (ks & 3) * 2 + uk)), b);
      const uint32_t qa0 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16);
      const uint32_t qa1 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8);
      mma_rows8<Act>(sa[ks & 1][0], sa[ks & 1][1], qa0, qa1, b[0], b[1]);
      mma_rows8<Act>(sa[2 + (ks & 1)][0], sa[2 + (ks & 1)][1], qa0, qa1, b[2], b[3]);
    }
    const float s0[2] = {sa[0][0] + sa[1][0], sa[0][1] + sa[1][1]};
    const float s1[2] = {sa[2][0] + sa[3][0], sa[2][1] + sa[3][1]};
    const int tb = tok0 + kPageTokens * j;
    float sc[4] = {s0[0], s0[1], s1[0], s1[1]};
    const int tk[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      sc[q] = tb + tk[q] < tok1 ? AT::round(AT::round(sc[q]) * scale) : -INFINITY;
      mx = fmaxf(mx, sc[q]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(mrun, mx);
    const float alpha = mnew == -INFINITY ? 1.f : expf(mrun - mnew);
    float p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = sc[q] == -INFINITY ? 0.f : expf(sc[q] - mnew);
    lrun = fmaf(lrun, alpha, (p[0] + p[1]) + (p[2] + p[3]));
    mrun = mnew;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int nb = 0; nb < 16; ++nb) {
        o[nb][0] *= alpha;
        o[nb][1] *= alpha;
      }
    }
    uint32_t h0, l0, h1, l1;
    split_pair<Act>(p[0], p[1], h0, l0);
    split_pair<Act>(p[2], p[3], h1, l1);
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      uint32_t b[4];
      ldsm_x4_t(smem_u32(vp + (db >> 2) * kHalfBytes + sw_off(r_v, (db & 3) * 2 + uv)), b);
      mma_rows8<Act>(o[2 * db][0], o[2 * db][1], h0, h1, b[0], b[1]);
      mma_rows8<Act>(o[2 * db][0], o[2 * db][1], l0, l1, b[0], b[1]);
      mma_rows8<Act>(o[2 * db + 1][0], o[2 * db + 1][1], h0, h1, b[2], b[3]);
      mma_rows8<Act>(o[2 * db + 1][0], o[2 * db + 1][1], l0, l1, b[2], b[3]);
    }
    // the slot's ldmatrix reads before the TMA that refills it
    fence_proxy_async_smem();
    __syncwarp();
    if (issued < mine) issue(issued++);
  }
  if (done < mine) {
    // a copy did not land in time: wait (bounded) for the ones still in flight
    for (int i = done; i < issued; ++i)
      mbar_wait(&full[i % RING], static_cast<uint32_t>(i / RING) & 1u, a.status, kStatusAttnRing);
  }
  lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
  lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
  __syncthreads();  // every ring is idle: its bytes now hold the warps' partials
  if (g < NREP) {
#pragma unroll
    for (int nb = 0; nb < 16; ++nb)
      *reinterpret_cast<float2*>(ow + (warp * NREP + g) * kHeadDim + nb * 8 + 2 * c) =
          make_float2(o[nb][0], o[nb][1]);
    if (c == 0) {
      mls[(warp * NREP + g) * 2] = mrun;
      mls[(warp * NREP + g) * 2 + 1] = lrun;
    }
  }
  __syncthreads();

  // thread d merges dim d of every query head of the group
  const int d = threadIdx.x;
  float acc[NREP], Mh[NREP], Lh[NREP];
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMW; ++w) M = fmaxf(M, mls[(w * NREP + h) * 2]);
    float L = 0.f, v = 0.f;
#pragma unroll
    for (int w = 0; w < kMW; ++w) {
      const float mw = mls[(w * NREP + h) * 2];
      const float wt = mw == -INFINITY ? 0.f : expf(mw - M);
      L = fmaf(wt, mls[(w * NREP + h) * 2 + 1], L);
      v = fmaf(wt, ow[(w * NREP + h) * kHeadDim + d], v);
    }
    acc[h] = v;
    Mh[h] = M;
    Lh[h] = L;
  }
  Act* out = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(m) * a.out_ld +
             static_cast<size_t>(kvh) * NREP * kHeadDim + d;
  if (S == 1) {
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      const float inv = Lh[h] > 0.f ? 1.f / Lh[h] : 0.f;
      out[h * kHeadDim] = AT::from_f(acc[h] * inv);
    }
  } else {
    // partials of this split; the last CTA of (row, kv head) combines them
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      const size_t prow = (static_cast<size_t>(m) * QH + kvh * NREP + h) * a.splits;
      __stcg(a.part_o + (prow + split) * kHeadDim + d, acc[h]);
      if (d == 0) {
        __stcg(a.part_ml + (prow + split) * 2, Mh[h]);
        __stcg(a.part_ml + (prow + split) * 2 + 1, Lh[h]);
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int old = atomicAdd(a.counters + m * KVH + kvh, 1);
      *flag = old == S - 1;
    }
    __syncthreads();
    if (*flag) {
      __threadfence();
      for (int e = threadIdx.x; e < NREP * S; e += kMW * 32) {
        const int h = e / S, s2 = e % S;
        const size_t prow = (static_cast<size_t>(m) * QH + kvh * NREP + h) * a.splits;
        mlc[(h * 32 + s2) * 2] = __ldcg(a.part_ml + (prow + s2) * 2);
        mlc[(h * 32 + s2) * 2 + 1] = __ldcg(a.part_ml + (prow + s2) * 2 + 1);
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const size_t prow = (static_cast<size_t>(m) * QH + kvh * NREP + h) * a.splits;
        float M = -INFINITY;
        for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, mlc[(h * 32 + s2) * 2]);
        float L = 0.f, v = 0.f;
        for (int s2 = 0; s2 < S; ++s2) {
          const float ms = mlc[(h * 32 + s2) * 2];
          const float wt = ms == -INFINITY ? 0.f : expf(ms - M);
          L = fmaf(wt, mlc[(h * 32 + s2) * 2 + 1], L);
          v = fmaf(wt, __ldcg(a.part_o + (prow + s2) * kHeadDim + d), v);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        out[h * kHeadDim] = AT::from_f(v * inv);
      }
      if (threadIdx.x == 0) a.counters[m * KVH + kvh] = 0;
    }
  }
  // the new token's K/V reach the page last (no read in this launch needs them)
  if (fresh && warp == 0) {
    const size_t off =
        ((static_cast<size_t>(blk_pos) * KVH + kvh) * kPageTokens + (pos % kPageTokens)) *
            kHeadDim + lane * 4;
    store4(reinterpret_cast<Act*>(a.kv.k) + off, kn);
    store4(reinterpret_cast<Act*>(a.kv.v) + off, vn);
  }
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Page view of one pool: rows = num_blocks * kv_heads * 16 tokens of 128
// dims; a box is one page's 16 rows x 64 dims.
bool page_map(EncodeTiledFn enc, CUtensorMap* m, const void* base, uint64_t rows, bool bf16) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHeadDim), rows};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHeadDim) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kPageTokens)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename Act, int NREP, int RING>
cudaError_t launch_t(const PageMaps& maps, const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  auto kern = attn_decode_mma_kernel<Act, NREP, RING>;
  constexpr int smem = mma_smem_bytes<RING>();
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.sh.kv_heads, a.splits, a.M);
  cfg.blockDim = dim3(kMW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, maps, a);
}

template <typename Act, int RING>
cudaError_t launch_ring(const PageMaps& maps, const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  switch (a.sh.q_heads / a.sh.kv_heads) {
    case 1: return launch_t<Act, 1, RING>(maps, a, s, pdl);
    case 2: return launch_t<Act, 2, RING>(maps, a, s, pdl);
    case 4: return launch_t<Act, 4, RING>(maps, a, s, pdl);
    case 5: return launch_t<Act, 5, RING>(maps, a, s, pdl);
    case 8: return launch_t<Act, 8, RING>(maps, a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// Page slots per warp: 2 (3 CTAs per SM) unless the caller asks for 3 (2 CTAs).
template <typename Act>
cudaError_t launch_act(const PageMaps& maps, const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  return a.mma_ring == 3 ? launch_ring<Act, 3>(maps, a, s, pdl)
                         : launch_ring<Act, 2>(maps, a, s, pdl);
}

}  // namespace

bool attn_decode_mma_supported(const AttnDecodeArgs& a) {
  const int rep = a.sh.kv_heads > 0 ? a.sh.q_heads / a.sh.kv_heads : 0;
  return a.num_blocks > 0 && a.sh.head_dim == kHeadDim && a.sh.q_heads % a.sh.kv_heads == 0 &&
         (rep == 1 || rep == 2 || rep == 4 || rep == 5 || rep == 8) && a.splits <= 32 &&
         (reinterpret_cast<uintptr_t>(a.kv.k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.kv.v) & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t attn_decode_mma_launch(const AttnDecodeArgs& a, int act, cudaStream_t s, bool pdl) {
  if (!attn_decode_mma_supported(a)) return cudaErrorInvalidValue;
  if (a.splits > 1 && (!a.part_o || !a.part_ml || !a.counters)) return cudaErrorInvalidValue;
  EncodeTiledFn enc = encode_fn();
  PageMaps maps;
  const uint64_t rows = static_cast<uint64_t>(a.num_blocks) * a.sh.kv_heads * kPageTokens;
  if (!page_map(enc, &maps.k, a.kv.k, rows, act == 0) ||
      !page_map(enc, &maps.v, a.kv.v, rows, act == 0))
    return cudaErrorInvalidValue;
  return act == 0 ? launch_act<__nv_bfloat16>(maps, a, s, pdl)
                  : launch_act<__half>(maps, a, s, pdl);
}

}  // namespace dialb200
