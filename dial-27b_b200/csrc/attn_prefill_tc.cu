// Causal prefill attention on the 5th-generation tensor cores.
//
// Replaces grouped_prefill_attention (dial-core/src/models/qwen3_vl/text.rs:1283-1327,
// causal mask llama3/cache.rs:102-113) for prompts of >= 64 tokens: a
// flash-style pass per (128-query block, query head) over the session's paged
// KV, instead of one CUDA-core decode item per query row.
//
//  * q_rope_kernel: per-head RMSNorm + RoPE of the new queries (the decode
//    path's rounding), written as bf16 rows for TMA; the new K/V are appended
//    to the pages beforehand by the existing kv_append kernel.
//  * attn_tc_kernel (192 threads): warp 4 loads Q once and, per 128-key
//    block, the 8 K and 8 V pages of the kv head with 2-D TMA (128-byte
//    swizzle) into a double buffer; warp 5 issues tcgen05.mma kind::f16:
//    S = Q K^T (M=128 queries, N=128 keys, K=128 dims) into TMEM columns
//    [0, 128), then O += P V (K-major P from shared memory, MN-major V) into
//    TMEM columns [128, 256); warps 0-3 own one query row per thread: they
//    read S with tcgen05.ld, form scores act(act(q.k) * act(1/sqrt(d))) with
//    the causal mask, keep the running max / sum in f32, rescale the O row in
//    TMEM when the max moves, write P = exp(s - max) as bf16 into a swizzled
//    K-major tile, and finally store act(O / sum).
// Probabilities feed the tensor core as bf16 (the reference rounds its
// normalised probabilities to the activation dtype too); every mbarrier wait
// is bounded and the CTA frees its TMEM on every exit path.
#include <cuda.h>

#include "attention.h"
#include "attn_dev.cuh"
#include "common.cuh"

namespace dialb200 {
namespace {

constexpr int kQ = 128;       // queries per CTA
constexpr int kKB = 128;      // keys per block
// warps 0-3 and 6-9: softmax (two per 32-row TMEM lane quarter, one per
// 64-key half of each block); warp 4: loads; warp 5: MMA
constexpr int kThreads = 320;
constexpr int TILE = 128 * 128 * 2;     // one 128 x 128 bf16 tile (two 64-column halves)
constexpr int HALF = 128 * 64 * 2;      // one 64-column half: [128 rows][128 B]
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE;           // [2] key tiles
constexpr int OFF_V = OFF_K + 2 * TILE;       // [2] value tiles
constexpr int OFF_P = OFF_V + 2 * TILE;       // probabilities
constexpr int OFF_XCH = OFF_P + TILE;        // row max exchange [2 parities][2 halves][128]
constexpr int OFF_BAR = OFF_XCH + 2 * 2 * 128 * 4;
// qbar, kfull[2], kfree[2], vfull[2], vfree[2], sbar[2], pready, obar, fin
constexpr int NBAR = 14;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;
// S double-buffered in [0,128) and [128,256), O in [256,384): Q K^T of block
// j+1 runs on the tensor core while the softmax warps work on block j
constexpr int kTmemCols = 512;
constexpr int kStatusAttnTc = 0x501;

// f32 accumulator, bf16 A and B, K-major A; B K-major (S = Q K^T) or
// MN-major (O += P V); M = N = 128.
constexpr uint32_t idesc(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

// K-major operand with 128-byte rows, 128-byte swizzle, 8-row groups 1 KB apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// MN-major operand (V: keys x dims with dims contiguous): 64-element halves
// 16 KB apart (leading byte offset), 8-key groups 1 KB apart (stride offset).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(HALF >> 4) << 16) |
         (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t id,
                                    uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tcgen05.ld of 16 columns without the wait: several loads share one wait
__device__ __forceinline__ void ld16_async(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// (lo, hi) f32 -> bf16x2, round to nearest even
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// bf16x2 product, rounded once to bf16: the exact product of two bf16 values
// fits an f32, so this equals round(round(a) * b) formed in f32
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ void st16_async(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]));
}

// ------------------------------------------------------------ q rotation
// Query head h of token t: RMSNorm + RoPE (bf16 rounding) -> q_rot[t][h*128].
__global__ void __launch_bounds__(256) q_rope_kernel(const AttnPrefillArgs a) {
  using Act = __nv_bfloat16;
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = a.p0 + t;
  if (pos < 0 || pos >= a.sh.max_pos) return;  // kv_append records the bad position
  const Act* qkv = reinterpret_cast<const Act*>(a.qkv) + static_cast<size_t>(t) * a.qkv_ld;
  const Act* cos_row = reinterpret_cast<const Act*>(a.cos) + static_cast<size_t>(pos) * (kHeadDim / 2);
  const Act* sin_row = reinterpret_cast<const Act*>(a.sin) + static_cast<size_t>(pos) * (kHeadDim / 2);
  Act* out = reinterpret_cast<Act*>(a.q_rot) + static_cast<size_t>(t) * a.sh.q_heads * kHeadDim;
  for (int h = warp; h < a.sh.q_heads; h += 8) {
    float q[4];
    load4(qkv + h * kHeadDim + lane * 4, q);
    norm_rope<Act>(q, reinterpret_cast<const Act*>(a.q_norm_w), a.sh.eps, cos_row, sin_row, lane);
    store4(out + h * kHeadDim + lane * 4, q);
  }
}

// ------------------------------------------------------------ attention
struct TcMaps {
  CUtensorMap q, k, v;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ TcMaps maps, const AttnPrefillArgs a, int nrep) {
  using AT = ActTraits<__nv_bfloat16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* qbar = bars;
  uint64_t* kfull = bars + 1;   // [2] key tile landed
  uint64_t* kfree = bars + 3;   // [2] key tile read by Q K^T
  uint64_t* vfull = bars + 5;   // [2] value tile landed
  uint64_t* vfree = bars + 7;   // [2] value tile read by P V
  uint64_t* sbar = bars + 9;    // [2] S buffer of block j written
  uint64_t* pready = bars + 11;
  uint64_t* obar = bars + 12;
  uint64_t* fin = bars + 13;  // the MMA thread's own "all my MMAs are done"
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the causally longest query blocks first: the short ones fill the tail
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kQ;  // first query row of the CTA
  const int h = blockIdx.y, kvh = h / nrep;
  const int KVH = a.sh.kv_heads;
  // keys [0, last] are visible to some query of the block
  const int last_q = min(q0 + kQ - 1, a.M - 1);
  const int last_key = a.p0 + last_q;
  const int nkb = last_key / kKB + 1;

  if (tid == 0) {
    mbar_init(qbar, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&kfull[b], 1);
      mbar_init(&kfree[b], 1);
      mbar_init(&vfull[b], 1);
      mbar_init(&vfree[b], 1);
      mbar_init(&sbar[b], 1);
    }
    mbar_init(pready, 2 * kQ);  // every softmax thread of both halves
    mbar_init(obar, 1);
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;  // S of block j: tmem + (j & 1) * 128

  if (warp == 4) {
    // ------------------------------------------------------------ loads
    if (lane == 0) {
      mbar_arrive_expect_tx(qbar, TILE);
      tma2d(smem + OFF_Q, &maps.q, h * kHeadDim, q0, qbar);
      tma2d(smem + OFF_Q + HALF, &maps.q, h * kHeadDim + 64, q0, qbar);
      // K of block j as soon as Q K^T of block j-2 has read its buffer, V as
      // soon as P V of block j-2 has
      for (int j = 0; j < nkb; ++j) {
        const int b = j & 1;
        int rows[kKB / kPageTokens];
#pragma unroll
        for (int pg = 0; pg < kKB / kPageTokens; ++pg) {
          const int page = min(j * (kKB / kPageTokens) + pg, a.sh.max_blocks - 1);
          rows[pg] = (checked_block(a, a.block_table[page]) * KVH + kvh) * kPageTokens;
        }
        if (j >= 2 && !mbar_wait(&kfree[b], static_cast<uint32_t>(j / 2 - 1) & 1u, a.status,
                                 kStatusAttnTc))
          break;
        mbar_arrive_expect_tx(&kfull[b], TILE);
#pragma unroll
        for (int pg = 0; pg < kKB / kPageTokens; ++pg) {
          uint8_t* kt = smem + OFF_K + b * TILE + pg * 2048;
          tma2d(kt, &maps.k, 0, rows[pg], &kfull[b]);
          tma2d(kt + HALF, &maps.k, 64, rows[pg], &kfull[b]);
        }
        if (j >= 2 && !mbar_wait(&vfree[b], static_cast<uint32_t>(j / 2 - 1) & 1u, a.status,
                                 kStatusAttnTc))
          break;
        mbar_arrive_expect_tx(&vfull[b], TILE);
#pragma unroll
        for (int pg = 0; pg < kKB / kPageTokens; ++pg) {
          uint8_t* vt = smem + OFF_V + b * TILE + pg * 2048;
          tma2d(vt, &maps.v, 0, rows[pg], &vfull[b]);
          tma2d(vt + HALF, &maps.v, 64, rows[pg], &vfull[b]);
        }
      }
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t sq = smem_u32(smem + OFF_Q), sp = smem_u32(smem + OFF_P);
      bool ok = mbar_wait(qbar, 0, a.status, kStatusAttnTc);
      auto issue_s = [&](int jj) {
        // S[jj & 1] = Q K^T over 128 dims: 8 steps of 16
        const uint32_t sk = smem_u32(smem + OFF_K + (jj & 1) * TILE);
        const uint32_t ts = tmem + static_cast<uint32_t>(jj & 1) * 128;
#pragma unroll
        for (int k16 = 0; k16 < kHeadDim / 16; ++k16) {
          const uint32_t off = (k16 >> 2) * HALF + (k16 & 3) * 32;
          mma(ts, kmajor_desc(sq + off), kmajor_desc(sk + off), idesc(false), k16 > 0 ? 1u : 0u);
        }
        commit(&kfree[jj & 1]);
        commit(&sbar[jj & 1]);
      };
      auto issue_pv = [&](int jj) {
        // O += P V over 128 keys: 8 steps of 16 keys
        const uint32_t sv = smem_u32(smem + OFF_V + (jj & 1) * TILE);
#pragma unroll
        for (int k16 = 0; k16 < kKB / 16; ++k16) {
          const uint32_t pa = sp + (k16 >> 2) * HALF + (k16 & 3) * 32;
          mma(tO, kmajor_desc(pa), mnmajor_desc(sv + k16 * 2048), idesc(true),
              (jj > 0 || k16 > 0) ? 1u : 0u);
        }
        commit(&vfree[jj & 1]);
        commit(obar);
      };
      if (ok && mbar_wait(&kfull[0], 0, a.status, kStatusAttnTc)) {
        fence_after();
        issue_s(0);
      } else {
        ok = false;
      }
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb) {
          // Q K^T of block j+1 overlaps the softmax of block j: its S buffer
          // was last read by the softmax of block j-1 (waited for below)
          if (!mbar_wait(&kfull[(j + 1) & 1], static_cast<uint32_t>((j + 1) / 2) & 1u, a.status,
                         kStatusAttnTc)) {
            ok = false;
            break;
          }
          fence_after();
          issue_s(j + 1);
        }
        // the softmax of block j has read S, written P and rescaled O
        if (!mbar_wait(pready, static_cast<uint32_t>(j) & 1u, a.status, kStatusAttnTc) ||
            !mbar_wait(&vfull[j & 1], static_cast<uint32_t>(j / 2) & 1u, a.status,
                       kStatusAttnTc)) {
          ok = false;
          break;
        }
        fence_after();
        issue_pv(j);
      }
      // nothing may still write TMEM when it is freed (a barrier of its own:
      // an extra phase on obar could run ahead of the softmax warps' waits)
      commit(fin);
      mbar_wait(fin, 0, a.status, kStatusAttnTc);
    }
  } else {
    // ---------------------------------------------- softmax + epilogue
    // two warps per 32 query rows (the TMEM lane quarter warp % 4 they may
    // read): half 0 takes keys / output dims 0-63 of every block, half 1 64-127
    const int quarter = warp & 3, half = warp >= 6 ? 1 : 0;
    const int r = quarter * 32 + lane;  // query row of the block = TMEM lane
    const int qi = q0 + r;
    const int qpos = a.p0 + qi;
    const float scale = AT::round(1.0f / sqrtf(static_cast<float>(kHeadDim)));
    const uint32_t scale2 = pack_bf16x2(scale, scale);
    constexpr uint32_t kBf16NegInf = 0xFF80u;
    const uint32_t lane_off = static_cast<uint32_t>(32 * quarter) << 16;
    float* xch = reinterpret_cast<float*>(smem + OFF_XCH);  // [parity][half][row]
    auto pair_sync = [&]() { named_bar_sync(1 + quarter, 64); };
    float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
    bool ok = true;
    int exchanged = 0;  // pair barriers passed; both warps of a pair pass nkb + 1
    for (int j = 0; j < nkb; ++j) {
      const bool okw = __all_sync(
          0xffffffffu, ok && mbar_wait(&sbar[j & 1], static_cast<uint32_t>(j / 2) & 1u, a.status,
                                       kStatusAttnTc));
      if (!okw) {
        ok = false;
        break;
      }
      fence_after();
      constexpr int KH = kKB / 2;  // keys of this half
      // scores of this row's half block as bf16 pairs (key 2i low, 2i+1 high)
      uint32_t sp[KH / 2];
      {
        uint32_t v[KH];
#pragma unroll
        for (int cb = 0; cb < KH / 16; ++cb)
          ld16_async(tmem + static_cast<uint32_t>(j & 1) * 128 + lane_off + half * KH + cb * 16,
                     v + cb * 16);
        ld_wait();
        const int kbase = j * kKB + half * KH;
        // every key of this half block visible to every row of the warp
        const bool open = kbase + KH - 1 <= a.p0 + q0 + quarter * 32 &&
                          q0 + quarter * 32 + 32 <= a.M;
        if (open) {
#pragma unroll
          for (int i = 0; i < KH / 2; ++i)
            sp[i] = mul_bf16x2(pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                               scale2);
        } else {
#pragma unroll
          for (int i = 0; i < KH / 2; ++i) {
            const uint32_t b = mul_bf16x2(
                pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), scale2);
            const bool row_ok = qi < a.M;
            const uint32_t lo = (row_ok && kbase + 2 * i <= qpos) ? (b & 0xFFFFu) : kBf16NegInf;
            const uint32_t hi = (row_ok && kbase + 2 * i + 1 <= qpos) ? (b >> 16) : kBf16NegInf;
            sp[i] = lo | (hi << 16);
          }
        }
      }
      uint32_t bm2 = sp[0];
#pragma unroll
      for (int i = 1; i < KH / 2; ++i) bm2 = max_bf16x2(bm2, sp[i]);
      float bm = fmaxf(__uint_as_float(bm2 << 16), __uint_as_float(bm2 & 0xFFFF0000u));
      // the row's block max: exchange with the other half (buffers by block
      // parity: a warp cannot be two blocks ahead of its partner)
      float* xj = xch + (j & 1) * 256;
      xj[half * 128 + r] = bm;
      pair_sync();
      ++exchanged;
      bm = fmaxf(bm, xj[(half ^ 1) * 128 + r]);
      const float m_new = fmaxf(m_run, bm);
      // exponentials through the hardware exp2: its relative error (about
      // 1e-6 here) is far below the bf16 rounding P receives
      const float alpha = (m_run == -INFINITY) ? 0.f : __expf(m_run - m_new);
      // p = exp(s - m) and the row sum in key order, as the f32 form computed
      // them (the packed scores change no value); a fully masked row
      // (m = -inf) gets p = 0
      const bool dead = m_new == -INFINITY;
      float psum = 0.f;
      uint32_t pp[KH / 2];
#pragma unroll
      for (int i = 0; i < KH / 2; ++i) {
        const float p0 = dead ? 0.f : __expf(__uint_as_float(sp[i] << 16) - m_new);
        const float p1 = dead ? 0.f : __expf(__uint_as_float(sp[i] & 0xFFFF0000u) - m_new);
        psum += p0;
        psum += p1;
        pp[i] = pack_bf16x2(p0, p1);
      }
      l_run = l_run * alpha + psum;
      m_run = m_new;
      if (j > 0) {
        // P V of block j-1 must be in O (and done reading P) before O is
        // rescaled and P rewritten
        const bool okp = __all_sync(
            0xffffffffu, mbar_wait(obar, static_cast<uint32_t>(j - 1) & 1u, a.status, kStatusAttnTc));
        if (!okp) {
          ok = false;
          break;
        }
        fence_after();
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
        // rescales its 32 rows, or none does when no row's max moved (alpha 1)
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t v[kHeadDim / 2];  // this half's 64 dims: four loads, one wait
          const uint32_t col = tO + lane_off + half * (kHeadDim / 2);
#pragma unroll
          for (int cb = 0; cb < kHeadDim / 32; ++cb) ld16_async(col + cb * 16, v + cb * 16);
          ld_wait();
#pragma unroll
          for (int e = 0; e < kHeadDim / 2; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
#pragma unroll
          for (int cb = 0; cb < kHeadDim / 32; ++cb) st16_async(col + cb * 16, v + cb * 16);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
      }
      // P row r as bf16 into the K-major swizzled tile: 16-byte chunk c holds keys 8c..8c+7
      uint8_t* prow = smem + OFF_P + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int jj = 0; jj < KH / 8; ++jj)  // this half's 8 chunks of 8 keys
        *reinterpret_cast<uint4*>(prow + half * HALF + ((jj ^ (r & 7)) << 4)) =
            make_uint4(pp[4 * jj], pp[4 * jj + 1], pp[4 * jj + 2], pp[4 * jj + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      mbar_arrive(pready);
    }
    // a warp that left the loop on a failed wait still meets its partner at
    // every exchange (the status word already holds the error)
    for (; exchanged < nkb; ++exchanged) pair_sync();
    // row sum = both halves' shares (same running max sequence)
    float* xl = xch + (nkb & 1) * 256;
    xl[half * 128 + r] = l_run;
    pair_sync();
    const float l_tot = l_run + xl[(half ^ 1) * 128 + r];
    if (ok) {
      const bool okw =
          __all_sync(0xffffffffu, mbar_wait(obar, static_cast<uint32_t>(nkb - 1) & 1u, a.status,
                                            kStatusAttnTc));
      if (okw) {
        fence_after();
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out) +
                              static_cast<size_t>(qi) * a.out_ld + h * kHeadDim +
                              half * (kHeadDim / 2);
#pragma unroll
        for (int cb = 0; cb < kHeadDim / 32; ++cb) {
          uint32_t v[16];
          ld16(tO + lane_off + half * (kHeadDim / 2) + cb * 16, v);
          if (qi < a.M) {
            uint4 o[2];
            __nv_bfloat16* hv = reinterpret_cast<__nv_bfloat16*>(o);
#pragma unroll
            for (int e = 0; e < 16; ++e) hv[e] = __float2bfloat16_rn(__uint_as_float(v[e]) * inv);
            *reinterpret_cast<uint4*>(orow + cb * 16) = o[0];
            *reinterpret_cast<uint4*>(orow + cb * 16 + 8) = o[1];
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 5)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
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

bool make_map(EncodeTiledFn enc, CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
              uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attn_prefill_tc_supported(const AttnPrefillArgs& a, int act) {
  const int rep = a.sh.q_heads / a.sh.kv_heads;
  return act == 0 && a.q_rot && a.num_blocks > 0 && a.M >= 64 && a.sh.head_dim == kHeadDim &&
         a.sh.q_heads % a.sh.kv_heads == 0 && rep >= 1 && a.out_ld % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.q_rot) & 15) == 0;
}

// After kv_append: rotate the queries, then the tensor-core attention.
cudaError_t attn_prefill_tc_launch(const AttnPrefillArgs& a, cudaStream_t s) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  q_rope_kernel<<<a.M, 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  TcMaps maps;
  const uint64_t pool_rows = static_cast<uint64_t>(a.num_blocks) * a.sh.kv_heads * kPageTokens;
  if (!make_map(enc, &maps.q, a.q_rot, static_cast<uint64_t>(a.sh.q_heads) * kHeadDim, a.M, kQ) ||
      !make_map(enc, &maps.k, a.kv.k, kHeadDim, pool_rows, kPageTokens) ||
      !make_map(enc, &maps.v, a.kv.v, kHeadDim, pool_rows, kPageTokens))
    return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.M + kQ - 1) / kQ, a.sh.q_heads);
  attn_tc_kernel<<<grid, kThreads, SMEM_BYTES, s>>>(maps, a, a.sh.q_heads / a.sh.kv_heads);
  return cudaGetLastError();
}

}  // namespace dialb200
