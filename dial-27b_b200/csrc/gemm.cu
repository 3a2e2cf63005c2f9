// Prefill W8A16 / FP8 linear (M >= 64 tokens) on the 5th-generation tensor cores.
//
// Replaces the reference's prefill kernel dial_w8a16_prefill_f16
// (dial-core/src/models/qwen3_vl/worker_w8a16.rs:186-224, a 16x16 shared-memory
// FMA tile) with a tcgen05 GEMM: y[m, n] = s[n] * sum_k q[n, k] * x[m, k].
//
// Two kernels per linear:
//  * prep: one CTA per token row stages x as f16 (RMSNorm fused when the
//    linear has one, same rounding as the decode path) with a power-of-two
//    pre-scale per row, into a scratch matrix read by TMA;
//  * gemm: one CTA per 256 output rows x 256 tokens (128 x 128 when the grid
//    would not cover the SMs).  Warp 0 streams the
//    int8 weight chunks (1-D bulk copies) and the f16 activation tile (2-D
//    TMA, 128-byte swizzle) into a 3-5 stage ring; warps 4-11 turn the int8
//    bytes into f16 (exact: PRMT into the 0x6400 exponent + HSUB2; e4m3 codes
//    by the hardware cvt, times the 128x128 block scale when there is one) written in
//    the same 128-byte-swizzled K-major layout (2-4 stage ring); warp 1 issues
//    tcgen05.mma.kind::f16 (two M=128 halves sharing the activation tile,
//    N=256, K=16, f32 accumulate in TMEM) and frees each stage with
//    tcgen05.commit; warps 4-11 read the accumulators
//    back with tcgen05.ld and apply the row scale, the row pre-scale and the
//    epilogue (store, residual add, SiLU(gate)*up).
// All mbarrier waits are bounded: on expiry a status code is recorded and the
// CTA drains its copies, waits for its MMAs, frees its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "gemm.h"
#include "gemv.h"
#include "gemv_dev.cuh"

namespace dialb200 {
namespace {

constexpr int kEpiPartial = 8;  // split-K: scaled f32 partial sums into GemmArgs::part
constexpr int kStatusGemmWait = 0x401;

// Tile configurations: 256 weight rows (two M=128 MMAs sharing the activation
// tile) x 256 tokens for large grids, 128 x 128 when that would leave SMs idle;
// K per stage is one weight chunk: 64 (int8 / e4m3) or 128 (NVFP4, 1152-byte
// chunks with their group scales).  Operand tiles are K-major with 64-column
// (128-byte) swizzle atoms: A [half][atom][128 rows][128 B], B [atom][BN][128 B].
template <int BM_, int BN_, int BK_ = 64>
struct Cfg {
  static constexpr int BM = BM_;  // weight rows per CTA
  static constexpr int BN = BN_;  // tokens per CTA: the MMA N
  static constexpr int BK = BK_;  // K per ring stage
  static constexpr int NATOM = BK / 64;
  static constexpr int CHUNK = BK == 128 ? 1152 : 1024;  // bytes per 16-row weight chunk
  // Three rings: weight bytes (RSTAGES stages of RK k-steps, one bulk copy of
  // RK contiguous chunks per 16-row tile; freed by the dequant warps), the
  // activation tiles (BSTAGES, 2-D TMA, freed by the MMAs) and the dequantized
  // weights (ASTAGES, freed by the MMAs).  Every bulk copy, TMA and tcgen05
  // instruction costs its issuing thread about 70-80 cycles (measured with
  // clock64 around them), so the per-k-step issue work is spread out: RK
  // k-steps per copy, two weight-producer threads for 256-row tiles, and two
  // MMA threads for 128-row tiles (even / odd k-steps into two accumulators,
  // added in the epilogue).
  static constexpr int RK = (BM == 128 && BK == 64) ? 4 : BM == 256 ? 1 : 2;
  static constexpr bool MMA2 = BM == 128;
  static constexpr int NPROD = BM == 256 ? 2 : 1;
  // dequant warps: 8, or 16 for 256-row tiles (twice the bytes per k-step)
  static constexpr int DQW = BM == 256 ? 16 : 8;
  static constexpr int THREADS = 128 + 32 * DQW + (MMA2 ? 32 : 0);
  static constexpr int RSTAGES = BM == 256 ? 2 : BK == 128 ? 3 : BN <= 64 ? 3 : 2;
  static constexpr int BSTAGES = BM == 256 ? 4 : BK == 128 ? 2 : BN <= 64 ? 6 : 4;
  static constexpr int ASTAGES = (BM == 256 || BK == 128) ? 2 : 4;  // dequantized-weight ring
  static_assert(!MMA2 || (BSTAGES % 2 == 0 && ASTAGES % 2 == 0),
                "two MMA threads own alternate ring slots");
  static constexpr int A_HALF = 128 * BK * 2;  // one 128-row MMA operand
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_ATOM = BN * 128;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int RAW_BYTES = (BM / 16) * CHUNK * RK;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + ASTAGES * A_BYTES;
  static constexpr int OFF_RAW = OFF_B + BSTAGES * B_BYTES;
  // barriers: wfull, wfree [RSTAGES]; bfull, bfree [BSTAGES]; aready, afree
  // [ASTAGES]; accfull
  static constexpr int OFF_BAR = (OFF_RAW + RSTAGES * RAW_BYTES + 15) / 16 * 16;
  static constexpr int OFF_TMEM =
      OFF_BAR + (2 * RSTAGES + 2 * BSTAGES + 2 * ASTAGES + 1) * 8;
  static constexpr int OFF_XEXP = OFF_TMEM + 16;
  static constexpr int SMEM_BYTES = OFF_XEXP + BN * 4 + 1024;  // + room to align to 1024
  // one BN-column accumulator per 128-row half, or per MMA thread
  static constexpr int kTmemCols = MMA2 ? 2 * BN : (BM / 128) * BN;
  // instruction descriptor: f32 accumulator, f16 A and B, both K-major, N = BN, M = 128
  static constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                     (static_cast<uint32_t>(128 >> 4) << 24);
  static_assert(SMEM_BYTES <= 232448, "shared memory plan too large");
};

// Shared-memory operand descriptor of a K-major tile with 128-byte rows and
// the 128-byte swizzle: 8-row groups 1024 bytes apart, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ prep
// Row m of x -> xh[m][0..Kp) as f16 * 2^-xexp[m] (RMSNorm first when norm_w).
// One warp per row (8 rows per CTA): a first pass over the row takes the sum
// of squares and the bound of the staged values (warp reductions only), the
// second re-reads the row (an L2 hit) and writes it converted.
constexpr int kPrepRows = 8;

template <typename Act, bool NORM>
__global__ void __launch_bounds__(kPrepRows * 32) prep_kernel(const GemmArgs a) {
  using AT = ActTraits<Act>;
  constexpr bool SCALE = std::is_same<Act, __nv_bfloat16>::value;
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * kPrepRows + (threadIdx.x >> 5);
  if (m >= a.M) return;
  const int K = a.w.K, Kp = a.w.K_pad, nv = K / 8;
  const uint4* xr =
      reinterpret_cast<const uint4*>(reinterpret_cast<const Act*>(a.x) + static_cast<size_t>(m) * a.x_ld);
  const uint4* wr = reinterpret_cast<const uint4*>(a.norm_w);
  float ss = 0.f, am = 0.f;
#pragma unroll 4
  for (int i = lane; i < nv; i += 32) {
    float xf[8], wf[8];
    unpack8<Act>(__ldcg(xr + i), xf);  // written by the previous kernel: read through L2
    if (NORM) unpack8<Act>(__ldg(wr + i), wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss = fmaf(xf[e], xf[e], ss);
      am = fmaxf(am, fabsf(NORM ? xf[e] * wf[e] : xf[e]));
    }
  }
  ss = warp_sum(ss);
  am = warp_max(am);
  float rms = 1.f;
  if (NORM) rms = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(K)) + a.eps));
  int e = 0;
  if (SCALE) {
    const float bound = NORM ? __fdiv_rn(am, rms) * 1.02f : am;
    if (bound >= 16384.f) e = ilogbf(bound) - 13;
  }
  const float sc = exp2i(-e);
  __half* orow = a.xh + static_cast<size_t>(m) * Kp;
#pragma unroll 4
  for (int i = lane; i < nv; i += 32) {
    float xf[8], wf[8];
    unpack8<Act>(__ldcg(xr + i), xf);
    if (NORM) unpack8<Act>(__ldg(wr + i), wf);
    uint4 o;
    __half* h = reinterpret_cast<__half*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float v = xf[q];
      if (NORM) {
        v = AT::round(__fdiv_rn(v, rms));
        v = AT::round(v * wf[q]);
      }
      h[q] = __float2half_rn(v * sc);
    }
    *reinterpret_cast<uint4*>(orow + static_cast<size_t>(i) * 8) = o;
  }
  for (int k = K + lane; k < Kp; k += 32) orow[k] = __float2half_rn(0.f);
  if (lane == 0) a.xexp[m] = e;
}

// The same with one CTA of 256 threads per row: more loads in flight per row
// for calls of few rows.
template <typename Act, bool NORM>
__global__ void __launch_bounds__(256) prep_row_kernel(const GemmArgs a) {
  using AT = ActTraits<Act>;
  constexpr bool SCALE = std::is_same<Act, __nv_bfloat16>::value;
  constexpr int NT = 256, VEC = 12;  // rows up to 24576 columns (27B-class down_proj: 21504)
  __shared__ float red[16];
  const int m = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.w.K, Kp = a.w.K_pad, nv = K / 8;
  const uint4* xr =
      reinterpret_cast<const uint4*>(reinterpret_cast<const Act*>(a.x) + static_cast<size_t>(m) * a.x_ld);
  const uint4* wr = reinterpret_cast<const uint4*>(a.norm_w);
  uint4 xv[VEC], wv[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int i = tid + j * NT;
    if (i < nv) {
      xv[j] = xr[i];
      if (NORM) wv[j] = wr[i];
    }
  }
  float ss = 0.f, am = 0.f;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
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
    red[warp] = ss;
    red[8 + warp] = am;
  }
  __syncthreads();
  ss = 0.f;
  am = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ss += red[i];
    am = fmaxf(am, red[8 + i]);
  }
  float rms = 1.f;
  if (NORM) rms = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(K)) + a.eps));
  int e = 0;
  if (SCALE) {
    const float bound = NORM ? __fdiv_rn(am, rms) * 1.02f : am;
    if (bound >= 16384.f) e = ilogbf(bound) - 13;
  }
  const float sc = exp2i(-e);
  __half* orow = a.xh + static_cast<size_t>(m) * Kp;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int i = tid + j * NT;
    if (i < nv) {
      float xf[8], wf[8];
      unpack8<Act>(xv[j], xf);
      if (NORM) unpack8<Act>(wv[j], wf);
      uint4 o;
      __half* h = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float v = xf[q];
        if (NORM) {
          v = AT::round(__fdiv_rn(v, rms));
          v = AT::round(v * wf[q]);
        }
        h[q] = __float2half_rn(v * sc);
      }
      *reinterpret_cast<uint4*>(orow + static_cast<size_t>(i) * 8) = o;
    }
  }
  for (int k = K + tid; k < Kp; k += NT) orow[k] = __float2half_rn(0.f);
  if (tid == 0) a.xexp[m] = e;
}

// ------------------------------------------------------------------ gemm
template <typename Act, int FMT, int EPI, int BM_, int BN_, int BK_>
__global__ void __launch_bounds__(Cfg<BM_, BN_, BK_>::THREADS, 1)
    w8a16_gemm_kernel(const __grid_constant__ CUtensorMap tmap, const GemmArgs a) {
  using AT = ActTraits<Act>;
  using G = Cfg<BM_, BN_, BK_>;
  constexpr int BM = G::BM, BN = G::BN, BK = G::BK, ASTAGES = G::ASTAGES;
  constexpr int RST = G::RSTAGES, BST = G::BSTAGES;
  constexpr int CHUNK = G::CHUNK, NATOM = G::NATOM, B_ATOM = G::B_ATOM;
  constexpr int A_BYTES = G::A_BYTES, A_HALF = G::A_HALF, B_BYTES = G::B_BYTES;
  constexpr int RAW_BYTES = G::RAW_BYTES, OFF_A = G::OFF_A, OFF_B = G::OFF_B, RK = G::RK;
  constexpr bool MMA2 = G::MMA2;
  constexpr int NPROD = G::NPROD;
  constexpr int OFF_RAW = G::OFF_RAW, OFF_BAR = G::OFF_BAR, OFF_TMEM = G::OFF_TMEM;
  constexpr int OFF_XEXP = G::OFF_XEXP, kTmemCols = G::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // weight bytes landed
  uint64_t* wfree = wfull + RST;         // weight slot read by the 8 dequant warps
  uint64_t* bfull = wfree + RST;         // activation tile landed
  uint64_t* bfree = bfull + BST;         // activation tile read by the MMAs
  uint64_t* aready = bfree + BST;        // dequantized weights written (8 warps)
  uint64_t* afree = aready + ASTAGES;    // MMAs reading them finished
  uint64_t* accfull = afree + ASTAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
  int* sxexp = reinterpret_cast<int*>(smem + OFF_XEXP);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tok0 = blockIdx.x * BN;
  const int blk = blockIdx.y;  // 256-row block = tiles [16 blk, 16 blk + 16)
  // k-steps (BK = one chunk) of this split: [KB0, KB0 + NK) of the row's C
  const int KB0 = static_cast<int>(static_cast<long long>(a.w.C) * blockIdx.z / gridDim.z);
  const int NK =
      static_cast<int>(static_cast<long long>(a.w.C) * (blockIdx.z + 1) / gridDim.z) - KB0;
  const int C = a.w.C;

  if (tid == 0) {
    for (int s = 0; s < RST; ++s) {
      mbar_init(&wfull[s], NPROD);
      mbar_init(&wfree[s], G::DQW + (a.couple ? 1 : 0));
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bfree[s], 1);
    }
    for (int s = 0; s < ASTAGES; ++s) {
      mbar_init(&aready[s], G::DQW);
      mbar_init(&afree[s], 1);
    }
    mbar_init(accfull, MMA2 ? 2 : 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid >= 128 && tid < 128 + BN) {
    const int t = tok0 + (tid - 128);
    sxexp[tid - 128] = t < a.M ? a.xexp[t] : 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || (NPROD == 2 && warp == 2)) {
    // ------------------------------------------------- weight producer(s)
    // producer p copies tiles [p T/NPROD, (p+1) T/NPROD) of the block; weight
    // stage r holds k-steps [r RK, r RK + nk)
    if (lane == 0) {
      constexpr int TPP = (BM / 16) / NPROD;  // 16-row tiles per producer
      const int c0 = (warp == 0 ? 0 : 1) * TPP;
      const int NR = (NK + RK - 1) / RK;
      int it = 0;
      for (; it < NR; ++it) {
        const int kb = KB0 + it * RK, s = it % RST, nk = min(RK, NK - it * RK);
        if (it >= RST &&
            !mbar_wait_sleep(&wfree[s], static_cast<uint32_t>(it / RST - 1) & 1u, a.status,
                       kStatusGemmWait))
          break;
        mbar_arrive_expect_tx(&wfull[s], static_cast<uint32_t>(TPP * nk * CHUNK));
        uint8_t* raw = smem + OFF_RAW + s * RAW_BYTES;
#pragma unroll
        for (int c = c0; c < c0 + TPP; ++c) {
          const size_t t = static_cast<size_t>(blk) * (BM / 16) + c;
          bulk_g2s(raw + c * RK * CHUNK, a.w.tiles + (t * C + kb) * CHUNK,
                   static_cast<uint32_t>(nk * CHUNK), &wfull[s]);
        }
      }
      // every copy issued must land before the CTA retires
      for (int j = it > RST ? it - RST : 0; j < it; ++j)
        if (!mbar_wait_sleep(&wfull[j % RST], static_cast<uint32_t>(j / RST) & 1u, a.status,
                       kStatusGemmWait))
          break;
    }
  } else if (warp == 3) {
    // ------------------------------------------------ activation producer
    if (lane == 0) {
      int it = 0;
      for (; it < NK; ++it) {
        const int kb = KB0 + it, s = it % BST;
        if (it >= BST &&
            !mbar_wait_sleep(&bfree[s], static_cast<uint32_t>(it / BST - 1) & 1u, a.status,
                       kStatusGemmWait))
          break;
        mbar_arrive_expect_tx(&bfull[s], B_BYTES);
#pragma unroll
        for (int at = 0; at < NATOM; ++at)
          tma_load_2d(smem + OFF_B + s * B_BYTES + at * B_ATOM, &tmap, kb * BK + at * 64, tok0,
                      &bfull[s]);
      }
      for (int j = it > BST ? it - BST : 0; j < it; ++j)
        if (!mbar_wait_sleep(&bfull[j % BST], static_cast<uint32_t>(j / BST) & 1u, a.status,
                       kStatusGemmWait))
          break;
    }
  } else if (warp == 1 || (MMA2 && warp == 4 + G::DQW)) {
    // -------------------------------------------------------------- MMA
    // MMA2: thread `par` takes k-steps par, par + 2, ... into accumulator par
    if (lane == 0) {
      constexpr int STEP = MMA2 ? 2 : 1;
      const int par = warp == 1 ? 0 : 1;
      const uint32_t tacc = tmem + (MMA2 ? static_cast<uint32_t>(par * BN) : 0u);
      for (int it = par; it < NK; it += STEP) {
        const int s = it % BST, sa_i = it % ASTAGES;
        if (!mbar_wait_sleep(&aready[sa_i], static_cast<uint32_t>(it / ASTAGES) & 1u, a.status,
                       kStatusGemmWait))
          break;
        if (!mbar_wait_sleep(&bfull[s], static_cast<uint32_t>(it / BST) & 1u, a.status,
                       kStatusGemmWait))
          break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + OFF_A + sa_i * A_BYTES);
        const uint32_t sb = smem_u32(smem + OFF_B + s * B_BYTES);
#pragma unroll
        for (int k16 = 0; k16 < BK / 16; ++k16) {
          const uint32_t acc = (it != par || k16 != 0) ? 1u : 0u;
          const uint32_t ka = (k16 >> 2) * 16384 + (k16 & 3) * 32;  // atom, 16-col step
          const uint64_t db = sw128_desc(sb + (k16 >> 2) * B_ATOM + (k16 & 3) * 32);
          tc_mma(tacc, sw128_desc(sa + ka), db, G::kIdesc, acc);  // rows 0..127
          if constexpr (BM == 256)  // rows 128..255 into the second accumulator
            tc_mma(tmem + BN, sw128_desc(sa + A_HALF + ka), db, G::kIdesc, acc);
        }
        tc_commit(&afree[sa_i]);
        tc_commit(&bfree[s]);
        if (a.couple && (it % RK == RK - 1 || it == NK - 1)) tc_commit(&wfree[(it / RK) % RST]);
      }
      tc_commit(accfull);
      // the accumulators (and TMEM) stay in use until every MMA has finished
      mbar_wait_sleep(accfull, 0, a.status, kStatusGemmWait);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dequant
    if constexpr (FMT == kFmtNvfp4G16) {
      // 128 rows x 128 K per stage: thread dt takes row dt/2, K half dt%2 =
      // 32 nibble bytes (four 16-value groups) and its four e4m3 group scales;
      // e2m1 * e4m3 is exact in f16 (the f32 global scale is in the epilogue)
      static_assert(BM == 128 && BK == 128, "NVFP4 tiles are 128 x 128 K");
      const int dt = tid - 128;
      const int r = dt >> 1, part = dt & 1;
      const int c = r >> 4, rr = r & 15;
      for (int it = 0; it < NK; ++it) {
        const int rs = it / RK, s = rs % RST, sa_i = it % ASTAGES;
        if (!mbar_wait_sleep(&wfull[s], static_cast<uint32_t>(rs / RST) & 1u, a.status,
                       kStatusGemmWait))
          break;
        const uint8_t* ch = smem + OFF_RAW + s * RAW_BYTES + (c * RK + it % RK) * CHUNK;
        const uint4 n0 = *reinterpret_cast<const uint4*>(ch + rr * 64 + part * 32);
        const uint4 n1 = *reinterpret_cast<const uint4*>(ch + rr * 64 + part * 32 + 16);
        const uint32_t scw = *reinterpret_cast<const uint32_t*>(ch + 1024 + rr * 8 + part * 4);
        // the weight stage is free once its last k-step's bytes are in registers;
        // the proxy fence orders these generic reads before the bulk copy that
        // refills the slot (an async-proxy write)
        if (it % RK == RK - 1 || it == NK - 1) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&wfree[s]);
        }
        if (it >= ASTAGES &&
            !mbar_wait_sleep(&afree[sa_i], static_cast<uint32_t>(it / ASTAGES - 1) & 1u, a.status,
                       kStatusGemmWait))
          break;
        const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(scw & 0xffffu));
        const uint32_t s23 = e4m3x2_to_f16x2(static_cast<uint16_t>(scw >> 16));
        const __half2 sc2[4] = {__low2half2(*reinterpret_cast<const __half2*>(&s01)),
                                __high2half2(*reinterpret_cast<const __half2*>(&s01)),
                                __low2half2(*reinterpret_cast<const __half2*>(&s23)),
                                __high2half2(*reinterpret_cast<const __half2*>(&s23))};
        const uint32_t wd[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
        uint8_t* arow = smem + OFF_A + sa_i * A_BYTES + part * 16384 + (r >> 3) * 1024 +
                        (r & 7) * 128;
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // word i = 8 values = one 16-byte output chunk
          uint32_t o4[4];
          e2m1x8_to_f16x2x4(wd[i], o4);
#pragma unroll
          for (int q2 = 0; q2 < 4; ++q2) {
            const __half2 hv = __hmul2(*reinterpret_cast<const __half2*>(&o4[q2]), sc2[i >> 1]);
            o4[q2] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(arow + ((i ^ (r & 7)) << 4)) =
              make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[sa_i]);
      }
    } else {
    // thread dt converts BPT bytes: part `part` of row `row` of 16-row chunk c
    constexpr int BPT = BM * 64 / (32 * G::DQW);  // 32 bytes
    constexpr int TPR = 64 / BPT;      // threads per 64-byte row
    constexpr int NV = BPT / 16;       // 16-byte loads per thread
    const int dt = tid - 128;
    const int c = dt / (16 * TPR), within = dt % (16 * TPR);
    const int row = within / TPR, part = within % TPR;
    const int r = c * 16 + row;           // row of the block
    const int h = r >> 7, rh = r & 127;   // MMA half and row inside it
    // FP8 block-128: this thread's 128-row scale block (original row order;
    // the fused gate/up tile holds gate rows 8t.. in rows 0-7, up rows I+8t..)
    const float* bsc_row = nullptr;
    if constexpr (FMT == kFmtFp8Block128) {
      const int n = blk * BM + r, t = n >> 4, tr = n & 15;
      const int orig = !a.w.swiglu ? n : (tr < 8 ? 8 * t + tr : a.w.N / 2 + 8 * t + tr - 8);
      bsc_row = a.w.blk_scale + static_cast<size_t>(orig / 128) * a.w.blk_ld;
    }
    for (int it = 0; it < NK; ++it) {
      const int kb = KB0 + it, rs = it / RK, s = rs % RST, sa_i = it % ASTAGES;
      float bscale = 1.f;
      if constexpr (FMT == kFmtFp8Block128) bscale = __ldg(bsc_row + (kb >> 1));
      if (!mbar_wait_sleep(&wfull[s], static_cast<uint32_t>(rs / RST) & 1u, a.status,
                     kStatusGemmWait))
        break;
      const uint4* src = reinterpret_cast<const uint4*>(
          smem + OFF_RAW + s * RAW_BYTES + (c * RK + it % RK) * CHUNK + row * 64 + part * BPT);
      uint4 wv[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) wv[i] = src[i];
      // raw bytes are in registers; the weight stage is free after its last
      // k-step, once the proxy fence orders these generic reads before the
      // bulk copy that refills the slot (an async-proxy write)
      if (it % RK == RK - 1 || it == NK - 1) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfree[s]);
      }
      if (it >= ASTAGES &&
          !mbar_wait_sleep(&afree[sa_i], static_cast<uint32_t>(it / ASTAGES - 1) & 1u, a.status,
                     kStatusGemmWait))
        break;
      uint8_t* arow = smem + OFF_A + sa_i * A_BYTES + h * A_HALF + (rh >> 3) * 1024 + (rh & 7) * 128;
#pragma unroll
      for (int i = 0; i < 2 * NV; ++i) {  // 16-byte output chunk j = k 8j .. 8j+7
        const int j = part * 2 * NV + i;
        const uint32_t w0 = (&wv[i >> 1].x)[(i & 1) * 2];
        const uint32_t w1 = (&wv[i >> 1].x)[(i & 1) * 2 + 1];
        uint4 o;
        if constexpr (FMT == kFmtW8A16Row) {
          o.x = i8_lo_pair(w0);
          o.y = i8_hi_pair(w0);
          o.z = i8_lo_pair(w1);
          o.w = i8_hi_pair(w1);
        } else {
          o.x = e4m3x2_to_f16x2(static_cast<uint16_t>(w0 & 0xffffu));
          o.y = e4m3x2_to_f16x2(static_cast<uint16_t>(w0 >> 16));
          o.z = e4m3x2_to_f16x2(static_cast<uint16_t>(w1 & 0xffffu));
          o.w = e4m3x2_to_f16x2(static_cast<uint16_t>(w1 >> 16));
          if constexpr (FMT == kFmtFp8Block128) {
            // the 128 x 128 block scale varies along K, so it is applied here
            // (e4m3 * scale rounded to f16; relative error <= 2^-11)
            uint32_t* ow = &o.x;
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ow[q2]));
              const __half2 hs = __floats2half2_rn(f.x * bscale, f.y * bscale);
              ow[q2] = *reinterpret_cast<const uint32_t*>(&hs);
            }
          }
        }
        *reinterpret_cast<uint4*>(arow + ((j ^ (rh & 7)) << 4)) = o;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&aready[sa_i]);
    }
    }

    // ---------------------------------------------------------- epilogue
    // the whole warp takes the same branch (tcgen05.ld is warp-collective)
    const bool acc_ok =
        __all_sync(0xffffffffu, mbar_wait_sleep(accfull, 0, a.status, kStatusGemmWait));
    // Every dequant warp takes part: warp 4 + ew reads TMEM lane quarter
    // ew % 4 of accumulator half hh, for token part cp of NCP.
    constexpr int NH = BM / 128, NCP = G::DQW / 4 / NH, EPT = G::DQW * 32;
    static_assert(NCP >= 1 && (BN / 16) % NCP == 0, "epilogue token split");
    const int ew = warp - 4;
    const int hh = (ew >> 2) % NH, cp = (ew >> 2) / NH;
    // Output columns of this block: BM rows, or BM / 2 SwiGLU columns.
    constexpr int OW = EPI == kEpiSwiglu ? BM / 2 : BM;
    const int col0 = blk * OW;
    const int ntok = min(BN, a.M - tok0);
    // Staged epilogue (residual and SwiGLU): the block's output tile
    // [ntok][OW] is assembled in the activation ring (idle once every MMA has
    // finished: each of its TMA loads was consumed by an MMA), so that the
    // residual is read and the output written with coalesced 16-byte accesses
    // instead of one dependent 2-byte access per thread and token.  Plain
    // stores measured faster written directly (no barrier, nothing to wait for).
    const bool staged = (EPI == kEpiResidual || EPI == kEpiSwiglu) && (a.out_ld % 8) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                        col0 + OW <= (EPI == kEpiSwiglu ? a.w.N / 2 : a.w.N);
    static_assert(OW <= BST * BK, "output tile must fit the activation ring");
    if (ew < G::DQW) {
      const int q = warp & 3;          // TMEM lane quarter this warp may read
      const int rr = hh * 128 + 32 * q + lane;  // row of the block
      float rs = a.w.row_scale ? a.w.row_scale[static_cast<size_t>(blk) * BM + rr] : 1.f;
      if constexpr (FMT == kFmtNvfp4G16) rs *= a.w.global_scale;
      const int n = blk * BM + rr;
      const int tr = rr & 15;  // row inside the 16-row tile
      // SwiGLU output column (the fused gate/up tile holds gate rows 8t.. in
      // rows 0-7 and up rows in 8-15)
      const int jl = (rr >> 4) * 8 + (tr & 7);
      const int jcol = col0 + jl;
      Act* T = reinterpret_cast<Act*>(smem + OFF_B);  // [BN][OW] when staged
      constexpr int VPR = OW / 8;                      // 16-byte vectors per token row
      const int et = tid - 128;                        // 0 .. EPT-1
      if (staged && EPI == kEpiResidual) {
#pragma unroll 8
        for (int i = et; i < ntok * VPR; i += EPT) {
          const int tk = i / VPR, v = i % VPR;
          reinterpret_cast<uint4*>(T + tk * OW)[v] = *reinterpret_cast<const uint4*>(
              reinterpret_cast<const Act*>(a.out) + static_cast<size_t>(tok0 + tk) * a.out_ld +
              col0 + v * 8);
        }
      }
      if (staged) named_bar_sync(1, EPT);
      if (acc_ok) {
        tc_fence_after();
        constexpr int CBP = BN / 16 / NCP;  // 16-token column blocks per part
        for (int cb = cp * CBP; cb < (cp + 1) * CBP; ++cb) {
          uint32_t v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + hh * BN + cb * 16, v);
          if constexpr (MMA2) {
            // the odd k-steps' accumulator (none when the split has one k-step)
            if (NK > 1) {
              uint32_t v2[16];
              tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + BN + cb * 16, v2);
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                v[jj] = __float_as_uint(__uint_as_float(v[jj]) + __uint_as_float(v2[jj]));
            }
          }
          if constexpr (EPI == kEpiPartial) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int tk = cb * 16 + jj, tok = tok0 + tk;
              // this split's scaled partial sum, rounded once the splits are added
              if (tok < a.M && n < a.w.N)
                a.part[(static_cast<size_t>(blockIdx.z) * a.M + tok) * a.w.N + n] =
                    __uint_as_float(v[jj]) * (exp2i(sxexp[tk]) * rs);
            }
          } else if (staged) {
            if constexpr (EPI == kEpiSwiglu) {
              // tokens in pairs: the gate lane forms the even token's output,
              // its up partner (lane ^ 8) the odd token's
              const bool gate = tr < 8;
#pragma unroll
              for (int jj = 0; jj < 16; jj += 2) {
                const int tk = cb * 16 + jj;
                const float y0 = AT::round(__uint_as_float(v[jj]) * (exp2i(sxexp[tk]) * rs));
                const float y1 =
                    AT::round(__uint_as_float(v[jj + 1]) * (exp2i(sxexp[tk + 1]) * rs));
                const float recv = __shfl_xor_sync(0xffffffffu, gate ? y1 : y0, 8);
                const float g = gate ? y0 : recv, u = gate ? recv : y1;
                const int tko = tk + (gate ? 0 : 1);
                if (tko < ntok) T[tko * OW + jl] = AT::from_f(silu_mul_ref<Act>(g, u));
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int tk = cb * 16 + jj;
                if (tk < ntok) {
                  const float y = AT::round(__uint_as_float(v[jj]) * (exp2i(sxexp[tk]) * rs));
                  Act* t = T + tk * OW + rr;
                  *t = EPI == kEpiResidual ? AT::from_f(y + AT::to_f(*t)) : AT::from_f(y);
                }
              }
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int tk = cb * 16 + jj, tok = tok0 + tk;
              const float y = AT::round(__uint_as_float(v[jj]) * (exp2i(sxexp[tk]) * rs));
              if constexpr (EPI == kEpiSwiglu) {
                const float yu = __shfl_down_sync(0xffffffffu, y, 8);
                if (tr < 8 && tok < a.M && jcol < a.w.N / 2)
                  reinterpret_cast<Act*>(a.out)[static_cast<size_t>(tok) * a.out_ld + jcol] =
                      AT::from_f(silu_mul_ref<Act>(y, yu));
              } else {
                if (tok < a.M && n < a.w.N) {
                  Act* o = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(tok) * a.out_ld + n;
                  *o = EPI == kEpiResidual ? AT::from_f(y + AT::to_f(*o)) : AT::from_f(y);
                }
              }
            }
          }
        }
      }
      if (staged) {
        named_bar_sync(1, EPT);
#pragma unroll 8
        for (int i = et; i < ntok * VPR; i += EPT) {
          const int tk = i / VPR, v = i % VPR;
          *reinterpret_cast<uint4*>(reinterpret_cast<Act*>(a.out) +
                                    static_cast<size_t>(tok0 + tk) * a.out_ld + col0 + v * 8) =
              reinterpret_cast<const uint4*>(T + tk * OW)[v];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2)
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

template <typename Act, int FMT, int EPI, int BM, int BN, int BK = 64>
cudaError_t launch_gemm(const CUtensorMap& map, const GemmArgs& a, cudaStream_t s, int ks = 1) {
  using G = Cfg<BM, BN, BK>;
  auto kern = w8a16_gemm_kernel<Act, FMT, EPI, BM, BN, BK>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.M + BN - 1) / BN, a.w.T / (BM / 16), ks);
  kern<<<grid, G::THREADS, G::SMEM_BYTES, s>>>(map, a);
  return cudaGetLastError();
}

// Split-K epilogue: out = epilogue(act(sum over the ks partials, in split
// order)); one thread per output element (SwiGLU: per gate/up pair).
template <typename Act, int EPI>
__global__ void splitk_finalize_kernel(const GemmArgs a, int ks) {
  using AT = ActTraits<Act>;
  const int N = a.w.N;
  const int cols = EPI == kEpiSwiglu ? N / 2 : N;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(a.M) * cols) return;
  const int tok = static_cast<int>(idx / cols), j = static_cast<int>(idx % cols);
  auto total = [&](int n) {
    float y = 0.f;
    for (int z = 0; z < ks; ++z) y += a.part[(static_cast<size_t>(z) * a.M + tok) * N + n];
    return AT::round(y);
  };
  Act* o = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(tok) * a.out_ld + j;
  if constexpr (EPI == kEpiSwiglu) {
    // fused gate/up rows: tile t holds gate rows 8t.. in rows 0-7, up rows in 8-15
    const int t = j >> 3, tr = j & 7;
    *o = AT::from_f(silu_mul_ref<Act>(total(16 * t + tr), total(16 * t + 8 + tr)));
  } else if constexpr (EPI == kEpiResidual) {
    *o = AT::from_f(total(j) + AT::to_f(*o));
  } else {
    *o = AT::from_f(total(j));
  }
}

template <typename Act, int FMT, int BK>
cudaError_t launch_split(const CUtensorMap& map, const GemmArgs& a, int epi, int ks, int bn,
                         cudaStream_t s) {
  cudaError_t e = bn == 64 ? launch_gemm<Act, FMT, kEpiPartial, 128, 64, BK>(map, a, s, ks)
                           : launch_gemm<Act, FMT, kEpiPartial, 128, 128, BK>(map, a, s, ks);
  if (e != cudaSuccess) return e;
  const long long n = static_cast<long long>(a.M) * (epi == kEpiSwiglu ? a.w.N / 2 : a.w.N);
  const int blocks = static_cast<int>((n + 255) / 256);
  switch (epi) {
    case kEpiStore: splitk_finalize_kernel<Act, kEpiStore><<<blocks, 256, 0, s>>>(a, ks); break;
    case kEpiResidual: splitk_finalize_kernel<Act, kEpiResidual><<<blocks, 256, 0, s>>>(a, ks); break;
    case kEpiSwiglu: splitk_finalize_kernel<Act, kEpiSwiglu><<<blocks, 256, 0, s>>>(a, ks); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// 256 x 256 tiles when they give at least half the SMs a CTA (measured: a
// half-empty wave of the larger tile still beats 3+ waves of 128 x 128),
// else 128 x 128.  Calls of at most 128 rows (one token tile either way)
// take 128 x 128 tiles, filled up by split-K where the caller allows it.
bool use_big_tiles(const GemmArgs& a) {
  if (a.M <= 128) return false;
  const bool fits = a.w.T % 16 == 0 && (a.w.swiglu ? (a.w.N / 2) % 128 == 0 : a.w.N % 256 == 0);
  return fits && 2 * static_cast<long long>((a.M + 255) / 256) * (a.w.T / 16) >= sm_count();
}

// K splits for a 128-row-tile launch: the count (1..8, at least 4 k-steps
// each, partials within the workspace) that minimises the weight stream over
// the SM waves it fills plus the f32 partials written and read back.
// Measured basis: one CTA per SM; a half-empty last wave leaves its SMs idle.
int k_splits(const GemmArgs& a, int bn) {
  if (!a.part) return 1;
  const int sms = sm_count();
  const long long base = static_cast<long long>((a.M + bn - 1) / bn) * (a.w.T / 8);
  const double wbytes =
      static_cast<double>(a.w.N) * a.w.K * (a.w.fmt == kFmtNvfp4G16 ? 0.5625 : 1.0);
  int best = 1;
  double best_cost = 0.0;
  for (int ks = 1; ks <= 8; ++ks) {
    if (ks > 1 && (a.w.C / ks < 4 || static_cast<size_t>(ks) * a.M * a.w.N * 4 > a.part_bytes))
      break;
    const long long ctas = base * ks;
    const long long waves = (ctas + sms - 1) / sms;
    const double fill = static_cast<double>(ctas) / (static_cast<double>(sms) * waves);
    const double cost = wbytes / fill + (ks > 1 ? 8.0 * ks * a.M * a.w.N : 0.0);
    if (ks == 1 || cost < best_cost * 0.999) {
      best = ks;
      best_cost = cost;
    }
  }
  return best;
}

template <typename Act, int FMT>
cudaError_t launch_fmt(const CUtensorMap& map, const GemmArgs& a, int epi, bool big, int bn,
                       cudaStream_t s) {
  if constexpr (FMT == kFmtNvfp4G16) {
    switch (epi) {
      case kEpiStore: return launch_gemm<Act, FMT, kEpiStore, 128, 128, 128>(map, a, s);
      case kEpiResidual: return launch_gemm<Act, FMT, kEpiResidual, 128, 128, 128>(map, a, s);
      case kEpiSwiglu: return launch_gemm<Act, FMT, kEpiSwiglu, 128, 128, 128>(map, a, s);
      default: return cudaErrorInvalidValue;
    }
  } else {
    switch (epi) {
      case kEpiStore:
        return big ? launch_gemm<Act, FMT, kEpiStore, 256, 256>(map, a, s)
               : bn == 64 ? launch_gemm<Act, FMT, kEpiStore, 128, 64>(map, a, s)
                          : launch_gemm<Act, FMT, kEpiStore, 128, 128>(map, a, s);
      case kEpiResidual:
        return big ? launch_gemm<Act, FMT, kEpiResidual, 256, 256>(map, a, s)
               : bn == 64 ? launch_gemm<Act, FMT, kEpiResidual, 128, 64>(map, a, s)
                          : launch_gemm<Act, FMT, kEpiResidual, 128, 128>(map, a, s);
      case kEpiSwiglu:
        return big ? launch_gemm<Act, FMT, kEpiSwiglu, 256, 256>(map, a, s)
               : bn == 64 ? launch_gemm<Act, FMT, kEpiSwiglu, 128, 64>(map, a, s)
                          : launch_gemm<Act, FMT, kEpiSwiglu, 128, 128>(map, a, s);
      default: return cudaErrorInvalidValue;
    }
  }
}

template <typename Act>
cudaError_t launch_act(const CUtensorMap& map, const GemmArgs& a, int epi, bool big, int ks,
                       int bn, cudaStream_t s, const CUtensorMap* tail_map = nullptr,
                       const GemmArgs* tail = nullptr) {
  const int prep_blocks = (a.M + kPrepRows - 1) / kPrepRows;
  if (a.M < 256) {  // few rows: a CTA per row keeps more of each row's loads in flight
    if (a.norm_w)
      prep_row_kernel<Act, true><<<a.M, 256, 0, s>>>(a);
    else
      prep_row_kernel<Act, false><<<a.M, 256, 0, s>>>(a);
  } else if (a.norm_w) {
    prep_kernel<Act, true><<<prep_blocks, kPrepRows * 32, 0, s>>>(a);
  } else {
    prep_kernel<Act, false><<<prep_blocks, kPrepRows * 32, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (ks > 1) {
    switch (a.w.fmt) {
      case kFmtW8A16Row: return launch_split<Act, kFmtW8A16Row, 64>(map, a, epi, ks, bn, s);
      case kFmtFp8Row: return launch_split<Act, kFmtFp8Row, 64>(map, a, epi, ks, bn, s);
      case kFmtFp8Block128: return launch_split<Act, kFmtFp8Block128, 64>(map, a, epi, ks, bn, s);
      case kFmtNvfp4G16: return launch_split<Act, kFmtNvfp4G16, 128>(map, a, epi, ks, bn, s);
      default: return cudaErrorInvalidValue;
    }
  }
  if (tail) {  // rows past the full waves of 256 x 256 tiles: 128 x 128 tiles (W8A16)
    e = launch_fmt<Act, kFmtW8A16Row>(map, a, epi, true, 256, s);
    if (e != cudaSuccess) return e;
    return launch_fmt<Act, kFmtW8A16Row>(*tail_map, *tail, epi, false, 128, s);
  }
  switch (a.w.fmt) {
    case kFmtW8A16Row: return launch_fmt<Act, kFmtW8A16Row>(map, a, epi, big, bn, s);
    case kFmtFp8Row: return launch_fmt<Act, kFmtFp8Row>(map, a, epi, big, bn, s);
    case kFmtFp8Block128: return launch_fmt<Act, kFmtFp8Block128>(map, a, epi, big, bn, s);
    case kFmtNvfp4G16: return launch_fmt<Act, kFmtNvfp4G16>(map, a, epi, false, 128, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool gemm_w8a16_supported(const DevQLinear& w) {
  const bool scales = (w.fmt == kFmtW8A16Row || w.fmt == kFmtFp8Row) ? w.row_scale != nullptr
                     : w.fmt == kFmtFp8Block128                     ? w.blk_scale != nullptr
                                                                    : w.fmt == kFmtNvfp4G16;
  return scales && w.T % 8 == 0 && w.K % 8 == 0 && w.K <= 12 * 8 * 256 &&
         (w.swiglu ? (w.N / 2) % 64 == 0 : w.N % 128 == 0);
}

size_t gemm_scratch_bytes(int rows, int k_pad) {
  const size_t xh = (static_cast<size_t>(rows) * k_pad * 2 + 255) / 256 * 256;
  return xh + (static_cast<size_t>(rows) * 4 + 255) / 256 * 256;
}

cudaError_t gemm_w8a16_launch(const GemmArgs& a, int act, int epi, cudaStream_t s) {
  if (!gemm_w8a16_supported(a.w) || a.M < 1 || !a.xh || !a.xexp || !a.out) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.x) & 15) || (a.x_ld % 8) ||
      (a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15)) ||
      (reinterpret_cast<uintptr_t>(a.xh) & 255))
    return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu && !a.w.swiglu) return cudaErrorInvalidValue;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  GemmArgs a2 = a;
  // weight slots are released once the dequant warps hold the bytes and have
  // fenced their reads against the refill (DIAL_B200_GEMM_COUPLE=1: also wait
  // for the k-step's MMAs)
  a2.couple = 0;
  if (const char* v = std::getenv("DIAL_B200_GEMM_COUPLE")) a2.couple = std::atoi(v);
  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.w.K_pad), static_cast<cuuint64_t>(a.M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.w.K_pad) * 2};
  const bool big = a.w.fmt != kFmtNvfp4G16 && use_big_tiles(a);
  // 64-token tiles for calls of at most 64 rows (int8 / e4m3 weights)
  const int bn = big ? 256 : (a.w.fmt != kFmtNvfp4G16 && a.M <= 64 ? 64 : 128);
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(bn)};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.xh, dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const int ks = big ? 1 : k_splits(a, bn);
  // Wave tail: when the 256 x 256 tiles fill W whole SM waves and leave a
  // last wave less than half full, the weight blocks of that last wave run
  // instead as 128 x 128 tiles in a second launch (a quarter of the work per
  // CTA, so the tail costs about a third of a wave instead of a whole one).
  // W8A16 only: its row scales and 1 KB chunks slice by tile.
  int tail_blocks = 0;
  if (big && a.w.fmt == kFmtW8A16Row && a.w.T % 16 == 0) {
    const char* v = std::getenv("DIAL_B200_GEMM_TAIL");
    if (!v || std::atoi(v) != 0) {
      const long long nt = (a.M + 255) / 256, nb = a.w.T / 16, sms = sm_count();
      const long long waves = nt * nb / sms, rem = nt * nb % sms;
      const long long nb_full = waves * sms / nt;
      // the tail's 128 x 128 tiles must fit one wave (measured: QKV at 2048
      // tokens, whose tail would take 1.3 waves, went 126 -> 131 us; gate/up
      // went 363 -> 342 us)
      const long long tail_ctas = 2 * (nb - nb_full) * ((a.M + 127) / 128);
      if (waves >= 1 && rem > 0 && 2 * rem <= sms && nb_full >= 1 && nb_full < nb &&
          tail_ctas <= sms)
        tail_blocks = static_cast<int>(nb - nb_full);
    }
  }
  if (tail_blocks > 0) {
    const int t0 = a.w.T - 16 * tail_blocks;  // first tile of the tail
    GemmArgs head = a2, tail = a2;
    head.w.T = t0;
    head.w.N = 16 * t0;
    tail.w.T = a.w.T - t0;
    tail.w.N = 16 * tail.w.T;
    tail.w.tiles = a.w.tiles + static_cast<size_t>(t0) * a.w.C * 1024;
    tail.w.row_scale = a.w.row_scale + static_cast<size_t>(t0) * 16;
    tail.out = reinterpret_cast<char*>(a.out) +
               static_cast<size_t>(epi == kEpiSwiglu ? 8 * t0 : 16 * t0) * 2;  // 2-byte activations
    CUtensorMap tmap;
    const cuuint32_t tbox[2] = {64, 128};
    if (enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.xh, dims, strides, tbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    return act == 0 ? launch_act<__nv_bfloat16>(map, head, epi, true, 1, 256, s, &tmap, &tail)
                    : launch_act<__half>(map, head, epi, true, 1, 256, s, &tmap, &tail);
  }
  return act == 0 ? launch_act<__nv_bfloat16>(map, a2, epi, big, ks, bn, s)
                  : launch_act<__half>(map, a2, epi, big, ks, bn, s);
}

}  // namespace dialb200
