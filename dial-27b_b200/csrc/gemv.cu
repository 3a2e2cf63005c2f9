// Decode-path linear (M <= 8 tokens per launch): a memory-bound, dequant-fused
// GEMV for the weight formats of DIAL's worker linears.
//
// Reference kernels this replaces (all in lisa301/DIAL-27B):
//   dial_w8a16_decode_f16   dial-core/src/models/qwen3_vl/worker_w8a16.rs:146-184
//   dial_fp8_decode_f16     dial-core/src/models/qwen3_8/cuda_quant.rs:102-133
//   dial_nvfp4_decode_f16   dial-core/src/models/qwen3_8/cuda_quant.rs:67-100
// plus the dense candle Linear used for the lm_head (qwen3_vl.rs:1325-1335).
//
// Design (one CTA per SM, 16 consumer warps + 1 producer warp):
//  * The producer streams the CTA's contiguous range of 16-row weight tiles
//    through a shared-memory ring with 1-D bulk async copies (TMA engine),
//    32 chunks (32-36 KB) per stage, completion tracked on mbarriers; each
//    consumer warp takes two chunks of a stage (16 warps keep enough
//    independent dequant + MMA chains in flight to follow the copies).  It
//    starts before griddepcontrol.wait, so weight streaming overlaps the tail
//    of the previous kernel (programmatic dependent launch).
//  * Activations are staged once per CTA in shared memory as f16 (with a
//    power-of-two pre-scale that keeps bf16 values exact and in range); the
//    RMSNorm that precedes the QKV and gate/up projections is computed here.
//  * Each lane converts its own weight bytes into m16n8k16 A fragments in
//    registers (int8: PRMT+HSUB2, e4m3/e2m1: hardware cvt) and issues
//    register-fed MMAs with f32 accumulation; the K order inside a chunk is
//    permuted identically for weights and activations.
//  * Per-tile partial sums of the 8 warps are reduced in shared memory and
//    the epilogue applies the row scale and one of: store, residual add
//    (o_proj/down), or SiLU(gate)*up (fused gate/up projection).
#include "common.cuh"
#include "gemv.h"
#include "gemv_dev.cuh"

namespace dialb200 {
namespace {

// Consumer warps per CTA (template NW): 16, with 32-chunk stages, while the
// staged activation rows leave room for them; 8, with 16-chunk stages, when
// more rows per launch fit that way (each launch re-streams the weights).
// Every consumer warp takes two chunks of a stage.
constexpr int kMaxSlots = 16;
constexpr int kMaxM = 8;
constexpr int kSmemBudget = 232448;         // 227 KB opt-in per CTA
constexpr int kMiscFlag = 32, kMiscKeys = 64, kMiscScratch = 128;  // offsets in the misc area

struct SmemPlan {
  int ring_off, x_off, red_off, misc_off, bsc_off, bar_off, total;
  int slots, xs_stride, bsc_rows_lo, bsc_rows_hi;
  int sc;  // chunks per ring stage
};

// Chunks per ring stage.  int8 / e4m3 / dense: two per consumer warp (their
// MMAs interleave in chunk_pair_mma).  NVFP4: a stage of 2*nw .. 3*nw chunks
// taken round-robin (warp w: chunks w, w + nw, w + 2 nw), sized so that a
// tile's C chunks cost the fewest stage x chunks-per-warp steps: C = 40
// (K = 5120) then runs as one 40-chunk stage of 2-3 chunks per warp instead
// of a full 32-chunk stage and an 8-chunk stage that keeps 12 warps idle.
__host__ __device__ inline int stage_chunks(const DevQLinear& w, int nw) {
  if (w.fmt != kFmtNvfp4G16) return 2 * nw;
  const int C = w.C;
  int best = 2 * nw, best_cost = (C + 2 * nw - 1) / (2 * nw) * 2;
  for (int sc = 2 * nw + 1; sc <= 3 * nw; ++sc) {
    const int per_warp = ((C < sc ? C : sc) + nw - 1) / nw;
    const int cost = (C + sc - 1) / sc * per_warp;
    if (cost < best_cost) {
      best = sc;
      best_cost = cost;
    }
  }
  return best;
}

// Block-scale row ranges a CTA needs for tiles [t0, t1).
__host__ __device__ inline void bsc_rows(const DevQLinear& w, int t0, int t1, int& lo0, int& nlo,
                                         int& hi0, int& nhi) {
  if (t1 <= t0) { lo0 = nlo = hi0 = nhi = 0; return; }
  if (w.swiglu) {
    const int I = w.N / 2;
    lo0 = (8 * t0) / 128;
    nlo = (8 * (t1 - 1)) / 128 - lo0 + 1;
    hi0 = (I + 8 * t0) / 128;
    nhi = (I + 8 * (t1 - 1)) / 128 - hi0 + 1;
  } else {
    lo0 = (16 * t0) / 128;
    nlo = (16 * (t1 - 1) + 15) / 128 - lo0 + 1;
    hi0 = 0;
    nhi = 0;
  }
}

__host__ inline SmemPlan make_plan(const DevQLinear& w, int M, int grid, int slots_req, int nw,
                                   int sc_req = 0) {
  SmemPlan p{};
  p.sc = stage_chunks(w, nw);
  // NVFP4 stage size override (2*nw .. 3*nw chunks)
  if (w.fmt == kFmtNvfp4G16 && sc_req >= 2 * nw && sc_req <= 3 * nw) p.sc = sc_req;
  const int stage = p.sc * fmt_chunk_bytes(w.fmt);
  p.xs_stride = w.K_pad + 8;
  const int x_bytes = ((M * p.xs_stride * 2) + 127) / 128 * 128;
  const int red_bytes = 2 * nw * 32 * 4 * 4;
  // misc: xexp [kMaxM] ints | argmax flag | argmax keys [kMaxM] | staging
  // scratch [2][nw] floats (block reduction of the activation statistics)
  const int misc_bytes = kMiscScratch + 2 * nw * 4;
  int bsc_bytes = 0;
  if (w.fmt == kFmtFp8Block128) {
    // worst case over CTAs: tiles per CTA <= ceil(T/grid)
    const int tpc = (w.T + grid - 1) / grid;
    const int rows_lo = w.swiglu ? (8 * tpc + 127) / 128 + 1 : (16 * tpc + 127) / 128 + 1;
    const int rows_hi = w.swiglu ? rows_lo : 0;
    p.bsc_rows_lo = rows_lo;
    p.bsc_rows_hi = rows_hi;
    bsc_bytes = (rows_lo + rows_hi) * w.blk_ld * 4;
    bsc_bytes = (bsc_bytes + 127) / 128 * 128;
  }
  const int bar_bytes = (2 * kMaxSlots + 2) * 8;
  const int fixed = x_bytes + red_bytes + misc_bytes + bsc_bytes + bar_bytes + 1024;
  int slots = (kSmemBudget - fixed) / stage;
  if (slots > kMaxSlots) slots = kMaxSlots;
  if (slots_req > 0 && slots_req < slots) slots = slots_req;
  p.slots = slots;
  p.ring_off = 0;
  p.x_off = slots * stage;
  p.red_off = p.x_off + x_bytes;
  p.misc_off = p.red_off + red_bytes;
  p.bsc_off = p.misc_off + misc_bytes;
  p.bar_off = p.bsc_off + bsc_bytes;
  p.total = p.bar_off + bar_bytes;
  return p;
}

// Consumer warps and rows per launch for M rows: rows per launch up to kMaxM,
// fewer when the staged activations would leave the weight ring under 4
// stages; 16 warps unless 8 warps need fewer launches.
__host__ inline void gemv_shape(const DevQLinear& w, int M, int& nw, int& group) {
  const int pgrid = std::max(1, std::min(w.T, 148));
  auto rows = [&](int n) {
    int g = kMaxM;
    while (g > 1 && make_plan(w, g, pgrid, 0, n).slots < 4) g >>= 1;
    return g;
  };
  const int g16 = rows(16), g8 = rows(8);
  const int l16 = (M + g16 - 1) / g16, l8 = (M + g8 - 1) / g8;
  nw = l16 <= l8 ? 16 : 8;
  group = nw == 16 ? g16 : g8;
}

template <int FMT>
struct XType { using T = __half; };

// ------------------------------------------------------------------ kernel
template <typename Act, int FMT, int EPI, bool NORM, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
    gemv_kernel(const GemvArgs a, const SmemPlan p) {
  constexpr int kNW = NW;                   // consumer warps
  using AT = ActTraits<Act>;
  using XT = typename std::conditional<FMT == kFmtDense, Act, __half>::type;
  constexpr bool kScaleX = (FMT != kFmtDense) && std::is_same<Act, __nv_bfloat16>::value;
  constexpr int CB = fmt_chunk_bytes(FMT);
  const int SC = p.sc;           // 2 * NW, or 2-3 * NW (NVFP4)
  const int SBYTES = SC * CB;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem + p.ring_off;
  XT* xs = reinterpret_cast<XT*>(smem + p.x_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  int* xexp = reinterpret_cast<int*>(smem + p.misc_off);
  float* scratch = reinterpret_cast<float*>(smem + p.misc_off + kMiscScratch);
  float* bsc = reinterpret_cast<float*>(smem + p.bsc_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + kMaxSlots;
  uint64_t* sbar = empty + kMaxSlots;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned long long tstamp[4] = {a.trace ? global_ns() : 0ull, 0ull, 0ull, 0ull};
  const int T = a.w.T, C = a.w.C;
  const int t0 = static_cast<int>(static_cast<long long>(T) * blockIdx.x / gridDim.x);
  const int t1 = static_cast<int>(static_cast<long long>(T) * (blockIdx.x + 1) / gridDim.x);
  const int spt = (C + SC - 1) / SC;
  const int NS = p.slots;

  int lo0 = 0, nlo = 0, hi0 = 0, nhi = 0;
  if constexpr (FMT == kFmtFp8Block128) bsc_rows(a.w, t0, t1, lo0, nlo, hi0, nhi);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kNW);
    }
    mbar_init(sbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kNW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if constexpr (FMT == kFmtFp8Block128) {
        const uint32_t row_bytes = static_cast<uint32_t>(a.w.blk_ld) * 4u;
        mbar_arrive_expect_tx(sbar, row_bytes * static_cast<uint32_t>(nlo + nhi));
        if (nlo) bulk_g2s(bsc, a.w.blk_scale + static_cast<size_t>(lo0) * a.w.blk_ld,
                          row_bytes * nlo, sbar);
        if (nhi) bulk_g2s(bsc + static_cast<size_t>(nlo) * a.w.blk_ld,
                          a.w.blk_scale + static_cast<size_t>(hi0) * a.w.blk_ld, row_bytes * nhi,
                          sbar);
      }
      // weights are read once per pass: evict them first so that activations,
      // norm weights and the KV cache stay in L2 between layers
      const uint64_t pol = l2_evict_first_policy();
      long long it = 0;
      int slot = 0;         // ring position and fill round, advanced incrementally
      uint32_t round = 0;
      bool ok = true;
      for (int t = t0; t < t1 && ok; ++t) {
        const uint8_t* src = a.w.tiles + static_cast<size_t>(t) * C * CB;
        for (int s = 0; s < spt; ++s, ++it) {
          if (round > 0 && !mbar_wait(&empty[slot], (round - 1) & 1u, a.status,
                                      kStatusEmptyWaitTimeout)) {
            ok = false;
            break;
          }
          const int nch = min(SC, C - s * SC);
          const uint32_t bytes = static_cast<uint32_t>(nch * CB);
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_g2s_hint(ring + static_cast<size_t>(slot) * SBYTES,
                        src + static_cast<size_t>(s) * SC * CB, bytes, &full[slot], pol);
          if (++slot == NS) {
            slot = 0;
            ++round;
          }
        }
      }
      // Drain: the most recent NS stages must have landed before the CTA may
      // retire, whether or not the consumers waited for them.
      const long long first = it > NS ? it - NS : 0;
      for (long long j = first; j < it; ++j) {
        const int slot = static_cast<int>(j % NS);
        if (!mbar_wait(&full[slot], static_cast<uint32_t>(j / NS) & 1u, a.status,
                       kStatusDrainTimeout))
          break;
      }
      if constexpr (FMT == kFmtFp8Block128) mbar_wait(sbar, 0, a.status, kStatusDrainTimeout);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  int* sflag = reinterpret_cast<int*>(smem + p.misc_off + kMiscFlag);
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem + p.misc_off + kMiscKeys);
  if constexpr (EPI == kEpiArgmax) {
    if (threadIdx.x < kMaxM) skey[threadIdx.x] = 0ull;
  }

  if constexpr (NORM) {
    // the RMSNorm weight is constant: bring it into L1 before the wait so
    // that staging after it touches only the activations in L2
    const char* nw = reinterpret_cast<const char*>(a.norm_w);
    for (int off = threadIdx.x * 128; off < a.w.K * static_cast<int>(sizeof(Act));
         off += kNW * 32 * 128)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(nw + off));
  }
  pdl_wait();
  if (a.trace) tstamp[1] = global_ns();
  stage_x<Act, XT, NORM, kScaleX, kNW>(a, xs, p.xs_stride, xexp, scratch);
  named_bar_sync(1, kNW * 32);
  if (a.trace) tstamp[2] = global_ns();
  if constexpr (FMT == kFmtFp8Block128) mbar_wait(sbar, 0, a.status, kStatusFullWaitTimeout);

  const int g = lane >> 2;
  const int tok = min(g, a.M - 1);
  const XT* xrow = xs + static_cast<size_t>(tok) * p.xs_stride;
  const int I = a.w.N / 2;

  int slot = 0;
  uint32_t round = 0;
  bool ok = true;
  int tile_i = 0;
  for (int t = t0; t < t1; ++t, ++tile_i) {
    // Epilogue operands of this tile (row scales, residual inputs) are loaded
    // now, so their latency hides behind the tile's stages.
    float pre_a = 1.f, pre_b = 1.f, pre_o = 0.f;
    if (threadIdx.x < 128) {
      const int rr = threadIdx.x >> 3, tt = threadIdx.x & 7;
      if constexpr (EPI == kEpiSwiglu) {
        if (threadIdx.x < 64 && a.w.row_scale) {
          pre_a = a.w.row_scale[t * 16 + rr];
          pre_b = a.w.row_scale[t * 16 + 8 + rr];
        }
      } else {
        const int n = t * 16 + rr;
        if (a.w.row_scale) pre_a = a.w.row_scale[t * 16 + rr];
        if constexpr (EPI == kEpiResidual) {
          if (tt < a.M && n < a.w.N)
            pre_o = AT::to_f(reinterpret_cast<const Act*>(a.out)[static_cast<size_t>(tt) * a.out_ld + n]);
        }
      }
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
    float pacc[4][4] = {};
    int rb_lo = 0, rb_hi = 0;
    if constexpr (FMT == kFmtFp8Block128) {
      if (a.w.swiglu) {
        rb_lo = (8 * t) / 128 - lo0;
        rb_hi = nlo + (I + 8 * t) / 128 - hi0;
      } else {
        rb_lo = rb_hi = (16 * t) / 128 - lo0;
      }
    }
    for (int s = 0; s < spt; ++s) {
      if (ok && !mbar_wait(&full[slot], round & 1u, a.status, kStatusFullWaitTimeout)) ok = false;
      const int nch = min(SC, C - s * SC);
      const uint8_t* st = ring + static_cast<size_t>(slot) * SBYTES;
      if (ok) {
        if constexpr (FMT == kFmtFp8Block128) {
          // only a warp with a chunk in this stage reads a block scale: the
          // others' column index is past the scales this CTA loaded
          if (warp * 2 < nch) {
            float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int ch = warp * 2 + j;
              if (ch < nch) chunk_mma<FMT, XT>(st + ch * CB, s * SC + ch, xrow, lane, tmp);
            }
            const int kb = (s * SC + warp * 2) / 2;
            const float slo = bsc[rb_lo * a.w.blk_ld + kb];
            const float shi = bsc[rb_hi * a.w.blk_ld + kb];
            acc[0] = fmaf(tmp[0], slo, acc[0]);
            acc[1] = fmaf(tmp[1], slo, acc[1]);
            acc[2] = fmaf(tmp[2], shi, acc[2]);
            acc[3] = fmaf(tmp[3], shi, acc[3]);
          }
        } else {
          const int ch0 = warp * 2, ch1 = warp * 2 + 1;
          if constexpr (FMT == kFmtW8A16Row || FMT == kFmtFp8Row) {
            if (nch == SC) {
              chunk_pair_mma<FMT, XT>(st + ch0 * CB, s * SC + ch0, xrow, lane, pacc);
            } else {
              if (ch0 < nch)
                chunk_mma<FMT, XT>(st + ch0 * CB, s * SC + ch0, xrow, lane, acc);
              if (ch1 < nch)
                chunk_mma<FMT, XT>(st + ch1 * CB, s * SC + ch1, xrow, lane, acc2);
            }
          } else if constexpr (FMT == kFmtNvfp4G16) {
            // round-robin: chunks warp, warp + NW (paired MMA chains), warp + 2 NW
            const int ca = warp, cb = warp + kNW, cc = warp + 2 * kNW;
            const int kc0 = s * SC;
            if (cb < nch)
              chunk_pair_nvfp4<XT>(st + ca * CB, kc0 + ca, st + cb * CB, kc0 + cb, xrow, lane, pacc);
            else if (ca < nch)
              chunk_mma<FMT, XT>(st + ca * CB, kc0 + ca, xrow, lane, acc);
            if (cc < nch) chunk_mma<FMT, XT>(st + cc * CB, kc0 + cc, xrow, lane, acc2);
          } else {
            if (ch0 < nch)
              chunk_mma<FMT, XT>(st + ch0 * CB, s * SC + ch0, xrow, lane, acc);
            if (ch1 < nch)
              chunk_mma<FMT, XT>(st + ch1 * CB, s * SC + ch1, xrow, lane, acc2);
          }
        }
      }
      // No proxy fence before the release: every shared-memory read of the
      // stage feeds an mma.sync, the empty asm below (it takes the
      // accumulators) keeps those MMAs ahead of the arrive in the instruction
      // stream, and a warp issues in order, so the reads have returned before
      // the arrive that lets the bulk copy refill the slot.  (A fence here
      // measured 1.2 % of the bs1 decode.)
      asm volatile("" : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc2[0]),
                   "+f"(acc2[1]), "+f"(acc2[2]), "+f"(acc2[3]));
      asm volatile("" : "+f"(pacc[0][0]), "+f"(pacc[0][1]), "+f"(pacc[0][2]), "+f"(pacc[0][3]),
                   "+f"(pacc[1][0]), "+f"(pacc[1][1]), "+f"(pacc[1][2]), "+f"(pacc[1][3]));
      asm volatile("" : "+f"(pacc[2][0]), "+f"(pacc[2][1]), "+f"(pacc[2][2]), "+f"(pacc[2][3]),
                   "+f"(pacc[3][0]), "+f"(pacc[3][1]), "+f"(pacc[3][2]), "+f"(pacc[3][3]));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == NS) {
        slot = 0;
        ++round;
      }
    }
    // ---- cross-warp reduction (double-buffered by tile parity)
    float* rb = red + (tile_i & 1) * (kNW * 128);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      acc[q] += acc2[q] + ((pacc[0][q] + pacc[1][q]) + (pacc[2][q] + pacc[3][q]));
    *reinterpret_cast<float4*>(rb + (warp * 32 + lane) * 4) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
    named_bar_sync(1, kNW * 32);
    const int i = threadIdx.x;
    auto gather = [&](int rr, int tt) {
      const int src_lane = (rr & 7) * 4 + (tt >> 1);
      const int reg = ((rr >> 3) << 1) | (tt & 1);
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kNW; ++w) v += rb[(w * 32 + src_lane) * 4 + reg];
      return v;
    };
    if constexpr (EPI == kEpiSwiglu) {
      if (i < 64) {
        const int rr = i >> 3, tt = i & 7;
        const int j = t * 8 + rr;
        if (tt < a.M && j < I) {
          float vg = gather(rr, tt), vu = gather(rr + 8, tt);
          float mul = exp2i(xexp[tt]);
          if constexpr (FMT == kFmtNvfp4G16) mul *= a.w.global_scale;
          const float sg = mul * pre_a, su = mul * pre_b;
          const float gq = AT::round(vg * sg), uq = AT::round(vu * su);
          Act* out = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(tt) * a.out_ld + j;
          *out = AT::from_f(silu_mul_ref<Act>(gq, uq));
        }
      }
    } else {
      if (i < 128) {
        const int rr = i >> 3, tt = i & 7;
        const int n = t * 16 + rr;
        if (tt < a.M && n < a.w.N) {
          float v = gather(rr, tt);
          float mul = exp2i(xexp[tt]);
          if constexpr (FMT == kFmtNvfp4G16) mul *= a.w.global_scale;
          mul *= pre_a;
          const float y = AT::round(v * mul);
          if constexpr (EPI == kEpiArgmax) {
            if (a.out)
              reinterpret_cast<Act*>(a.out)[static_cast<size_t>(tt) * a.out_ld + n] = AT::from_f(y);
            atomicMax(&skey[tt], argmax_key(y, n));
          } else {
            Act* out = reinterpret_cast<Act*>(a.out) + static_cast<size_t>(tt) * a.out_ld + n;
            if constexpr (EPI == kEpiResidual) {
              *out = AT::from_f(y + pre_o);
            } else {
              *out = AT::from_f(y);
            }
          }
        }
      }
    }
  }
  if (a.trace && threadIdx.x == 0) {
    tstamp[3] = global_ns();
    trace_record(a.trace, a.trace_tag, tstamp);
  }
  if constexpr (EPI == kEpiArgmax) {
    // CTA best -> global keys; the last CTA to arrive decodes and resets them.
    named_bar_sync(1, kNW * 32);
    if (threadIdx.x < a.M) atomicMax(&a.amax_key[threadIdx.x], skey[threadIdx.x]);
    __threadfence();
    named_bar_sync(1, kNW * 32);
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(a.amax_count, 1);
      *sflag = prev == static_cast<int>(gridDim.x) - 1;
    }
    named_bar_sync(1, kNW * 32);
    if (*sflag) {
      __threadfence();
      if (threadIdx.x < a.M) {
        const unsigned long long k = atomicExch(&a.amax_key[threadIdx.x], 0ull);
        a.amax_tok[threadIdx.x] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k));
      }
      if (threadIdx.x == 0) atomicExch(a.amax_count, 0);
    }
  }
}

template <typename Act, int FMT, int EPI, bool NORM, int NW>
cudaError_t launch_one(const GemvArgs& a, const GemvTuning& t, cudaStream_t stream) {
  const int slots_req = t.slots, grid_req = t.grid;
  const bool pdl = t.pdl;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int grid = grid_req > 0 ? grid_req : sms;
  if (grid > a.w.T) grid = a.w.T;
  const SmemPlan p = make_plan(a.w, a.M, grid, slots_req, NW, t.nvfp4_stage);
  if (p.slots < 2) return cudaErrorInvalidConfiguration;
  auto kern = gemv_kernel<Act, FMT, EPI, NORM, NW>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBudget);
  if (err != cudaSuccess) return err;
  // Largest shared-memory carveout, so that two CTAs of consecutive launches
  // can share an SM when their plans are small enough.
  err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((NW + 1) * 32);
  cfg.dynamicSmemBytes = p.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, p);
}

template <typename Act, int FMT, int EPI, bool NORM>
cudaError_t launch_nw(const GemvArgs& a, int nw, const GemvTuning& t, cudaStream_t s) {
  return nw == 16 ? launch_one<Act, FMT, EPI, NORM, 16>(a, t, s)
                  : launch_one<Act, FMT, EPI, NORM, 8>(a, t, s);
}

template <typename Act, int FMT>
cudaError_t dispatch_epi(const GemvArgs& a, int epi, bool norm, int nw, const GemvTuning& t,
                         cudaStream_t s) {
  if (epi == kEpiArgmax) {
    if constexpr (FMT == kFmtDense || FMT == kFmtW8A16Row)
      return norm ? launch_nw<Act, FMT, kEpiArgmax, true>(a, nw, t, s)
                  : launch_nw<Act, FMT, kEpiArgmax, false>(a, nw, t, s);
    return cudaErrorInvalidValue;
  }
  if (epi == kEpiStore)
    return norm ? launch_nw<Act, FMT, kEpiStore, true>(a, nw, t, s)
                : launch_nw<Act, FMT, kEpiStore, false>(a, nw, t, s);
  if (epi == kEpiResidual)
    return norm ? launch_nw<Act, FMT, kEpiResidual, true>(a, nw, t, s)
                : launch_nw<Act, FMT, kEpiResidual, false>(a, nw, t, s);
  if (epi == kEpiSwiglu)
    return norm ? launch_nw<Act, FMT, kEpiSwiglu, true>(a, nw, t, s)
                : launch_nw<Act, FMT, kEpiSwiglu, false>(a, nw, t, s);
  return cudaErrorInvalidValue;
}

template <typename Act>
cudaError_t dispatch_fmt(const GemvArgs& a, int epi, bool norm, int nw, const GemvTuning& t,
                         cudaStream_t s) {
  switch (a.w.fmt) {
    case kFmtW8A16Row: return dispatch_epi<Act, kFmtW8A16Row>(a, epi, norm, nw, t, s);
    case kFmtFp8Block128:
      return dispatch_epi<Act, kFmtFp8Block128>(a, epi, norm, nw, t, s);
    case kFmtFp8Row: return dispatch_epi<Act, kFmtFp8Row>(a, epi, norm, nw, t, s);
    case kFmtNvfp4G16: return dispatch_epi<Act, kFmtNvfp4G16>(a, epi, norm, nw, t, s);
    case kFmtDense: return dispatch_epi<Act, kFmtDense>(a, epi, norm, nw, t, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t gemv_launch(const GemvArgs& args, int act, int epi, bool norm, cudaStream_t stream,
                        const GemvTuning& tune) {
  if (args.M < 1 || args.w.T < 1 || args.w.C < 1) return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu && !args.w.swiglu) return cudaErrorInvalidValue;
  GemvArgs a = args;
  const size_t esz = 2;
  int nw = 16, group = 1;
  gemv_shape(args.w, args.M, nw, group);
  const int pgrid = std::max(1, std::min(args.w.T, 148));
  if (make_plan(args.w, group, pgrid, 0, nw).slots < 2) return cudaErrorInvalidConfiguration;
  for (int r0 = 0; r0 < args.M; r0 += group) {
    a.M = std::min(group, args.M - r0);
    a.x = static_cast<const char*>(args.x) + static_cast<size_t>(r0) * args.x_ld * esz;
    a.out = args.out ? static_cast<char*>(args.out) + static_cast<size_t>(r0) * args.out_ld * esz
                     : nullptr;
    if (epi == kEpiArgmax) {
      if (!args.amax_key || !args.amax_count || !args.amax_tok) return cudaErrorInvalidValue;
      a.amax_key = args.amax_key + r0;
      a.amax_count = args.amax_count + r0;
      a.amax_tok = args.amax_tok + r0;
    }
    cudaError_t e = act == 0 ? dispatch_fmt<__nv_bfloat16>(a, epi, norm, nw, tune, stream)
                             : dispatch_fmt<__half>(a, epi, norm, nw, tune, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int gemv_smem_bytes(const DevQLinear& w, int M, int grid, int slots) {
  int nw = 16, group = 1;
  gemv_shape(w, M, nw, group);
  return make_plan(w, std::min(M, group), grid, slots, nw).total;
}

}  // namespace dialb200
