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
// (arrival counter, self-resetting to zero).  Steps of more than 4 rows with
// groups of 4 query heads take the token-split form instead: each warp reads
// a quarter of every page and scores it for all 4 heads, so every K/V row is
// loaded once per CTA rather than once per warp.
#include <atomic>
#include <cmath>

#include "attention.h"
#include "attn_dev.cuh"
#include "common.cuh"

namespace dialb200 {
namespace {

constexpr int kD = kHeadDim;

// CTAs per SM the plain kernel is register-limited to: 6 for groups of 4
// query heads (80 registers, a few spills) keeps 48 KB of page loads in
// flight per SM instead of 32 KB at the unconstrained 4 CTAs.
template <int NREP>
constexpr int decode_min_ctas() { return NREP == 4 ? 6 : 1; }

template <typename Act, int NREP>
__global__ void __launch_bounds__(NREP * 32, decode_min_ctas<NREP>())
    attn_decode_kernel(const AttnDecodeArgs a) {
  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  __shared__ AttnItemSmem sm;
  attn_item<Act, NREP, true>(a, blockIdx.z, blockIdx.x, blockIdx.y, threadIdx.x >> 5,
                             threadIdx.x & 31, sm, 1);
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
}

// Token-split form: the group's warps share each page's tokens (TSG pages of
// loads in flight per warp) and merge their per-head partials in shared memory.
// One page per warp (96 registers, 5 CTAs per SM) measured ahead of 2 and 4
// (128 / 167 registers: 4 / 3 CTAs per SM).
constexpr int kTokSplitPages = 1;

template <typename Act, int NREP, int TSG>
__global__ void __launch_bounds__(NREP * 32) attn_decode_ts_kernel(const AttnDecodeArgs a) {
  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  __shared__ AttnItemSmem sm;
  __shared__ AttnTokSplitSmem<NREP> ts;
  attn_item<Act, NREP, true, 0, 0, TSG>(a, blockIdx.z, blockIdx.x, blockIdx.y, threadIdx.x >> 5,
                                        threadIdx.x & 31, sm, 1, nullptr, nullptr, nullptr,
                                        nullptr, &ts);
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
}

// Cluster form: the CL splits of a (row, kv head) that share a cluster merge
// their partials over distributed shared memory.
template <typename Act, int NREP, int CL>
__global__ void __launch_bounds__(NREP * 32) attn_decode_cluster_kernel(const AttnDecodeArgs a) {
  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  __shared__ AttnItemSmem sm;
  __shared__ AttnClusterSmem<NREP> cs;
  attn_item<Act, NREP, true, CL>(a, blockIdx.z, blockIdx.x, blockIdx.y, threadIdx.x >> 5,
                                 threadIdx.x & 31, sm, 1, &cs);
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
}

// Cluster form with the token-split scan.
template <typename Act, int NREP, int CL, int TSG>
__global__ void __launch_bounds__(NREP * 32) attn_decode_cluster_ts_kernel(const AttnDecodeArgs a) {
  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  __shared__ AttnItemSmem sm;
  __shared__ AttnClusterSmem<NREP> cs;
  __shared__ AttnTokSplitSmem<NREP> ts;
  attn_item<Act, NREP, true, CL, 0, TSG>(a, blockIdx.z, blockIdx.x, blockIdx.y, threadIdx.x >> 5,
                                         threadIdx.x & 31, sm, 1, &cs, nullptr, nullptr, nullptr,
                                         &ts);
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
}

// Ring form (optionally clustered, CL > 0): NREP query warps + one producer
// warp that streams each split's K/V pages through a shared-memory ring.
constexpr int kRingPages = 4;
constexpr int kRingBytes = kRingPages * 2 * kPageBytes;

template <typename Act, int NREP, int CL>
__global__ void __launch_bounds__((NREP + 1) * 32) attn_decode_ring_kernel(const AttnDecodeArgs a) {
  pdl_launch_dependents();
  const unsigned long long t_entry = a.trace ? global_ns() : 0ull;
  __shared__ AttnItemSmem sm;
  __shared__ AttnClusterSmem<NREP> cs;  // partials of the cluster merge (CL > 0)
  __shared__ uint64_t bars[2 * kRingPages];
  extern __shared__ __align__(128) uint8_t ring[];  // kRingBytes
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRingPages; ++i) {
      mbar_init(&bars[i], 1);                   // full: the producer's expect_tx
      mbar_init(&bars[kRingPages + i], NREP);   // empty: one arrival per query warp
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == NREP) {
    attn_ring_producer<CL, kRingPages>(a, blockIdx.z, blockIdx.x, blockIdx.y, lane, ring, bars,
                                       bars + kRingPages);
    return;
  }
  attn_item<Act, NREP, true, CL, kRingPages>(a, blockIdx.z, blockIdx.x, blockIdx.y, warp, lane, sm,
                                             1, &cs, ring, bars, bars + kRingPages);
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long t[4] = {t_entry, 0ull, 0ull, global_ns()};
    trace_record(a.trace, a.trace_tag, t);
  }
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
  norm_rope<Act>(k, reinterpret_cast<const Act*>(a.k_norm_w), a.sh.eps, cos_row, sin_row, lane);
  const int blk = checked_block(a, a.block_table[pos / kPageTokens]);
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

// Launch of the cluster form with CL splits per cluster; false when this
// device cannot hold such a cluster (the caller then takes the plain form).
template <typename Act, int NREP, int CL, bool RING, bool TS>
constexpr auto cluster_kernel() {
  if constexpr (RING) return attn_decode_ring_kernel<Act, NREP, CL>;
  else if constexpr (TS) return attn_decode_cluster_ts_kernel<Act, NREP, CL, kTokSplitPages>;
  else return attn_decode_cluster_kernel<Act, NREP, CL>;
}

template <typename Act, int NREP, int CL, bool RING, bool TS = false>
bool launch_cluster(const AttnDecodeArgs& a, cudaStream_t s, bool pdl, cudaError_t& err) {
  auto kern = cluster_kernel<Act, NREP, CL, RING, TS>();
  // per instantiation and device: checked once (racing first calls compute
  // the same answer); devices past the table are checked on every call
  constexpr int kMaxDev = 64;
  static std::atomic<int> usable_by_dev[kMaxDev];  // 0 unknown, 1 usable, 2 not
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>* slot = dev >= 0 && dev < kMaxDev ? &usable_by_dev[dev] : nullptr;
  int usable = slot ? slot->load(std::memory_order_relaxed) : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.sh.kv_heads, a.splits, a.M);
  cfg.blockDim = dim3((NREP + (RING ? 1 : 0)) * 32);
  cfg.dynamicSmemBytes = RING ? kRingBytes : 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = CL;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  if (usable == 0) {
    bool ok = CL <= 8 ||
              cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                  cudaSuccess;
    int n = 0;
    cfg.numAttrs = 1;
    ok = ok && cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess;
    if (!ok) cudaGetLastError();  // a refused size is an answer, not an error to keep
    usable = ok && n >= 1 ? 1 : 2;
    if (slot) slot->store(usable, std::memory_order_relaxed);
  }
  if (usable != 1) return false;
  cfg.numAttrs = 2;
  err = cudaLaunchKernelEx(&cfg, kern, a);
  return true;
}

template <typename Act, int NREP>
cudaError_t launch_decode_t(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  // splits of a (row, kv head) merged inside a cluster when they tile it,
  // for steps of few rows (measured: with 32 rows the cluster placement
  // costs more than the merge saves, 1604 vs 1803 tok/s)
  cudaError_t err = cudaSuccess;
  if (a.M > 4) {
    // plain form below
  } else if (a.page_ring) {
    if (a.splits % 16 == 0 && launch_cluster<Act, NREP, 16, true>(a, s, pdl, err)) return err;
    if (a.splits % 8 == 0 && launch_cluster<Act, NREP, 8, true>(a, s, pdl, err)) return err;
  } else {
    if constexpr (NREP == 4) {
      if (a.tok_split >= 2) {
        if (a.splits % 16 == 0 && launch_cluster<Act, NREP, 16, false, true>(a, s, pdl, err))
          return err;
        if (a.splits % 8 == 0 && launch_cluster<Act, NREP, 8, false, true>(a, s, pdl, err))
          return err;
      }
    }
    if (a.splits % 16 == 0 && launch_cluster<Act, NREP, 16, false>(a, s, pdl, err)) return err;
    if (a.splits % 8 == 0 && launch_cluster<Act, NREP, 8, false>(a, s, pdl, err)) return err;
  }
  // token split for steps of many rows (groups of 4 query heads); it takes
  // precedence over the page ring
  const bool ts = NREP == 4 && a.tok_split && a.M > 4;
  const bool ring = a.page_ring && !ts;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.sh.kv_heads, a.splits, a.M);
  cfg.blockDim = dim3((NREP + (ring ? 1 : 0)) * 32);
  cfg.dynamicSmemBytes = ring ? kRingBytes : 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (NREP == 4) {
    if (ts) return cudaLaunchKernelEx(&cfg, attn_decode_ts_kernel<Act, NREP, kTokSplitPages>, a);
  }
  return ring ? cudaLaunchKernelEx(&cfg, attn_decode_ring_kernel<Act, NREP, 0>, a)
              : cudaLaunchKernelEx(&cfg, attn_decode_kernel<Act, NREP>, a);
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
  // steps of many rows: the tensor-core form when the pool size is known
  if (a.M > 4 && a.num_blocks > 0 && attn_decode_mma_supported(a))
    return attn_decode_mma_launch(a, act, s, pdl);
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
  if (attn_prefill_tc_supported(a, act)) return attn_prefill_tc_launch(a, s);
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
