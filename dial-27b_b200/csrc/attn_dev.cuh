// Device-side decode attention over the paged KV cache, shared by the
// decode attention kernels (attention.cu).
//
// One work item = (row m, kv head, split): NREP warps (one per query head of
// the GQA group) run q-norm + RoPE, the item whose span holds the new token
// normalizes/rotates its K, appends K/V to the pages and scores it from
// shared memory, then an f32 online softmax over the span.  With several
// splits the partials land in scratch and the last item to arrive on the
// (row, kv head) counter combines them and writes the output.  In the
// token-split form (TSG > 0) the NREP warps instead share each page's tokens,
// each scoring its share for every query head of the group, and merge their
// per-head partials in shared memory before that combine.
//
// Reference: text.rs:1466-1467,1513-1514 (q/k norm), 1143-1153 (RoPE),
// llama3/cache.rs:169-237 (KV append), text.rs:1258-1281 (grouped decode).
#pragma once

#include <cmath>

#include "attention.h"
#include "common.cuh"

namespace dialb200 {

// A block id read from a caller's block table: when the pool size is known
// (num_blocks > 0) an id outside [0, num_blocks) records kStatusBadArgs and
// reads (and appends to) page 0 instead, so a bad table cannot reach memory
// outside the pools.
template <typename Args>
__device__ __forceinline__ int checked_block(const Args& a, int blk) {
  if (a.num_blocks > 0 && static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks)) {
    set_status(a.status, kStatusBadArgs);
    return 0;
  }
  return blk;
}

constexpr int kHeadDim = 128;

template <typename Act>
__device__ __forceinline__ void load4(const Act* p, float (&v)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const Act* h = reinterpret_cast<const Act*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = ActTraits<Act>::to_f(h[e]);
}

// L2-coherent load for data another CTA of the same grid may have written.
template <typename Act>
__device__ __forceinline__ void load4_cg(const Act* p, float (&v)[4]) {
  const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(p));
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
// (lane l: dims 4l..4l+3), with the norm weight (w) and the cos/sin values
// of dims (l % 16) * 4 .. +3 (c, s) already in registers.  Rounding points:
// m = act(sqrt(ss/d + eps)), y = act(act(x/m) * w); RoPE element ops rounded
// to act (candle CPU forms); the partner of dim i is i +/- d/2 (lane l^16).
template <typename Act>
__device__ __forceinline__ void norm_rope_pre(float (&x)[4], const float (&w)[4], float eps,
                                              const float (&c)[4], const float (&s)[4], int lane) {
  using AT = ActTraits<Act>;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = fmaf(x[e], x[e], ss);
  ss = warp_sum(ss);
  const float m = AT::round(__fsqrt_rn(__fdiv_rn(ss, static_cast<float>(kHeadDim)) + eps));
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = AT::round(AT::round(__fdiv_rn(x[e], m)) * w[e]);
  float partner[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
  const bool first = lane < 16;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float x1 = first ? x[e] : partner[e];
    const float x2 = first ? partner[e] : x[e];
    x[e] = first ? AT::round(AT::round(x1 * c[e]) - AT::round(x2 * s[e]))
                 : AT::round(AT::round(x1 * s[e]) + AT::round(x2 * c[e]));
  }
}

template <typename Act>
__device__ __forceinline__ void norm_rope(float (&x)[4], const Act* norm_w, float eps,
                                          const Act* cos_row, const Act* sin_row, int lane) {
  float w[4], c[4], s[4];
  load4(norm_w + lane * 4, w);
  load4(cos_row + (lane & 15) * 4, c);
  load4(sin_row + (lane & 15) * 4, s);
  norm_rope_pre<Act>(x, w, eps, c, s, lane);
}

// A row's context is cut into at most `max_splits` spans of >= 16 tokens.
constexpr int kMinSplitTokens = 16;

// Splits a row of context `ctx` uses: at most max_splits, at least
// min_tokens (kMinSplitTokens when 0) context tokens per split.
__host__ __device__ __forceinline__ int active_splits(int ctx, int max_splits,
                                                      int min_tokens = 0) {
  const int mt = min_tokens > 0 ? min_tokens : kMinSplitTokens;
  const int need = (ctx + mt - 1) / mt;
  return need < max_splits ? (need < 1 ? 1 : need) : max_splits;
}

__device__ __forceinline__ int lane_of_token(int t) {
  return (((t >> 3) & 1) << 4) | (((t >> 2) & 1) << 3) | (((t >> 1) & 1) << 2) | ((t & 1) << 1);
}

// Scratch shared by the NREP warps of one item.
struct AttnItemSmem {
  float kn[kHeadDim];
  float vn[kHeadDim];
  int last;
};

// Largest cluster: rank 0 issues all of its peers' loads at once.
constexpr int kMaxClusterLoads = 16;

// Per-CTA partials of the cluster combine, read by the cluster's rank-0 CTA
// through distributed shared memory (16-byte vector stores and loads).
template <int NREP>
struct __align__(16) AttnClusterSmem {
  float o[NREP][kHeadDim];
  float ml[NREP][2];
};

// Token-split form (register pages, many rows): the group's query heads
// after norm + RoPE, and each warp's partial (o, m, l) for every head of the
// group, merged per head after the span.
template <int NREP>
struct __align__(16) AttnTokSplitSmem {
  float q[NREP][kHeadDim];
  float o[NREP][NREP][kHeadDim];
  float ml[NREP][NREP][2];
};

__device__ __forceinline__ uint32_t cluster_map(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Every thread of every CTA of the cluster (shared-memory writes before it
// are visible to the cluster after it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Bytes of one page of one kv head (K or V): 16 tokens x 128 dims x 2 B.
constexpr int kPageBytes = kPageTokens * kHeadDim * 2;

// Producer warp of the ring form of attn_item: lane 0 streams the span's K
// and V pages of (row m, kv head, split) into the ring with bulk copies and
// waits (bounded) for them all to land; the warp then joins the cluster
// barriers of the query warps.  With a.rows_ready it reads the session,
// position and block table and issues the copies before griddepcontrol.wait
// (the page holding the new position is read stale; its new row is taken
// from q/k/v by the query warps).  Geometry as in attn_item.
template <int CL, int RING>
__device__ void attn_ring_producer(const AttnDecodeArgs& a, int m, int kvh, int split, int lane,
                                   uint8_t* ring, uint64_t* rfull, uint64_t* rempty) {
  if (a.rows_ready == 0) pdl_wait();
  const int sid = a.sid[m];
  int pos = a.pos[m];
  if (pos < 0 || pos >= a.sh.max_pos || pos / kPageTokens >= a.sh.max_blocks) pos = 0;
  const int ctx = pos + 1;
  const int S = active_splits(ctx, a.splits, a.min_split_tokens);
  bool active = true;
  if constexpr (CL > 0) {
    if (split / CL * CL >= S) return;
    active = split < S;
  } else {
    if (split >= S) return;
  }
  const int span = ((ctx + S - 1) / S + kPageTokens - 1) / kPageTokens * kPageTokens;
  const int tok0 = split * span;
  const int tok1 = active ? min(ctx, tok0 + span) : tok0;
  if (tok1 > tok0) {
    const int KVH = a.sh.kv_heads;
    const int32_t* bt = a.block_table + static_cast<size_t>(sid) * a.sh.max_blocks;
    const uint8_t* kpool = static_cast<const uint8_t*>(a.kv.k);
    const uint8_t* vpool = static_cast<const uint8_t*>(a.kv.v);
    const int pg_first = tok0 / kPageTokens;
    const int npages = (tok1 - tok0 + kPageTokens - 1) / kPageTokens;
    // the warp loads the block ids 32 at a time; lane 0 issues the copies
    int issued = 0, bt_lane = 0;
    bool ok = true;
    for (int pg = 0; pg < npages && ok; ++pg) {
      if ((pg & 31) == 0) bt_lane = pg + lane < npages ? checked_block(a, bt[pg_first + pg + lane]) : 0;
      const int blk = __shfl_sync(0xffffffffu, bt_lane, pg & 31);
      if (lane == 0) {
        const int slot = pg % RING;
        if (pg >= RING && !mbar_wait(&rempty[slot], static_cast<uint32_t>(pg / RING - 1) & 1u,
                                     a.status, kStatusAttnRing)) {
          ok = false;
        } else {
          const size_t off = (static_cast<size_t>(blk) * KVH + kvh) * kPageBytes;
          mbar_arrive_expect_tx(&rfull[slot], 2 * kPageBytes);
          bulk_g2s(ring + slot * (2 * kPageBytes), kpool + off, kPageBytes, &rfull[slot]);
          bulk_g2s(ring + slot * (2 * kPageBytes) + kPageBytes, vpool + off, kPageBytes,
                   &rfull[slot]);
          ++issued;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    // copies in flight must land before the CTA retires
    if (lane == 0)
      for (int pg = issued > RING ? issued - RING : 0; pg < issued; ++pg)
        if (!mbar_wait(&rfull[pg % RING], static_cast<uint32_t>(pg / RING) & 1u, a.status,
                       kStatusAttnRing))
          break;
  }
  __syncwarp();
  if constexpr (CL > 0) {
    cluster_sync_all();  // the query warps' partial exchange
    cluster_sync_all();
  }
}

// Combine of S_parts partial rows (m, l, acc) of (row m, kv head) through the
// scratch buffer: partial idx is stored, the last arrival on the (row, kv
// head) counter merges all of them, writes the output and resets the counter.
template <typename Act, int NREP, typename Sync>
__device__ void attn_global_combine(const AttnDecodeArgs& a, int m, int kvh, int h, int r,
                                    int lane, AttnItemSmem& sm, Sync group_sync, int S_parts,
                                    int idx, const float (&acc)[4], float mrun, float lrun,
                                    Act* out) {
  const int QH = a.sh.q_heads, KVH = a.sh.kv_heads;
  // partial rows are laid out with the allocation stride a.splits
  const size_t prow = (static_cast<size_t>(m) * QH + h) * a.splits;
  __stcg(reinterpret_cast<float4*>(a.part_o + (prow + idx) * kHeadDim + lane * 4),
         make_float4(acc[0], acc[1], acc[2], acc[3]));
  if (lane == 0) {
    __stcg(a.part_ml + (prow + idx) * 2, mrun);
    __stcg(a.part_ml + (prow + idx) * 2 + 1, lrun);
  }
  group_sync();
  if (r == 0 && lane == 0) {
    __threadfence();
    const int old = atomicAdd(a.counters + m * KVH + kvh, 1);
    sm.last = (old == S_parts - 1);
  }
  group_sync();
  const bool last = sm.last != 0;
  if (last) {
    __threadfence();
    // lane s2 < S_parts holds partial s2's (m, l); weights are broadcast by shuffles
    float ms_l = -INFINITY, ls_l = 0.f;
    if (lane < S_parts) {
      ms_l = __ldcg(a.part_ml + (prow + lane) * 2);
      ls_l = __ldcg(a.part_ml + (prow + lane) * 2 + 1);
    }
    const float M = warp_max(ms_l);
    const float w_l = (lane < S_parts && ms_l != -INFINITY) ? expf(ms_l - M) : 0.f;
    const float L = warp_sum(w_l * ls_l);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < S_parts; s0 += 8) {
      float4 po[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        po[u] = (s0 + u < S_parts)
                    ? __ldcg(reinterpret_cast<const float4*>(a.part_o + (prow + s0 + u) * kHeadDim + lane * 4))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = __shfl_sync(0xffffffffu, w_l, (s0 + u) & 31);
        if (s0 + u < S_parts) {
          o[0] = fmaf(w, po[u].x, o[0]);
          o[1] = fmaf(w, po[u].y, o[1]);
          o[2] = fmaf(w, po[u].z, o[2]);
          o[3] = fmaf(w, po[u].w, o[3]);
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= inv;
    store4(out, o);
  }
  group_sync();
  if (last && r == 0 && lane == 0) a.counters[m * KVH + kvh] = 0;
}

// Process item (m, kvh, split) of `a` with NREP warps; `r` = this warp's
// index in the group, `bar_id` a named barrier owned by the group.  PDL: the
// item executes griddepcontrol.wait itself, after the reads that a.rows_ready
// allows before it (block ids, the span's first K/V page, norm weights and
// RoPE rows); an item with nothing to do then exits without waiting.
//
// CL > 0: the CTAs of item splits [c*CL, (c+1)*CL) form one thread-block
// cluster; each keeps its partial in `cs` and the cluster's rank-0 CTA merges
// the active ones over distributed shared memory (one cluster covering all
// active splits writes the output directly; otherwise the cluster partials
// take the scratch-buffer combine).  Splits past the active count in an
// active cluster only join the two cluster barriers.
//
// RING > 0: the span's pages come from a shared-memory ring of RING pages
// (K page then V page, 4 KB each; full[] / empty[] mbarriers) that the
// CTA's producer warp fills (attn_ring_producer); the query warps read each
// page from shared memory and release its slot.
template <typename Act, int NREP, bool PDL = false, int CL = 0, int RING = 0, int TSG = 0>
__device__ void attn_item(const AttnDecodeArgs& a, int m, int kvh, int split, int r, int lane,
                          AttnItemSmem& sm, int bar_id, AttnClusterSmem<NREP>* csm = nullptr,
                          const uint8_t* ring = nullptr, uint64_t* rfull = nullptr,
                          uint64_t* rempty = nullptr, AttnTokSplitSmem<NREP>* tss = nullptr) {
  static_assert(TSG == 0 || (RING == 0 && kPageTokens % NREP == 0 && 32 % (TSG > 0 ? TSG : 1) == 0),
                "token split: register pages, NREP | 16, TSG | 32");
  using AT = ActTraits<Act>;
  const int QH = a.sh.q_heads, KVH = a.sh.kv_heads;
  const int h = kvh * NREP + r;
  auto group_sync = [&]() { named_bar_sync(bar_id, NREP * 32); };
  const bool early = PDL && a.rows_ready != 0;
  if (PDL && !early) pdl_wait();

  const int sid = a.sid[m];
  int pos = a.pos[m];
  const bool bad = pos < 0 || pos >= a.sh.max_pos || pos / kPageTokens >= a.sh.max_blocks;
  if (bad) {
    if (lane == 0 && r == 0) set_status(a.status, kStatusBadArgs);
    pos = 0;
  }
  const int ctx = pos + 1;
  const int32_t* bt = a.block_table + static_cast<size_t>(sid) * a.sh.max_blocks;
  // Splits actually used by this row: short contexts skip the partial/combine
  // round trip.  Uniform over the group, so every warp returns together.
  const int S = active_splits(ctx, a.splits, a.min_split_tokens);
  bool active = true;
  if constexpr (CL > 0) {
    if (split / CL * CL >= S) return;  // the whole cluster is idle: uniform over it
    active = split < S;
  } else {
    if (split >= S) return;
  }
  const int span = ((ctx + S - 1) / S + kPageTokens - 1) / kPageTokens * kPageTokens;
  const int tok0 = split * span;
  const int tok1 = active ? min(ctx, tok0 + span) : tok0;
  const bool owner = tok0 <= pos && pos < tok1;
  const int pg_first = tok0 / kPageTokens;
  const int npg = (tok1 - tok0 + kPageTokens - 1) / kPageTokens;

  const Act* qkv = reinterpret_cast<const Act*>(a.qkv) + static_cast<size_t>(m) * a.qkv_ld;
  const Act* cos_row = reinterpret_cast<const Act*>(a.cos) + static_cast<size_t>(pos) * (kHeadDim / 2);
  const Act* sin_row = reinterpret_cast<const Act*>(a.sin) + static_cast<size_t>(pos) * (kHeadDim / 2);
  Act* kpool = reinterpret_cast<Act*>(a.kv.k);
  Act* vpool = reinterpret_cast<Act*>(a.kv.v);
  const bool do_kv = owner && r == 0 && !bad;

  // Issue every load that does not depend on another one first: the block
  // id of the span's first page, q (and the new k/v), norm weights, cos/sin.
  const int blk_first = (RING == 0 && active) ? checked_block(a, bt[tok0 / kPageTokens]) : 0;
  // the other block ids of the span's first 32 pages (register form)
  const int bt_lane0 =
      (RING == 0 && active && lane < npg) ? checked_block(a, bt[pg_first + lane]) : 0;
  const int blk_pos = do_kv ? checked_block(a, bt[pos / kPageTokens]) : 0;
  float q[4], kn[4] = {0.f, 0.f, 0.f, 0.f}, vn[4] = {0.f, 0.f, 0.f, 0.f};
  if (!early) {
    load4_cg(qkv + h * kHeadDim + lane * 4, q);
    if (do_kv) {
      load4_cg(qkv + (QH + kvh) * kHeadDim + lane * 4, kn);
      load4_cg(qkv + (QH + KVH + kvh) * kHeadDim + lane * 4, vn);
    }
  }
  float qw[4], kw[4], cs[4], sn[4];
  load4(reinterpret_cast<const Act*>(a.q_norm_w) + lane * 4, qw);
  load4(reinterpret_cast<const Act*>(a.k_norm_w) + lane * 4, kw);
  load4(cos_row + (lane & 15) * 4, cs);
  load4(sin_row + (lane & 15) * 4, sn);
  // first page's K/V (depends only on the block id)
  uint2 kr[kPageTokens], vr[kPageTokens];
  // token-split form: TSG pages at a time, TPW tokens of each for this warp
  constexpr int TPW = TSG > 0 ? kPageTokens / NREP : 1;
  constexpr int TG = TSG > 0 ? TSG : 1;
  uint2 kg[TG][TPW], vg[TG][TPW];
  auto load_group = [&](int pg0, int bt_l) {
#pragma unroll
    for (int p = 0; p < TG; ++p) {
      const int blk = __shfl_sync(0xffffffffu, bt_l, (pg0 + p) & 31);
      if (pg0 + p < npg) {
        const size_t base =
            ((static_cast<size_t>(blk) * KVH + kvh) * kPageTokens + r * TPW) * kHeadDim + lane * 4;
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          kg[p][t] = *reinterpret_cast<const uint2*>(kpool + base + t * kHeadDim);
          vg[p][t] = *reinterpret_cast<const uint2*>(vpool + base + t * kHeadDim);
        }
      }
    }
  };
  if constexpr (TSG > 0) {
    if (active) load_group(0, bt_lane0);
  }
  if (RING == 0 && TSG == 0 && active) {
    const size_t base =
        (static_cast<size_t>(blk_first) * KVH + kvh) * kPageTokens * kHeadDim + lane * 4;
#pragma unroll
    for (int j = 0; j < kPageTokens; ++j) {
      kr[j] = *reinterpret_cast<const uint2*>(kpool + base + j * kHeadDim);
      vr[j] = *reinterpret_cast<const uint2*>(vpool + base + j * kHeadDim);
    }
  }
  if (early) {
    // the row pos[m] of this page is the new token: it is taken from q/k/v
    // below, never from the (not yet written) page
    pdl_wait();
    load4_cg(qkv + h * kHeadDim + lane * 4, q);
    if (do_kv) {
      load4_cg(qkv + (QH + kvh) * kHeadDim + lane * 4, kn);
      load4_cg(qkv + (QH + KVH + kvh) * kHeadDim + lane * 4, vn);
    }
  }

  norm_rope_pre<Act>(q, qw, a.sh.eps, cs, sn, lane);
  if constexpr (TSG > 0)
    *reinterpret_cast<float4*>(&tss->q[r][lane * 4]) = make_float4(q[0], q[1], q[2], q[3]);
  if (do_kv) {
    norm_rope_pre<Act>(kn, kw, a.sh.eps, cs, sn, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sm.kn[lane * 4 + e] = kn[e];
      sm.vn[lane * 4 + e] = vn[e];
    }
  }
  // The new token's K/V reach the pages last (no later read in this launch
  // needs them): no fence or barrier release below waits for these stores.
  auto append_kv = [&]() {
    if (do_kv) {
      const size_t off =
          ((static_cast<size_t>(blk_pos) * KVH + kvh) * kPageTokens + (pos % kPageTokens)) *
              kHeadDim + lane * 4;
      store4(kpool + off, kn);
      store4(vpool + off, vn);
    }
  };
  group_sync();

  const float scale = AT::round(1.0f / sqrtf(static_cast<float>(kHeadDim)));
  float mrun = -INFINITY, lrun = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int my_tok = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                     ((lane >> 1) & 1);

  // block ids of the span's pages, 32 at a time: lane l holds page (32i + l)
  int bt_lane = bt_lane0;
  if constexpr (TSG == 0) {
    for (int b0 = tok0, pg = 0; b0 < tok1; b0 += kPageTokens, ++pg) {
      if (RING == 0 && (pg & 31) == 0 && pg > 0)
        bt_lane = pg + lane < npg ? checked_block(a, bt[pg_first + pg + lane]) : 0;
      if constexpr (RING > 0) {
        // the page's K/V rows (lane: dims 4*lane.. of every token) from the ring
        const int slot = pg % RING;
        mbar_wait(&rfull[slot], static_cast<uint32_t>(pg / RING) & 1u, a.status, kStatusAttnRing);
        const uint8_t* kp = ring + slot * (2 * kPageBytes);
        const uint8_t* vp = kp + kPageBytes;
#pragma unroll
        for (int j = 0; j < kPageTokens; ++j) {
          kr[j] = *reinterpret_cast<const uint2*>(kp + j * kHeadDim * 2 + lane * 8);
          vr[j] = *reinterpret_cast<const uint2*>(vp + j * kHeadDim * 2 + lane * 8);
        }
        fence_proxy_async_smem();  // these reads before the copy that refills the slot
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[slot]);
      } else if (b0 != tok0) {
        const int blk = __shfl_sync(0xffffffffu, bt_lane, pg & 31);
        const size_t base = (static_cast<size_t>(blk) * KVH + kvh) * kPageTokens * kHeadDim + lane * 4;
#pragma unroll
        for (int j = 0; j < kPageTokens; ++j) {
          kr[j] = *reinterpret_cast<const uint2*>(kpool + base + j * kHeadDim);
          vr[j] = *reinterpret_cast<const uint2*>(vpool + base + j * kHeadDim);
        }
      }
      float v16[kPageTokens];
#pragma unroll
      for (int j = 0; j < kPageTokens; ++j) {
        const Act* kh = reinterpret_cast<const Act*>(&kr[j]);
        float d = 0.f;
        if (owner && b0 + j == pos) {
#pragma unroll
          for (int e = 0; e < 4; ++e) d = fmaf(q[e], sm.kn[lane * 4 + e], d);
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
          for (int e = 0; e < 4; ++e) acc[e] = fmaf(pj, sm.vn[lane * 4 + e], acc[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] = fmaf(pj, AT::to_f(vh[e]), acc[e]);
        }
      }
      mrun = mnew;
    }
  } else {
    // Token-split scan: warp r takes tokens r*TPW .. r*TPW+TPW-1 of every
    // page for all NREP query heads of the group.  The reduce-scatter leaves
    // lane pair (2i, 2i+1) with the score of (head i / TPW, token i % TPW);
    // each warp keeps an online softmax per head, merged below.
    float qa[NREP][4], oa[NREP][4];
#pragma unroll
    for (int hh = 0; hh < NREP; ++hh) {
      const float4 v = *reinterpret_cast<const float4*>(&tss->q[hh][lane * 4]);
      qa[hh][0] = v.x;
      qa[hh][1] = v.y;
      qa[hh][2] = v.z;
      qa[hh][3] = v.w;
#pragma unroll
      for (int e = 0; e < 4; ++e) oa[hh][e] = 0.f;
    }
    const int my_h = my_tok / TPW, my_t = my_tok % TPW;
    float mh = -INFINITY, lh = 0.f;
    for (int pg0 = 0; pg0 < npg; pg0 += TSG) {
      if (pg0 > 0) {
        if ((pg0 & 31) == 0) bt_lane = pg0 + lane < npg ? checked_block(a, bt[pg_first + pg0 + lane]) : 0;
        load_group(pg0, bt_lane);
      }
#pragma unroll
      for (int p = 0; p < TG; ++p) {
        if (pg0 + p >= npg) break;
        const int t0 = tok0 + (pg0 + p) * kPageTokens + r * TPW;  // this warp's first token
        float v16[kPageTokens];
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          const bool fresh = owner && t0 + t == pos;
          const Act* kh = reinterpret_cast<const Act*>(&kg[p][t]);
          float kf[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) kf[e] = fresh ? sm.kn[lane * 4 + e] : AT::to_f(kh[e]);
#pragma unroll
          for (int hh = 0; hh < NREP; ++hh) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) d = fmaf(qa[hh][e], kf[e], d);
            v16[hh * TPW + t] = d;
          }
        }
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
        const bool valid = t0 + my_t < tok1;
        s = valid ? AT::round(AT::round(s) * scale) : -INFINITY;
        // the head's TPW tokens sit on lane bits 1 .. log2(TPW)
        float bm = s;
#pragma unroll
        for (int k = 2; k < 2 * TPW; k <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, k));
        const float mnew = fmaxf(mh, bm);
        const float pr = valid ? expf(s - mnew) : 0.f;
        const float alpha = mnew == -INFINITY ? 1.f : expf(mh - mnew);
        float ls = pr;
#pragma unroll
        for (int k = 2; k < 2 * TPW; k <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, k);
        lh = lh * alpha + ls;
        mh = mnew;
        float vf[TPW][4];
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          const bool fresh = owner && t0 + t == pos;
          const Act* vh = reinterpret_cast<const Act*>(&vg[p][t]);
#pragma unroll
          for (int e = 0; e < 4; ++e) vf[t][e] = fresh ? sm.vn[lane * 4 + e] : AT::to_f(vh[e]);
        }
#pragma unroll
        for (int hh = 0; hh < NREP; ++hh) {
          const float ah = __shfl_sync(0xffffffffu, alpha, lane_of_token(hh * TPW));
#pragma unroll
          for (int e = 0; e < 4; ++e) oa[hh][e] *= ah;
#pragma unroll
          for (int t = 0; t < TPW; ++t) {
            const float pj = __shfl_sync(0xffffffffu, pr, lane_of_token(hh * TPW + t));
#pragma unroll
            for (int e = 0; e < 4; ++e) oa[hh][e] = fmaf(pj, vf[t][e], oa[hh][e]);
          }
        }
      }
    }
    // merge the warps' partials: warp r ends with query head r's (m, l, o)
#pragma unroll
    for (int hh = 0; hh < NREP; ++hh)
      *reinterpret_cast<float4*>(&tss->o[r][hh][lane * 4]) =
          make_float4(oa[hh][0], oa[hh][1], oa[hh][2], oa[hh][3]);
    if ((lane & 1) == 0 && my_t == 0) {
      tss->ml[r][my_h][0] = mh;
      tss->ml[r][my_h][1] = lh;
    }
    group_sync();
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NREP; ++w) mx = fmaxf(mx, tss->ml[w][r][0]);
#pragma unroll
    for (int w = 0; w < NREP; ++w) {
      const float mw = tss->ml[w][r][0];
      const float wt = mw == -INFINITY ? 0.f : expf(mw - mx);
      lrun = fmaf(wt, tss->ml[w][r][1], lrun);
      const float4 ov = *reinterpret_cast<const float4*>(&tss->o[w][r][lane * 4]);
      acc[0] = fmaf(wt, ov.x, acc[0]);
      acc[1] = fmaf(wt, ov.y, acc[1]);
      acc[2] = fmaf(wt, ov.z, acc[2]);
      acc[3] = fmaf(wt, ov.w, acc[3]);
    }
    mrun = mx;
  }

  Act* out =
      reinterpret_cast<Act*>(a.out) + static_cast<size_t>(m) * a.out_ld + h * kHeadDim + lane * 4;
  if constexpr (CL > 0) {
    if (active) {
      *reinterpret_cast<float4*>(&csm->o[r][lane * 4]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      if (lane == 0) {
        csm->ml[r][0] = mrun;
        csm->ml[r][1] = lrun;
      }
    }
    cluster_sync_all();
    const bool leader = split % CL == 0;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    float Mx = -INFINITY, L = 0.f;
    if (leader) {
      // warp r merges query head h over the cluster's active splits
      const int nact = min(S, split + CL) - split;
      float ms_l = -INFINITY, ls_l = 0.f;
      if (lane < nact) {
        const uint32_t pm = cluster_map(&csm->ml[r][0], lane);
        ms_l = ld_dsmem_f32(pm);
        ls_l = ld_dsmem_f32(pm + 4);
      }
      Mx = warp_max(ms_l);
      const float w_l = (lane < nact && ms_l != -INFINITY) ? expf(ms_l - Mx) : 0.f;
      L = warp_sum(w_l * ls_l);
      float4 po[kMaxClusterLoads];
#pragma unroll
      for (int u = 0; u < kMaxClusterLoads; ++u)
        po[u] = u < nact ? ld_dsmem_v4(cluster_map(&csm->o[r][lane * 4], u))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kMaxClusterLoads; ++u) {
        const float w = __shfl_sync(0xffffffffu, w_l, u);
        o[0] = fmaf(w, po[u].x, o[0]);
        o[1] = fmaf(w, po[u].y, o[1]);
        o[2] = fmaf(w, po[u].z, o[2]);
        o[3] = fmaf(w, po[u].w, o[3]);
      }
    }
    // peers keep their partials until rank 0 has read them; the stores come
    // after, so neither barrier waits on a global write
    cluster_sync_all();
    if (leader) {
      if (S <= CL) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] *= inv;
        store4(out, o);
      } else {
        attn_global_combine<Act, NREP>(a, m, kvh, h, r, lane, sm, group_sync, (S + CL - 1) / CL,
                                       split / CL, o, Mx, L, out);
      }
    }
    append_kv();
    return;
  }
  if (S == 1) {
    float o[4];
    const float inv = lrun > 0.f ? 1.f / lrun : 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = acc[e] * inv;
    store4(out, o);
    append_kv();
    group_sync();  // kn/vn reuse by the group's next item
    return;
  }

  attn_global_combine<Act, NREP>(a, m, kvh, h, r, lane, sm, group_sync, S, split, acc, mrun,
                                 lrun, out);
  append_kv();
}

}  // namespace dialb200
