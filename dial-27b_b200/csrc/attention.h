// Host interface of the attention kernels (attention.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dialb200 {

constexpr int kPageTokens = 16;  // tokens per paged-KV block

// Paged KV pool of one layer: [num_blocks][kv_heads][16][head_dim] (act dtype).
struct KvLayer {
  void* k;
  void* v;
};

struct AttnShape {
  int q_heads, kv_heads, head_dim;
  int max_blocks;      // block-table row length
  int max_pos;         // rows of the cos/sin tables
  float eps;
};

// Decode: M rows, each one new token of session sid[m] at position pos[m].
struct AttnDecodeArgs {
  AttnShape sh;
  const void* qkv;           // [M][qkv_ld]: q | k | v (pre-norm, pre-RoPE)
  int qkv_ld;
  const void* q_norm_w;      // [head_dim]
  const void* k_norm_w;      // [head_dim]
  const void* cos;           // [max_pos][head_dim/2]
  const void* sin;
  KvLayer kv;
  const int32_t* block_table;// [num_sessions][max_blocks]
  const int32_t* sid;        // [M]
  const int32_t* pos;        // [M]
  void* out;                 // [M][q_heads*head_dim]
  int out_ld;
  int M;
  int splits;                // KV splits per (row, kv head); 1 = no scratch use.
  int min_split_tokens;      // context tokens per split at least (0: 16)
                             // Each row's context is cut into `splits` equal
                             // 16-token-aligned spans at run time.
  float* part_o;             // [M][q_heads][splits][head_dim]
  float* part_ml;            // [M][q_heads][splits][2]
  int* counters;             // [M][kv_heads], zero on entry, left zero on exit
  int* status;
  // 1: sid, pos, the block table and the KV pages of positions < pos[m] are
  // complete before the launch (nothing a programmatically overlapped
  // predecessor writes), so the kernel reads them before griddepcontrol.wait
  // and waits only for q / k / v.  0: everything is read after the wait.
  int rows_ready;
  // 1: a producer warp streams each split's K/V pages through a shared-memory
  // ring (bulk copies); 0: every query warp loads its pages into registers.
  int page_ring;
  // Groups of 4 query heads, register form: the group's warps split each
  // page's tokens between them, each scoring its tokens for every query head
  // of the group, and merge their partials in shared memory.  1: for steps
  // of more than 4 rows; 2: also for the cluster-merge form of 4 rows or
  // fewer; 0: every warp reads every token for its own head.
  int tok_split;
  unsigned long long* trace; // opt-in timeline records (common.cuh), null = off
  int trace_tag;
  // Pages in each of the kv.k / kv.v pools ([num_blocks][kv_heads][16][128]).
  // Non-zero selects the tensor-core form (attn_decode_mma.cu) for steps of
  // more than 4 rows; 0 keeps the CUDA-core forms.
  int num_blocks;
  int mma_ring;  // tensor-core form: page slots per warp, 2 (default) or 3
};

bool attn_decode_mma_supported(const AttnDecodeArgs& a);
cudaError_t attn_decode_mma_launch(const AttnDecodeArgs& a, int act, cudaStream_t s, bool pdl);

// Scratch bytes needed for (M, splits).
size_t attn_decode_scratch_bytes(const AttnShape& sh, int M, int splits);

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, int act, cudaStream_t s, bool pdl);

// Status word of dial_b200_attention_decode_noalloc on device `dev` (0 when
// that entry point never ran there): read into *out and, with `clear`, set to
// zero; clearing a non-zero status also re-zeroes that entry point's split
// counters, which a call that gave up early may have left non-zero.  Allocates
// nothing.
cudaError_t noalloc_status(int dev, bool clear, int* out);

// Prefill of one session: M tokens at positions p0 .. p0+M-1.
struct AttnPrefillArgs {
  AttnShape sh;
  const void* qkv;
  int qkv_ld;
  const void* q_norm_w;
  const void* k_norm_w;
  const void* cos;
  const void* sin;
  KvLayer kv;
  const int32_t* block_table;  // this session's row [max_blocks]
  int p0;
  int M;
  int32_t* rows_scratch;       // [2*M] int32 scratch (per-row positions, sessions)
  void* out;                   // [M][q_heads*head_dim]
  int out_ld;
  int* status;
  // tensor-core path (bf16, M >= 64): rotated queries [M][q_heads*head_dim]
  // scratch and the KV pool's page count; null / 0 keep the CUDA-core path
  void* q_rot;
  int num_blocks;
};

bool attn_prefill_tc_supported(const AttnPrefillArgs& a, int act);
cudaError_t attn_prefill_tc_launch(const AttnPrefillArgs& a, cudaStream_t s);

cudaError_t attn_prefill_launch(const AttnPrefillArgs& a, int act, cudaStream_t s, bool pdl);

}  // namespace dialb200
