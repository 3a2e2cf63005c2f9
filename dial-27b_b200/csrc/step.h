// Host interface of the persistent decode-step kernel (step.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "attention.h"
#include "qlinear.h"

namespace dialb200 {

enum StepOpKind : int {
  kOpEmbed = 0,  // hidden[m] = embedding[tok_in[m]]
  kOpGemv = 1,   // one decoder linear (or the lm_head) with its fused prologue/epilogue
  kOpAttn = 2,   // q/k norm + RoPE + KV append + split-KV attention of one layer
};

struct StepOp {
  int kind;
  int epi;             // GemvEpilogue (kOpGemv)
  DevQLinear w;
  const void* x;       // [M][x_ld]
  int x_ld;
  const void* norm_w;  // RMSNorm weight [K] or null
  void* out;           // [M][out_ld]; may be null for the argmax head
  int out_ld;
  int S;               // ring stages per 16-row tile (ceil(C / 16))
  AttnDecodeArgs attn; // kOpAttn
};

struct StepArgs {
  const StepOp* ops;   // device array
  int n_ops;
  int M;               // rows (decode tokens), 1..kStepMaxM
  float eps;
  const void* embed;   // [vocab][H]
  int vocab, H;
  const int32_t* tok_in;
  void* hidden;        // [M][H]
  unsigned int* bar;   // grid barrier counter, zero at launch
  int* tile_cnt;       // per-tile arrival counters, zero on entry and exit
  float* tile_part;    // [grid][2][128] partial tile sums
  unsigned long long* amax_key;  // [M], zero on entry and exit
  int* amax_count;     // zero on entry and exit
  int32_t* tok_out;    // [M] sampled ids
  int32_t* tok_loop;   // device loop: tokens <- sampled (null: off)
  int32_t* pos_loop;   // device loop: positions += 1 (null: off)
  int* status;
  // Optional trace [n_ops][kTraceFields] (zeroed before the launch): per op
  // the latest CTA start (after the grid wait), the latest end of staging,
  // the latest and (as kTraceBig - t) the earliest CTA end, in %globaltimer ns.
  unsigned long long* trace;
};

constexpr int kStepMaxM = 8;
constexpr int kTraceFields = 4;
constexpr unsigned long long kTraceBig = 1ull << 62;

struct StepPlan {
  int slots, xs_stride;
  int x_off, red_off, tv_off, misc_off, attn_off, bar_off, total;
};

// Shared-memory plan for activations up to k_pad_max columns, `rows` rows;
// slots < 2 means the program does not fit.
StepPlan step_plan(int k_pad_max, int rows);

// Cooperative launch of one CTA per SM (grid <= SM count).  act: 0 = bf16,
// 1 = f16; nrep = q heads per kv head (1, 2, 4, 5 or 8).
cudaError_t step_launch(const StepArgs& a, const StepPlan& p, int act, int nrep, int grid,
                        cudaStream_t s);

}  // namespace dialb200
