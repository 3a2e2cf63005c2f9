/*
 * dial_b200.h -- C ABI of the B200-native DIAL decoder-layer path.
 *
 * The entry points replace, one for one, the two boundaries of the reference
 * (lisa301/DIAL-27B) on this path:
 *
 *   1. the linear custom op: candle `CustomOp1::cuda_fwd` implemented by
 *      `CudaW8A16Linear` (dial-core/src/models/qwen3_vl/worker_w8a16.rs:295-476)
 *      and `CudaQuantLinear` (dial-core/src/models/qwen3_8/cuda_quant.rs:256-500);
 *   2. the layer API: the `Forwarder` trait (dial-core/src/spm/mod.rs:230-287)
 *      as used by the Worker loop (dial-core/src/spm/worker.rs:740-796) and the
 *      Master (dial-core/src/models/qwen3_vl/qwen3_vl.rs:2018-2177), plus the
 *      per-connection KV `Cache` (dial-core/src/models/llama3/cache.rs).
 *
 * Conventions follow the reference's own C ABI (backends/qwen38_ggml/adapter.h):
 * opaque handles, an int status (0 = OK), and a caller-provided error buffer
 * that receives a NUL-terminated message.  No C++ exception crosses the ABI.
 * Device pointers are plain CUDA device addresses; `stream` is a cudaStream_t
 * (NULL = the legacy default stream).  Launches are asynchronous unless an
 * entry point says it synchronizes.  A handle is not thread-safe: serialize
 * calls per handle, as the reference serializes calls per GGML engine.
 */
#ifndef DIAL_B200_H
#define DIAL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 2: dial_b200_attn_shape gained num_blocks */
#define DIAL_B200_ABI_VERSION 2u

/* status codes */
#define DIAL_OK 0
#define DIAL_ERR_INVALID 1 /* bad argument or shape (reference: candle_core::Error::Msg) */
#define DIAL_ERR_CUDA 2    /* CUDA runtime error */
#define DIAL_ERR_DEVICE 3  /* a kernel recorded a device status (bounded wait expired, bad index) */

/* weight formats */
#define DIAL_FMT_W8A16_ROW 0    /* int8 [out,in] + f32 scale [out]      (worker_w8a16.rs:295-366) */
#define DIAL_FMT_FP8_BLOCK128 1 /* e4m3 [out,in] + f32 [ceil(out/128)][ceil(in/128)] */
#define DIAL_FMT_FP8_ROW 2      /* e4m3 [out,in] + f32 [out] or [1]     (cuda_quant.rs:58-65, 305-334) */
#define DIAL_FMT_NVFP4_G16 3    /* e2m1 packed [out,in/2] + e4m3 [out,in/16] + f32 global (cuda_quant.rs:43-56) */
#define DIAL_FMT_DENSE 4        /* activation-dtype dense [out,in] (candle Linear, lm_head) */

/* activation / tensor dtypes */
#define DIAL_ACT_BF16 0
#define DIAL_ACT_F16 1
#define DIAL_ACT_F32 2 /* source weights only */

/* Library version; replaces nothing (the reference links statically). */
uint32_t dial_b200_abi_version(void);

/* Read (and optionally clear) the device status of the current device.
 * A non-zero value names the first bounded wait that expired or the first
 * out-of-range index a kernel saw since the last clear: the word shared by
 * the engines and the scratch-taking ops, else the word of
 * dial_b200_attention_decode_noalloc (clearing also resets that entry
 * point's split counters).  Synchronizes; allocates nothing. */
int dial_b200_device_status(int* status_out, int clear, char* err, size_t err_size);

/* ------------------------------------------------------------------------ */
/* Linear op: CudaW8A16Linear / CudaQuantLinear                             */
/* ------------------------------------------------------------------------ */

typedef struct dial_b200_qlinear dial_b200_qlinear;

/* a1: row-wise symmetric int8 quantization of a dense [out_dim, in_dim]
 * weight, bit-identical to CudaW8A16Linear::from_linear
 * (worker_w8a16.rs:330-341).  `weight` is a host pointer; results go to the
 * host arrays q[out_dim*in_dim] and scale[out_dim]. */
int dial_b200_w8a16_quantize(const void* weight, int weight_dtype, int64_t out_dim, int64_t in_dim,
                             int8_t* q, float* scale, char* err, size_t err_size);

/* CudaW8A16Linear::from_linear (worker_w8a16.rs:302-366): quantize a dense
 * host weight [out_dim, in_dim] and keep it device resident.  `act` is the
 * activation dtype forward() accepts. */
int dial_b200_w8a16_from_dense(const void* weight, int weight_dtype, int64_t out_dim,
                               int64_t in_dim, int act, dial_b200_qlinear** out, char* err,
                               size_t err_size);

/* CudaQuantLinear::nvfp4 / ::fp8 (cuda_quant.rs:270-371) and the W8A16 /
 * dense formats from pre-quantized host arrays (see DIAL_FMT_* for layouts;
 * scales of NVFP4 are e4m3 codes, `global_scale` its f32 multiplier). */
int dial_b200_qlinear_create(int fmt, int act, const void* codes, const void* scales,
                             float global_scale, int64_t in_dim, int64_t out_dim,
                             dial_b200_qlinear** out, char* err, size_t err_size);

void dial_b200_qlinear_destroy(dial_b200_qlinear* lin);

/* CustomOp1::cuda_fwd (worker_w8a16.rs:402-475, cuda_quant.rs:406-499):
 * y[rows, out_dim] = x[rows, in_dim] . dequant(W)^T, both contiguous device
 * arrays of the activation dtype; y is caller-owned. */
int dial_b200_qlinear_forward(dial_b200_qlinear* lin, const void* x, void* y, int64_t rows,
                              void* stream, char* err, size_t err_size);

int64_t dial_b200_qlinear_in_dim(const dial_b200_qlinear* lin);
int64_t dial_b200_qlinear_out_dim(const dial_b200_qlinear* lin);
/* CudaQuantLinear::resident_bytes (cuda_quant.rs:345-356) */
int64_t dial_b200_qlinear_resident_bytes(const dial_b200_qlinear* lin);

/* ------------------------------------------------------------------------ */
/* Decode attention op                                                      */
/* ------------------------------------------------------------------------ */

/* Shape of the fused decode attention (head_dim must be 128). */
typedef struct {
  int32_t q_heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t max_blocks; /* block-table row length (16-token pages per session) */
  int32_t max_pos;    /* rows of the cos/sin tables */
  float eps;          /* q/k RMSNorm epsilon */
  int32_t act;        /* DIAL_ACT_BF16 or DIAL_ACT_F16 */
  int32_t num_blocks; /* pages in each of k_pages / v_pages; with more than 4
                         rows a positive value selects the tensor-core form
                         (mma.sync over TMA-staged pages), 0 the CUDA-core
                         forms.  When positive, a block id outside
                         [0, num_blocks) records the bad-argument device
                         status and page 0 is used instead.
                         dial_b200_attention_decode_noalloc ignores it */
} dial_b200_attn_shape;

/* Bytes of scratch dial_b200_attention_decode needs for `rows` rows and
 * `splits` KV splits (0 when splits == 1). */
int64_t dial_b200_attention_scratch_bytes(const dial_b200_attn_shape* sh, int64_t rows,
                                          int32_t splits);

/* One decode token per row, the fusion of QwenAttention::forward's q/k
 * RMSNorm (qwen3_vl/text.rs:1466-1467,1513-1514), RoPE (text.rs:1143-1153),
 * KV append (Cache::process_kv_decode_in_place, llama3/cache.rs:169-237) and
 * grouped_decode_attention (text.rs:1258-1281) over paged KV:
 *   qkv [rows, qkv_ld]: q | k | v of the new tokens (before norm and RoPE);
 *   k_pages / v_pages [num_blocks][kv_heads][16][128]; block_table
 *   [sessions][max_blocks]; sids / positions [rows] (device);
 *   out [rows, out_ld] receives the attention output (q_heads * 128 wide).
 * Row m appends its K/V at positions[m] of session sids[m] and attends to
 * positions 0..positions[m]; rows must name distinct sessions (a row reads
 * only keys already in the pages plus its own).  `scratch` (device, >=
 * dial_b200_attention_scratch_bytes) must be zero-filled before its first
 * use; the kernels leave it ready for the next call. */
int dial_b200_attention_decode(const dial_b200_attn_shape* sh, const void* qkv, int64_t qkv_ld,
                               const void* q_norm_w, const void* k_norm_w, const void* cos,
                               const void* sin, void* k_pages, void* v_pages,
                               const int32_t* block_table, const int32_t* sids,
                               const int32_t* positions, void* out, int64_t out_ld, int64_t rows,
                               int32_t splits, void* scratch, void* stream, char* err,
                               size_t err_size);

/* Limits of the static scratch behind dial_b200_attention_decode_noalloc. */
#define DIAL_B200_NOALLOC_MAX_PART_ROWS 2048 /* rows * q_heads * splits */
#define DIAL_B200_NOALLOC_MAX_COUNTERS 1024  /* rows * kv_heads */

/* dial_b200_attention_decode without the scratch argument: the split-KV
 * partials live in a fixed file-scope device array (about 1.07 MB per
 * device), so the call allocates nothing, for hosts that may not allocate on
 * the call path.  No counterpart in the reference (its attention allocates
 * through candle on every call).  Rejects (DIAL_ERR_INVALID) splits > 1 when
 * rows * q_heads * splits > DIAL_B200_NOALLOC_MAX_PART_ROWS or rows *
 * kv_heads > DIAL_B200_NOALLOC_MAX_COUNTERS.  The first call on a device sets
 * the scratch up (address lookup, zero fill, a synchronize): make it before
 * any stream capture.  Calls that overlap in time on one device share the
 * scratch and race: serialize them.  It runs the same kernel forms as
 * dial_b200_attention_decode.  Device-side status of this entry point (for
 * instance a position outside max_pos: that row's KV append is skipped) is
 * reported by dial_b200_device_status; after a non-zero status, clear it
 * there before the next call, which also re-zeroes the split counters. */
int dial_b200_attention_decode_noalloc(const dial_b200_attn_shape* sh, const void* qkv,
                                       int64_t qkv_ld, const void* q_norm_w, const void* k_norm_w,
                                       const void* cos, const void* sin, void* k_pages,
                                       void* v_pages, const int32_t* block_table,
                                       const int32_t* sids, const int32_t* positions, void* out,
                                       int64_t out_ld, int64_t rows, int32_t splits, void* stream,
                                       char* err, size_t err_size);

/* ------------------------------------------------------------------------ */
/* Gated-DeltaNet token mixer (Qwen3.8 hybrid linear-attention layers)      */
/* ------------------------------------------------------------------------ */

/* Shape of a Gated-DeltaNet layer (qwen3_8/config.rs:49-53; head dims must
 * be 128, conv kernel at most 8). */
typedef struct {
  int32_t k_heads;     /* linear_num_key_heads */
  int32_t v_heads;     /* linear_num_value_heads (a multiple of k_heads) */
  int32_t k_head_dim;  /* linear_key_head_dim */
  int32_t v_head_dim;  /* linear_value_head_dim */
  int32_t conv_kernel; /* linear_conv_kernel_dim */
  float eps;           /* rms_norm_eps of the gated norm */
  int32_t act;         /* DIAL_ACT_BF16 or DIAL_ACT_F16 */
} dial_b200_gdn_shape;

/* Bytes of the scratch dial_b200_gdn_forward needs for `seq_len` tokens. */
int64_t dial_b200_gdn_scratch_bytes(const dial_b200_gdn_shape* sh, int64_t seq_len);

/* GatedDeltaNet::forward (qwen3_8/text.rs:390-481) from the outputs of its
 * input projections to the input of out_proj, for one session (device
 * arrays; the projections and out_proj are dial_b200_qlinear_forward calls):
 *   mixed [seq_len][2*k_heads*128 + v_heads*128] = in_proj_qkv(x) (q | k | v),
 *   z [seq_len][v_heads*128] = in_proj_z(x), b and a [seq_len][v_heads];
 *   conv_weight [channels][conv_kernel] (activation dtype); dt_bias, a_log
 *   [v_heads] and norm_weight [128] as f32;
 *   conv_state [channels][conv_kernel-1] (activation dtype) and
 *   recurrent_state [v_heads][128][128] (f32): the per-session linear-attention
 *   cache (llama3/cache.rs:267-290), read unless index_pos == 0 (a sequence
 *   start, cache.rs semantics) and replaced by the state after the call;
 *   core_out [seq_len][v_heads*128] receives the gated-normed output.
 * Asynchronous on `stream`.  Tokens of one call are scanned in order. */
int dial_b200_gdn_forward(const dial_b200_gdn_shape* sh, const void* mixed, const void* z,
                          const void* b, const void* a, const void* conv_weight,
                          const float* dt_bias, const float* a_log, const float* norm_weight,
                          void* conv_state, float* recurrent_state, int64_t seq_len,
                          int64_t index_pos, void* scratch, void* core_out, void* stream,
                          char* err, size_t err_size);

/* ------------------------------------------------------------------------ */
/* Decoder layers: Forwarder + per-session KV cache + Worker                */
/* ------------------------------------------------------------------------ */

typedef struct dial_b200_engine dial_b200_engine;

/* Shape contract of llama3::Config (dial-core/src/models/llama3/config.rs:68-85)
 * plus the engine's capacities. */
typedef struct {
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t vocab_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  float rms_norm_eps;
  float rope_theta;
  int32_t max_seq_len;  /* per-session KV capacity in tokens (--kv-cache-max-len) */
  int32_t max_sessions; /* concurrent sessions (one reference TCP connection each) */
  int32_t max_tokens;   /* rows per forward call (decode batch or prefill chunk) */
  int32_t act;          /* DIAL_ACT_BF16 or DIAL_ACT_F16 */
  int32_t linear_fmt;   /* DIAL_FMT_* of the layer linears */
  int32_t first_layer;  /* layer range owned by this engine (a topology node / stage) */
  int32_t num_layers;
  int32_t has_embed;    /* owns the token embedding (first stage) */
  int32_t has_head;     /* owns ln_f + lm_head + greedy argmax (last stage) */
} dial_b200_model_config;

/* Worker::new (spm/worker.rs:469-523): allocate weights, paged KV and work
 * buffers for the owned layers on `device`. */
int dial_b200_engine_create(const dial_b200_model_config* cfg, int device,
                            dial_b200_engine** out, char* err, size_t err_size);
void dial_b200_engine_destroy(dial_b200_engine* eng);

/* Seeded random-init weights generated on the device:
 * bf16 N(0, std) via `normal_table_bits` (65536 bf16 quantiles, host array),
 * norm weights 1.0, linears quantized to the engine's format at load. */
int dial_b200_engine_load_synthetic(dial_b200_engine* eng, uint64_t seed,
                                    const uint16_t* normal_table_bits, char* err, size_t err_size);

/* Explicit weights (host arrays).  which: 0 qkv (fused q|k|v rows),
 * 1 o_proj, 2 gate_up (fused gate|up rows), 3 down_proj, 4 lm_head. */
int dial_b200_engine_set_linear(dial_b200_engine* eng, int layer, int which, int fmt,
                                const void* codes, const void* scales, float global_scale,
                                int64_t out_dim, int64_t in_dim, char* err, size_t err_size);
/* which: 0 input_layernorm, 1 post_attention_layernorm, 2 q_norm, 3 k_norm,
 * 4 final norm (ln_f), 5 embedding [vocab, hidden]. */
int dial_b200_engine_set_tensor(dial_b200_engine* eng, int layer, int which, const void* host,
                                int64_t numel, char* err, size_t err_size);

/* Forwarder::forward (spm/mod.rs:236-242, text.rs:1636-1688): one session,
 * `seq_len` tokens starting at `index_pos`; hidden [seq_len, hidden] device
 * array updated in place.  index_pos == 0 starts the session over
 * (Cache::process_kv replace semantics, cache.rs:133-136). */
int dial_b200_layer_forward(dial_b200_engine* eng, int layer, void* hidden, int64_t seq_len,
                            int32_t session, int64_t index_pos, void* stream, char* err,
                            size_t err_size);

/* Forwarder::forward_local_batch (spm/mod.rs:268-277): a contiguous layer
 * range in one call; validates the whole range before touching the cache. */
int dial_b200_range_forward(dial_b200_engine* eng, int first_layer, int count, void* hidden,
                            int64_t seq_len, int32_t session, int64_t index_pos, void* stream,
                            char* err, size_t err_size);

/* Ragged multi-session decode: row m is one new token of session sids[m] at
 * positions[m] (host arrays); hidden [rows, hidden] device, in place. */
int dial_b200_batch_decode_forward(dial_b200_engine* eng, int first_layer, int count,
                                   void* hidden, int64_t rows, const int32_t* sids,
                                   const int32_t* positions, void* stream, char* err,
                                   size_t err_size);

/* Cache::clear / as_new for one session (cache.rs:240-265). */
int dial_b200_session_reset(dial_b200_engine* eng, int32_t session, char* err, size_t err_size);

/* Embedding::forward (qwen3_vl.rs:3302): tokens_dev [rows] -> hidden [rows, H]. */
int dial_b200_embed(dial_b200_engine* eng, const int32_t* tokens_dev, int64_t rows, void* hidden,
                    void* stream, char* err, size_t err_size);

/* ln_f + lm_head + greedy argmax (qwen3_vl.rs:2462-2487, 138-143) on `rows`
 * hidden rows; logits_dev [rows, vocab] may be NULL (an internal buffer is
 * used); tokens_dev [rows] receives the argmax ids. */
int dial_b200_head(dial_b200_engine* eng, const void* hidden, int64_t rows, void* logits_dev,
                   int32_t* tokens_dev, void* stream, char* err, size_t err_size);

/* One greedy decode step end to end, host buffers (synchronizes): tokens ->
 * embed -> owned layers -> head -> next tokens.  Engine must own the whole
 * model (has_embed && has_head && all layers).  Replays a CUDA graph per
 * distinct `rows`. */
int dial_b200_decode_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_host,
                          const int32_t* sids_host, const int32_t* positions_host,
                          int32_t* next_tokens_host, char* err, size_t err_size);

/* Greedy generation for one session (Master::generate, spm/master.rs:56-103):
 * prefill of `n_prompt` tokens then `n_gen` decode steps; out_tokens[n_gen]
 * (host).  ttft_s / decode_s receive wall times (may be NULL). */
int dial_b200_generate(dial_b200_engine* eng, int32_t session, const int32_t* prompt,
                       int64_t n_prompt, int64_t n_gen, int32_t* out_tokens, double* ttft_s,
                       double* decode_s, char* err, size_t err_size);

/* Device-resident decode loop for measurement: `n_steps` replays of the
 * step graph with the sampled tokens fed back on the device; rows of state
 * are seeded by dial_b200_decode_loop_prepare (synchronous: it waits for
 * loop replays still running on the engine stream).  dial_b200_decode_loop_run
 * is asynchronous on the engine stream. */
int dial_b200_decode_loop_prepare(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_host,
                                  const int32_t* sids_host, const int32_t* positions_host,
                                  char* err, size_t err_size);
int dial_b200_decode_loop_run(dial_b200_engine* eng, int64_t rows, int64_t n_steps, char* err,
                              size_t err_size);
/* Pipeline stage decode: one stage's share of a decode step with no host
 * synchronisation, for stages chained by NCCL send/recv (the in-box
 * replacement of the Master -> Worker hop, spm/client.rs:391-453 and
 * spm/worker.rs:740-796).  dial_b200_stage_prepare sets the rows' sessions
 * and positions on the device (synchronous, host arrays); every
 * dial_b200_stage_step then runs
 *   [has_embed: tokens_dev -> embedding ->] owned layers on hidden [rows, H]
 *   [-> has_head: ln_f + lm_head + argmax -> tokens_out_dev]
 * and advances the positions by one, as one CUDA graph (captured on first use
 * per (rows, buffer addresses)) launched on `stream`. */
int dial_b200_stage_prepare(dial_b200_engine* eng, int64_t rows, const int32_t* sids_host,
                            const int32_t* positions_host, char* err, size_t err_size);
int dial_b200_stage_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_dev,
                         void* hidden, int32_t* tokens_out_dev, void* stream, char* err,
                         size_t err_size);
/* dial_b200_stage_step for the prepared rows [row_offset, row_offset + rows):
 * the micro-batch form of the stage loop, where the sessions prepared by
 * dial_b200_stage_prepare are cut into micro-batches that are in flight on
 * different stages at once (the per-connection concurrency of the
 * reference's Worker, spm/worker.rs:316-325, 899-912).  One graph per
 * (offset, rows, buffer addresses); positions of those rows advance by one. */
int dial_b200_stage_step_rows(dial_b200_engine* eng, int64_t row_offset, int64_t rows,
                              const int32_t* tokens_dev, void* hidden, int32_t* tokens_out_dev,
                              void* stream, char* err, size_t err_size);

/* Stage link over peer memory: the in-box hop between pipeline stages on
 * different GPUs without NCCL (spm/client.rs:391-453 send, spm/worker.rs:
 * 740-796 receive).  Each stage owns an inbox in its own HBM;
 * dial_b200_stage_link_handle writes the 64-byte CUDA IPC handle of it, the
 * processes exchange the handles, and dial_b200_stage_link_open maps the next
 * stage's inbox (every stage but the last) and the first stage's (the last
 * stage).  Then dial_b200_stage_link_step is one decode step of this stage as
 * one CUDA graph on `stream`: [receive the hidden state (or, first stage, the
 * tokens) from this stage's inbox ->] embed / owned layers / head [-> write
 * the hidden state (or the sampled tokens) into the next (first) stage's
 * inbox], positions advanced; the receive waits on device (bounded:
 * DIAL_ERR_DEVICE after 2 s) and the first layer's weights stream meanwhile.
 * The first stage passes tokens_dev on the first step of a run (after
 * dial_b200_stage_prepare or a finish) and NULL after it;
 * dial_b200_stage_link_finish (first stage) receives the last step's tokens
 * into tokens_host (synchronizes), so every message sent is received.  The
 * stages must run on distinct GPUs (a receive waits for another GPU). */
int dial_b200_stage_link_handle(dial_b200_engine* eng, void* handle_out, char* err,
                                size_t err_size);
int dial_b200_stage_link_open(dial_b200_engine* eng, const void* next_handle,
                              const void* first_handle, char* err, size_t err_size);
int dial_b200_stage_link_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_dev,
                              void* stream, char* err, size_t err_size);
int dial_b200_stage_link_finish(dial_b200_engine* eng, int64_t rows, int32_t* tokens_host,
                                void* stream, char* err, size_t err_size);

/* Copy the loop's current tokens/positions back to host (synchronizes). */
int dial_b200_decode_loop_state(dial_b200_engine* eng, int64_t rows, int32_t* tokens_host,
                                int32_t* positions_host, char* err, size_t err_size);

/* The engine's CUDA stream (cudaStream_t) for event timing by the caller. */
void* dial_b200_engine_stream(dial_b200_engine* eng);

/* Fill a session's KV pages [0, length) with seeded N(0,1) bf16 values for
 * every owned layer (ragged multi-session benchmarks start from such a
 * cache); uses the normal table of load_synthetic scaled by `std`. */
int dial_b200_session_fill_random(dial_b200_engine* eng, int32_t session, int64_t length,
                                  uint64_t seed, const uint16_t* normal_table_bits, char* err,
                                  size_t err_size);

/* Number of kernels one device-loop decode step launches for `rows` rows,
 * counted as the kernel nodes of the captured step graph; -1 on error. */
int64_t dial_b200_step_kernel_count(dial_b200_engine* eng, int64_t rows);

/* Number of kernels dial_b200_generate launches for a prompt of `n_prompt`
 * tokens up to the first token (embed, the prefill layers, the head), counted
 * from a capture of that work that is never launched; -1 on error. */
int64_t dial_b200_prefill_kernel_count(dial_b200_engine* eng, int64_t n_prompt);

/* Measurement hook: launch one owned layer's linear (`which` as in
 * set_linear, with the epilogue the decode step uses) `iters` times back to
 * back on the engine stream over the engine's work buffers; layer < 0
 * rotates over every owned layer (no launch finds its weights in L2).
 * Asynchronous. */
int dial_b200_engine_linear_replay(dial_b200_engine* eng, int layer, int which, int64_t rows,
                                   int64_t iters, char* err, size_t err_size);

/* Algorithmic bytes one launch of that linear moves (weights + scales +
 * activations in + out), the roofline numerator. */
int64_t dial_b200_engine_linear_bytes(dial_b200_engine* eng, int layer, int which, int64_t rows);

#ifdef __cplusplus
}
#endif

#endif /* DIAL_B200_H */
