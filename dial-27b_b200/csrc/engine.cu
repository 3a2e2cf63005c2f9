// C++ host side of the B200 DIAL path: the linear op object (the
// CudaW8A16Linear / CudaQuantLinear equivalent), the layer engine (Forwarder
// + per-session paged KV cache + Worker), graph-captured decode steps, and
// the extern "C" entry points declared in include/dial_b200.h.
#include <cuda_fp16.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <tuple>
#include <memory>
#include <string>
#include <vector>

#include "../../include/dial_b200.h"
#include "attention.h"
#include "gemm.h"
#include "gemv.h"
#include "layout.h"
#include "link.h"
#include "trace.h"
#include "misc.h"

using namespace dialb200;

namespace {

// ------------------------------------------------------------------ errors
struct Error {
  int code;
  std::string msg;
};

int report(char* err, size_t n, int code, const std::string& msg) {
  if (err && n) {
    std::snprintf(err, n, "%s", msg.c_str());
  }
  return code;
}

std::string fmtstr(const char* f, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, f);
  std::vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

#define DIAL_CUDA(call)                                                                   \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      throw Error{DIAL_ERR_CUDA, fmtstr("%s failed: %s", #call, cudaGetErrorString(e_))}; \
  } while (0)

#define DIAL_CHECK(cond, ...)                                \
  do {                                                       \
    if (!(cond)) throw Error{DIAL_ERR_INVALID, fmtstr(__VA_ARGS__)}; \
  } while (0)

template <typename F>
int guarded(char* err, size_t n, F&& f) {
  try {
    f();
    return DIAL_OK;
  } catch (const Error& e) {
    return report(err, n, e.code, e.msg);
  } catch (const std::exception& e) {
    return report(err, n, DIAL_ERR_INVALID, e.what());
  }
}

// Device status word, one per device, allocated on first use (`create`); the
// reader passes create = false and sees nullptr on a device that has none.
int* device_status_word(bool create = true) {
  static int* words[64] = {nullptr};
  int dev = 0;
  DIAL_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw Error{DIAL_ERR_INVALID, "device index out of range"};
  if (!words[dev] && create) {
    DIAL_CUDA(cudaMalloc(&words[dev], sizeof(int)));
    DIAL_CUDA(cudaMemset(words[dev], 0, sizeof(int)));
  }
  return words[dev];
}

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  explicit DevBuf(size_t b) { alloc(b); }
  void alloc(size_t b) {
    release();
    if (b) DIAL_CUDA(cudaMalloc(&p, b));
    bytes = b;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  ~DevBuf() { release(); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) { release(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
    return *this;
  }
  template <typename T> T* as() const { return static_cast<T*>(p); }
};

size_t act_size(int dtype) { return dtype == DIAL_ACT_F32 ? 4 : 2; }

// ------------------------------------------------------------ linear object
struct Linear {
  DevQLinear d{};
  DevBuf tiles, row_scale, blk_scale;
  int act = DIAL_ACT_BF16;
  int64_t in_dim = 0, out_dim = 0;
  int64_t resident = 0;
  bool ready() const { return tiles.p != nullptr; }
};

void geometry(Linear& L, int fmt, int64_t N, int64_t K, int swiglu) {
  DIAL_CHECK(N > 0 && K > 0, "linear shape must be positive, got [%lld,%lld]", (long long)N,
             (long long)K);
  DIAL_CHECK(N < (1ll << 30) && K < (1ll << 30), "linear shape too large");
  if (swiglu) DIAL_CHECK(N % 2 == 0, "fused gate/up needs an even row count, got %lld", (long long)N);
  const int kch = fmt_kch(fmt);
  L.d = DevQLinear{};
  L.d.fmt = fmt;
  L.d.N = static_cast<int>(N);
  L.d.K = static_cast<int>(K);
  L.d.K_pad = static_cast<int>((K + kch - 1) / kch * kch);
  L.d.C = L.d.K_pad / kch;
  L.d.T = swiglu ? static_cast<int>((N / 2 + 7) / 8) : static_cast<int>((N + 15) / 16);
  L.d.swiglu = swiglu;
  L.d.global_scale = 1.f;
  L.in_dim = K;
  L.out_dim = N;
}

void alloc_tiles(Linear& L) {
  const size_t bytes = static_cast<size_t>(L.d.T) * L.d.C * fmt_chunk_bytes(L.d.fmt);
  L.tiles.alloc(bytes);
  L.d.tiles = L.tiles.as<uint8_t>();
}

void set_row_scales_from_device(Linear& L, const float* scale_dev, cudaStream_t s) {
  L.row_scale.alloc(static_cast<size_t>(L.d.T) * 16 * sizeof(float));
  DIAL_CUDA(tile_row_scales(scale_dev, L.d, L.row_scale.as<float>(), s));
  L.d.row_scale = L.row_scale.as<float>();
}

// Build a linear from host arrays in one of the DIAL_FMT_* layouts.
void build_linear_host(Linear& L, int fmt, int act, const void* codes, const void* scales,
                       float global_scale, int64_t N, int64_t K, int swiglu, cudaStream_t s) {
  DIAL_CHECK(codes != nullptr, "weight codes pointer is null");
  DIAL_CHECK(act == DIAL_ACT_BF16 || act == DIAL_ACT_F16, "activation dtype must be BF16 or F16");
  geometry(L, fmt, N, K, swiglu);
  L.act = act;
  int64_t code_bytes = 0, row_ld = 0;
  switch (fmt) {
    case DIAL_FMT_W8A16_ROW:
    case DIAL_FMT_FP8_ROW:
    case DIAL_FMT_FP8_BLOCK128:
      code_bytes = N * K;
      row_ld = K;
      break;
    case DIAL_FMT_NVFP4_G16:
      DIAL_CHECK(K % 16 == 0, "NVFP4 QuantLinear input dimension %lld is not divisible by 16",
                 (long long)K);
      code_bytes = N * K / 2;
      row_ld = K / 2;
      break;
    case DIAL_FMT_DENSE:
      code_bytes = N * K * 2;
      row_ld = K * 2;
      break;
    default:
      DIAL_CHECK(false, "unknown weight format %d", fmt);
  }
  alloc_tiles(L);
  DevBuf tmp(static_cast<size_t>(code_bytes));
  DIAL_CUDA(cudaMemcpyAsync(tmp.p, codes, code_bytes, cudaMemcpyHostToDevice, s));
  DIAL_CUDA(tile_codes(tmp.as<uint8_t>(), row_ld, L.d, L.tiles.as<uint8_t>(), s));
  L.resident = static_cast<int64_t>(L.tiles.bytes);
  if (fmt == DIAL_FMT_W8A16_ROW || fmt == DIAL_FMT_FP8_ROW) {
    DIAL_CHECK(scales != nullptr, "scale pointer is null");
    // One f32 scale per output row; a per-tensor FP8 scale is expanded to
    // every row by the caller, as try_cuda_fp8 does (quant.rs:416-427).
    std::vector<float> sc(static_cast<size_t>(N));
    std::memcpy(sc.data(), scales, sc.size() * sizeof(float));
    DevBuf sdev(sc.size() * sizeof(float));
    DIAL_CUDA(cudaMemcpyAsync(sdev.p, sc.data(), sdev.bytes, cudaMemcpyHostToDevice, s));
    set_row_scales_from_device(L, sdev.as<float>(), s);
    L.resident += N * 4;
    DIAL_CUDA(cudaStreamSynchronize(s));
  } else if (fmt == DIAL_FMT_FP8_BLOCK128) {
    DIAL_CHECK(scales != nullptr, "scale pointer is null");
    const int64_t nbr = (N + 127) / 128, nbc = (K + 127) / 128;
    const int ld = static_cast<int>((nbc + 3) / 4 * 4);
    std::vector<float> sc(static_cast<size_t>(nbr * ld), 0.f);
    const float* hs = static_cast<const float*>(scales);
    for (int64_t r = 0; r < nbr; ++r)
      for (int64_t c = 0; c < nbc; ++c) sc[r * ld + c] = hs[r * nbc + c];
    L.blk_scale.alloc(sc.size() * sizeof(float));
    DIAL_CUDA(cudaMemcpyAsync(L.blk_scale.p, sc.data(), L.blk_scale.bytes, cudaMemcpyHostToDevice,
                              s));
    L.d.blk_scale = L.blk_scale.as<float>();
    L.d.blk_ld = ld;
    L.resident += nbr * nbc * 4;
    DIAL_CUDA(cudaStreamSynchronize(s));
  } else if (fmt == DIAL_FMT_NVFP4_G16) {
    DIAL_CHECK(scales != nullptr, "scale pointer is null");
    DevBuf sdev(static_cast<size_t>(N * K / 16));
    DIAL_CUDA(cudaMemcpyAsync(sdev.p, scales, sdev.bytes, cudaMemcpyHostToDevice, s));
    DIAL_CUDA(tile_nvfp4_scales(sdev.as<uint8_t>(), K / 16, L.d, L.tiles.as<uint8_t>(), s));
    L.d.global_scale = global_scale;
    L.resident = N * K / 2 + N * K / 16 + 4;
    DIAL_CUDA(cudaStreamSynchronize(s));
  } else {
    DIAL_CUDA(cudaStreamSynchronize(s));
  }
}

// W8A16 from a dense device weight [N, K] of dtype src_dtype.
void build_w8a16_from_device_dense(Linear& L, const void* w_dev, int src_dtype, int act, int64_t N,
                                   int64_t K, int swiglu, cudaStream_t s) {
  geometry(L, DIAL_FMT_W8A16_ROW, N, K, swiglu);
  L.act = act;
  alloc_tiles(L);
  DevBuf q(static_cast<size_t>(N * K)), sc(static_cast<size_t>(N) * 4);
  DIAL_CUDA(quantize_rows(w_dev, src_dtype, static_cast<int>(N), static_cast<int>(K),
                          q.as<int8_t>(), sc.as<float>(), s));
  DIAL_CUDA(tile_codes(q.as<uint8_t>(), K, L.d, L.tiles.as<uint8_t>(), s));
  set_row_scales_from_device(L, sc.as<float>(), s);
  L.resident = N * K + N * 4;
  DIAL_CUDA(cudaStreamSynchronize(s));
}

// FP8 block-128 or NVFP4 from a dense bf16 device weight [N, K] (synthetic
// models of the 27B-class configuration), quantized on the device.
void build_quant_from_device_bf16(Linear& L, int fmt, const uint16_t* w_dev, int act, int64_t N,
                                  int64_t K, int swiglu, cudaStream_t s) {
  geometry(L, fmt, N, K, swiglu);
  L.act = act;
  alloc_tiles(L);
  if (fmt == DIAL_FMT_FP8_BLOCK128) {
    const int64_t nbr = (N + 127) / 128, nbc = (K + 127) / 128;
    const int ld = static_cast<int>((nbc + 3) / 4 * 4);
    DevBuf codes(static_cast<size_t>(N * K));
    L.blk_scale.alloc(static_cast<size_t>(nbr * ld) * sizeof(float));
    DIAL_CUDA(cudaMemsetAsync(L.blk_scale.p, 0, L.blk_scale.bytes, s));
    DIAL_CUDA(quantize_fp8_block128_dev(w_dev, static_cast<int>(N), static_cast<int>(K),
                                        codes.as<uint8_t>(), L.blk_scale.as<float>(), ld, s));
    DIAL_CUDA(tile_codes(codes.as<uint8_t>(), K, L.d, L.tiles.as<uint8_t>(), s));
    L.d.blk_scale = L.blk_scale.as<float>();
    L.d.blk_ld = ld;
    L.resident = N * K + nbr * nbc * 4;
  } else if (fmt == DIAL_FMT_NVFP4_G16) {
    DIAL_CHECK(K % 16 == 0, "NVFP4 needs in_dim %% 16 == 0 (got %lld)", (long long)K);
    DevBuf packed(static_cast<size_t>(N * K / 2)), sc(static_cast<size_t>(N * K / 16)), amax(16);
    DIAL_CUDA(quantize_nvfp4_dev(w_dev, N * K, packed.as<uint8_t>(), sc.as<uint8_t>(),
                                 amax.as<unsigned>(), s));
    DIAL_CUDA(tile_codes(packed.as<uint8_t>(), K / 2, L.d, L.tiles.as<uint8_t>(), s));
    DIAL_CUDA(tile_nvfp4_scales(sc.as<uint8_t>(), K / 16, L.d, L.tiles.as<uint8_t>(), s));
    unsigned bits = 0;
    DIAL_CUDA(cudaMemcpyAsync(&bits, amax.p, 4, cudaMemcpyDeviceToHost, s));
    DIAL_CUDA(cudaStreamSynchronize(s));
    float am = 0.f;
    std::memcpy(&am, &bits, 4);
    L.d.global_scale = am > 0.f ? static_cast<float>(static_cast<double>(am) / 6.0 / 448.0) : 1.f;
    L.resident = N * K / 2 + N * K / 16 + 4;
  } else {
    DIAL_CHECK(false, "device quantizer for format %d not available", fmt);
  }
  DIAL_CUDA(cudaStreamSynchronize(s));
}

void build_dense_from_device(Linear& L, const void* w_dev, int act, int64_t N, int64_t K,
                             cudaStream_t s) {
  geometry(L, DIAL_FMT_DENSE, N, K, 0);
  L.act = act;
  alloc_tiles(L);
  DIAL_CUDA(tile_codes(static_cast<const uint8_t*>(w_dev), K * 2, L.d, L.tiles.as<uint8_t>(), s));
  L.resident = N * K * 2;
  DIAL_CUDA(cudaStreamSynchronize(s));
}

GemvTuning g_tuning() {
  GemvTuning t;
  if (const char* v = std::getenv("DIAL_B200_GEMV_SLOTS")) t.slots = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_GEMV_GRID")) t.grid = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_GEMV_NVFP4_STAGE")) t.nvfp4_stage = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_PDL")) t.pdl = std::atoi(v) != 0;
  if (const char* v = std::getenv("DIAL_B200_GEMM_MIN_ROWS")) t.gemm_min_rows = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_ATTN_MIN_SPLIT")) t.attn_min_split = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_ATTN_TC")) t.attn_tc = std::atoi(v) != 0;
  if (const char* v = std::getenv("DIAL_B200_ATTN_RING")) t.attn_ring = std::atoi(v) != 0;
  if (const char* v = std::getenv("DIAL_B200_ATTN_TOKSPLIT")) t.attn_tok_split = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_ATTN_MMA")) t.attn_mma = std::atoi(v) != 0;
  if (const char* v = std::getenv("DIAL_B200_ATTN_MMA_MIN_SPLIT")) t.attn_mma_min_split = std::atoi(v);
  if (const char* v = std::getenv("DIAL_B200_ATTN_MMA_RING")) t.attn_mma_ring = std::atoi(v);
  return t;
}

// Buffers of the tcgen05 GEMM: activation staging (gemm_scratch_bytes(M,
// K_pad) bytes) and an optional split-K workspace.
constexpr size_t kGemmPartBytes = 24u << 20;  // split-K workspace per engine

struct GemmScratch {
  void* stage = nullptr;
  float* part = nullptr;
  size_t part_bytes = 0;
};

// Calls of M >= gemm_min_rows rows on a supported weight take the tcgen05
// GEMM when staging scratch is given; everything else the decode GEMV.
bool use_gemm(const Linear& L, int M, bool have_scratch) {
  const int min_rows = g_tuning().gemm_min_rows;
  return have_scratch && min_rows > 0 && M >= min_rows && gemm_w8a16_supported(L.d);
}

void run_gemm(const Linear& L, const void* x, int x_ld, const void* norm_w, float eps, void* out,
              int out_ld, int M, int epi, cudaStream_t s, int* status, const GemmScratch& sc) {
  void* scratch = sc.stage;
  GemmArgs g{};
  g.w = L.d;
  g.x = x;
  g.x_ld = x_ld;
  g.norm_w = norm_w;
  g.eps = eps;
  g.out = out;
  g.out_ld = out_ld;
  g.M = M;
  g.xh = static_cast<__half*>(scratch);
  const size_t xh_bytes = (static_cast<size_t>(M) * L.d.K_pad * 2 + 255) / 256 * 256;
  g.xexp = reinterpret_cast<int*>(static_cast<char*>(scratch) + xh_bytes);
  g.status = status;
  g.part = sc.part;
  g.part_bytes = sc.part_bytes;
  DIAL_CUDA(gemm_w8a16_launch(g, L.act, epi, s));
}

void run_linear(const Linear& L, const void* x, int x_ld, const void* norm_w, float eps, void* out,
                int out_ld, int M, int epi, cudaStream_t s, int* status,
                const GemmScratch* scratch = nullptr, unsigned long long* trace = nullptr,
                int trace_tag = 0) {
  if (use_gemm(L, M, scratch != nullptr && scratch->stage != nullptr)) {
    run_gemm(L, x, x_ld, norm_w, eps, out, out_ld, M, epi, s, status, *scratch);
    return;
  }
  GemvArgs a{};
  a.w = L.d;
  a.x = x;
  a.x_ld = x_ld;
  a.norm_w = norm_w;
  a.eps = eps;
  a.out = out;
  a.out_ld = out_ld;
  a.M = M;
  a.status = status;
  a.trace = trace;
  a.trace_tag = trace_tag;
  DIAL_CUDA(gemv_launch(a, L.act, epi, norm_w != nullptr, s, g_tuning()));
}

}  // namespace

struct dial_b200_qlinear {
  Linear L;
  int device = 0;
  DevBuf scratch;  // tcgen05 GEMM staging, grown on the first call with that many rows
};

// =================================================================== engine
namespace {

struct LayerW {
  Linear qkv, o, gate_up, down;
  DevBuf input_norm, post_norm, q_norm, k_norm;
  DevBuf kpool, vpool;
};

struct Graph {
  cudaGraph_t g = nullptr;
  cudaGraphExec_t exec = nullptr;
  ~Graph() {
    if (exec) cudaGraphExecDestroy(exec);
    if (g) cudaGraphDestroy(g);
  }
};

}  // namespace

struct dial_b200_engine {
  dial_b200_model_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  int H = 0, I = 0, V = 0, QH = 0, KVH = 0, D = 0, QKV = 0;
  int max_blocks = 0, max_rows_decode = 0;
  std::vector<LayerW> layers;  // owned layers, index l - first_layer
  DevBuf embed, final_norm;
  Linear lm_head;
  DevBuf cos, sin, block_table;
  DevBuf hidden, qkv, attn, inter;
  DevBuf tok_in, sid, pos, tok_out, rows_scratch;
  DevBuf part_o, part_ml, counters;
  DevBuf amax_key, amax_count;  // head argmax keys / arrival counters, zero between steps
  DevBuf gemm_scratch;          // prefill GEMM activation staging (max_tokens rows)
  DevBuf gemm_part;             // split-K partial sums of small-row GEMM calls
  GemmScratch scratch() { return GemmScratch{gemm_scratch.p, gemm_part.as<float>(), gemm_part.bytes}; }
  DevBuf trace;                 // DIAL_B200_TRACE=<csv>: per-CTA timeline of decode steps
  std::string trace_path;
  // stage link over peer memory (link.h): this stage's inbox (IPC-exported),
  // counters [hidden received, tokens received, hidden sent, tokens sent], the
  // opened inboxes of the next stage and (last stage) of the first stage
  DevBuf link_in, link_cnt;
  uint8_t* link_next = nullptr;
  uint8_t* link_first = nullptr;
  std::map<std::tuple<int64_t, const void*>, std::unique_ptr<Graph>> link_graphs;
  int32_t* h_in = nullptr;   // pinned: [3][max_rows] tokens, sids, positions
  int32_t* h_out = nullptr;  // pinned: [max_rows] tokens + status
  int* status = nullptr;
  std::map<int64_t, std::unique_ptr<Graph>> step_graphs, loop_graphs;
  // pipeline-stage decode graphs keyed by (rows, tokens in, hidden, tokens out)
  std::map<std::tuple<int64_t, const void*, const void*, const void*>, std::unique_ptr<Graph>>
      stage_graphs;

  size_t esz() const { return 2; }
  LayerW& layer(int l) {
    DIAL_CHECK(l >= cfg.first_layer && l < cfg.first_layer + cfg.num_layers,
               "layer %d is not owned by this engine (owns %d..%d)", l, cfg.first_layer,
               cfg.first_layer + cfg.num_layers - 1);
    return layers[l - cfg.first_layer];
  }
  // KV splits available to a decode batch of M rows: up to 32 per (row, kv
  // head), fewer for large batches (4096 / (kv_heads * M), at least 1); the
  // kernel uses as many as the row's context fills with 16-token spans.
  int splits_for(int M) const {
    const int s = 4096 / std::max(1, KVH * M);
    return std::max(1, std::min(32, s));
  }
  AttnShape shape() const {
    AttnShape sh{};
    sh.q_heads = QH;
    sh.kv_heads = KVH;
    sh.head_dim = D;
    sh.max_blocks = max_blocks;
    sh.max_pos = cfg.max_seq_len;
    sh.eps = cfg.rms_norm_eps;
    return sh;
  }
};

namespace {

void engine_init(dial_b200_engine* e, const dial_b200_model_config& c, int device) {
  e->cfg = c;
  e->device = device;
  DIAL_CUDA(cudaSetDevice(device));
  DIAL_CHECK(c.hidden_size > 0 && c.num_attention_heads > 0 && c.num_key_value_heads > 0,
             "invalid model config");
  DIAL_CHECK(c.hidden_size % c.num_attention_heads == 0, "hidden_size %% heads != 0");
  DIAL_CHECK(c.num_attention_heads % c.num_key_value_heads == 0, "heads %% kv_heads != 0");
  DIAL_CHECK(c.act == DIAL_ACT_BF16 || c.act == DIAL_ACT_F16, "act must be BF16 or F16");
  DIAL_CHECK(c.linear_fmt == DIAL_FMT_W8A16_ROW || c.linear_fmt == DIAL_FMT_FP8_BLOCK128 ||
                 c.linear_fmt == DIAL_FMT_FP8_ROW || c.linear_fmt == DIAL_FMT_NVFP4_G16 ||
                 c.linear_fmt == DIAL_FMT_DENSE,
             "unknown linear format %d", c.linear_fmt);
  DIAL_CHECK(c.first_layer >= 0 && c.num_layers >= 0 &&
                 c.first_layer + c.num_layers <= c.num_hidden_layers,
             "layer range [%d, %d) outside the model's %d layers", c.first_layer,
             c.first_layer + c.num_layers, c.num_hidden_layers);
  DIAL_CHECK(c.max_seq_len > 0 && c.max_sessions > 0 && c.max_tokens > 0, "capacities must be > 0");
  e->H = c.hidden_size;
  e->I = c.intermediate_size;
  e->V = c.vocab_size;
  e->QH = c.num_attention_heads;
  e->KVH = c.num_key_value_heads;
  e->D = c.hidden_size / c.num_attention_heads;
  DIAL_CHECK(e->D == 128, "head_dim must be 128 (got %d)", e->D);
  DIAL_CHECK(e->H % 8 == 0 && e->I % 8 == 0, "hidden/intermediate must be multiples of 8");
  e->QKV = (e->QH + 2 * e->KVH) * e->D;
  e->max_blocks = (c.max_seq_len + kPageTokens - 1) / kPageTokens;
  e->max_rows_decode = std::min(c.max_tokens, 1024);
  DIAL_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  e->status = device_status_word();

  const size_t es = e->esz();
  const size_t T = static_cast<size_t>(c.max_tokens);
  e->layers.resize(c.num_layers);
  const size_t pool_elems = static_cast<size_t>(c.max_sessions) * e->max_blocks * e->KVH *
                            kPageTokens * e->D;
  for (auto& L : e->layers) {
    L.input_norm.alloc(e->H * es);
    L.post_norm.alloc(e->H * es);
    L.q_norm.alloc(e->D * es);
    L.k_norm.alloc(e->D * es);
    L.kpool.alloc(pool_elems * es);
    L.vpool.alloc(pool_elems * es);
    DIAL_CUDA(cudaMemsetAsync(L.kpool.p, 0, L.kpool.bytes, e->stream));
    DIAL_CUDA(cudaMemsetAsync(L.vpool.p, 0, L.vpool.bytes, e->stream));
  }
  if (c.has_embed) e->embed.alloc(static_cast<size_t>(e->V) * e->H * es);
  if (c.has_head) e->final_norm.alloc(e->H * es);

  // RoPE tables (cache.rs:37-67): inv_freq in f32, angle = pos * inv_freq in
  // f32, cos/sin of that angle, rounded to the activation dtype.
  {
    const int half = e->D / 2;
    std::vector<uint16_t> ct(static_cast<size_t>(c.max_seq_len) * half),
        st(static_cast<size_t>(c.max_seq_len) * half);
    auto to_act = [&](float v) -> uint16_t {
      if (c.act == DIAL_ACT_F16) {
        __half h = __float2half_rn(v);
        return *reinterpret_cast<uint16_t*>(&h);
      }
      uint32_t b;
      std::memcpy(&b, &v, 4);
      const uint32_t bias = ((b >> 16) & 1u) + 0x7fffu;
      return static_cast<uint16_t>((b + bias) >> 16);
    };
    for (int i = 0; i < half; ++i) {
      const float expo = static_cast<float>(2 * i) / static_cast<float>(e->D);
      const float inv = 1.0f / std::pow(c.rope_theta, expo);
      for (int p = 0; p < c.max_seq_len; ++p) {
        const float ang = static_cast<float>(p) * inv;
        ct[static_cast<size_t>(p) * half + i] = to_act(static_cast<float>(std::cos(static_cast<double>(ang))));
        st[static_cast<size_t>(p) * half + i] = to_act(static_cast<float>(std::sin(static_cast<double>(ang))));
      }
    }
    e->cos.alloc(ct.size() * 2);
    e->sin.alloc(st.size() * 2);
    DIAL_CUDA(cudaMemcpy(e->cos.p, ct.data(), e->cos.bytes, cudaMemcpyHostToDevice));
    DIAL_CUDA(cudaMemcpy(e->sin.p, st.data(), e->sin.bytes, cudaMemcpyHostToDevice));
  }
  // Static paged layout: session s owns blocks [s*MB, (s+1)*MB).
  {
    std::vector<int32_t> bt(static_cast<size_t>(c.max_sessions) * e->max_blocks);
    for (size_t i = 0; i < bt.size(); ++i) bt[i] = static_cast<int32_t>(i);
    e->block_table.alloc(bt.size() * 4);
    DIAL_CUDA(cudaMemcpy(e->block_table.p, bt.data(), e->block_table.bytes, cudaMemcpyHostToDevice));
  }
  e->hidden.alloc(T * e->H * es);
  e->qkv.alloc(T * e->QKV * es);
  e->attn.alloc(T * e->QH * e->D * es);
  e->inter.alloc(T * e->I * es);
  e->tok_in.alloc(T * 4);
  e->sid.alloc(T * 4);
  e->pos.alloc(T * 4);
  e->tok_out.alloc(T * 4);
  e->rows_scratch.alloc(2 * T * 4);
  {
    const int kmax = std::max({e->H, e->I, e->QH * e->D});
    const int kpad = (kmax + 63) / 64 * 64;
    e->gemm_scratch.alloc(gemm_scratch_bytes(static_cast<int>(T), kpad));
    if (T >= 16) e->gemm_part.alloc(kGemmPartBytes);
  }
  if (c.has_head) {
    e->amax_key.alloc(static_cast<size_t>(T) * 8);
    e->amax_count.alloc(static_cast<size_t>(T) * 4);
    DIAL_CUDA(cudaMemset(e->amax_key.p, 0, e->amax_key.bytes));
    DIAL_CUDA(cudaMemset(e->amax_count.p, 0, e->amax_count.bytes));
  }
  // split-KV scratch: largest M * splits over decode batch sizes
  size_t max_rows_splits = 0;
  for (int M = 1; M <= e->max_rows_decode; ++M) {
    const int S = e->splits_for(M);
    if (S > 1) max_rows_splits = std::max(max_rows_splits, static_cast<size_t>(M) * S);
  }
  if (max_rows_splits) {
    e->part_o.alloc(max_rows_splits * e->QH * e->D * 4);
    e->part_ml.alloc(max_rows_splits * e->QH * 2 * 4);
    e->counters.alloc(static_cast<size_t>(e->max_rows_decode) * e->KVH * 4);
    DIAL_CUDA(cudaMemset(e->counters.p, 0, e->counters.bytes));
  }
  if (const char* tp = std::getenv("DIAL_B200_TRACE")) {
    constexpr unsigned long long kRecords = 1ull << 18;
    e->trace_path = tp;
    e->trace.alloc((kTraceHeader + kRecords * kTraceWords) * 8);
    const unsigned long long hdr[2] = {0ull, kRecords};
    DIAL_CUDA(cudaMemset(e->trace.p, 0, e->trace.bytes));
    DIAL_CUDA(cudaMemcpy(e->trace.p, hdr, sizeof(hdr), cudaMemcpyHostToDevice));
  }
  DIAL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&e->h_in), 3 * T * 4, cudaHostAllocDefault));
  DIAL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&e->h_out), (T + 1) * 4, cudaHostAllocDefault));
  DIAL_CUDA(cudaStreamSynchronize(e->stream));
}

void fill_ones(DevBuf& b, int64_t n, cudaStream_t s, int act) {
  const uint16_t one = act == DIAL_ACT_F16 ? 0x3C00 : 0x3F80;
  DIAL_CUDA(fill_u16(b.as<uint16_t>(), n, one, s));
}

// Synthetic streams: layer l parts use stream ((l+1) << 8) + part.
enum SynthPart { kPq = 0, kPk = 1, kPv = 2, kPo = 3, kPgate = 4, kPup = 5, kPdown = 6 };
constexpr uint64_t kStreamEmbed = 0xE0000, kStreamLmHead = 0xE0002;
uint64_t layer_stream(int l, int part) { return (static_cast<uint64_t>(l + 1) << 8) + part; }

void engine_load_synthetic(dial_b200_engine* e, uint64_t seed, const uint16_t* table_host) {
  DIAL_CHECK(table_host != nullptr, "normal table is null");
  const int fmt = e->cfg.linear_fmt;
  DIAL_CHECK(fmt == DIAL_FMT_W8A16_ROW || fmt == DIAL_FMT_FP8_BLOCK128 || fmt == DIAL_FMT_NVFP4_G16,
             "synthetic load supports W8A16, FP8 block-128 and NVFP4 (engine uses %d)", fmt);
  // dense bf16 weight -> this engine's linear format
  auto build = [&](Linear& L, const uint16_t* w, int64_t N, int64_t K, int swiglu) {
    if (fmt == DIAL_FMT_W8A16_ROW)
      build_w8a16_from_device_dense(L, w, kSrcBf16, e->cfg.act, N, K, swiglu, e->stream);
    else
      build_quant_from_device_bf16(L, fmt, w, e->cfg.act, N, K, swiglu, e->stream);
  };
  cudaStream_t s = e->stream;
  DevBuf table(65536 * 2);
  DIAL_CUDA(cudaMemcpy(table.p, table_host, table.bytes, cudaMemcpyHostToDevice));
  const uint16_t* tb = table.as<uint16_t>();
  const int H = e->H, I = e->I, QH = e->QH, KVH = e->KVH, D = e->D;
  const int act = e->cfg.act;
  DIAL_CHECK(act == DIAL_ACT_BF16, "synthetic weights are bf16; engine act must be BF16");
  size_t max_elems = std::max<size_t>({static_cast<size_t>(e->QKV) * H, static_cast<size_t>(2) * I * H,
                                       static_cast<size_t>(H) * I});
  DevBuf tmp(max_elems * 2);
  uint16_t* t = tmp.as<uint16_t>();
  for (int li = 0; li < e->cfg.num_layers; ++li) {
    const int l = e->cfg.first_layer + li;
    LayerW& L = e->layers[li];
    const int64_t nq = static_cast<int64_t>(QH) * D * H, nk = static_cast<int64_t>(KVH) * D * H;
    DIAL_CUDA(synth_table_fill(t, nq, seed, layer_stream(l, kPq), 0, tb, s));
    DIAL_CUDA(synth_table_fill(t + nq, nk, seed, layer_stream(l, kPk), 0, tb, s));
    DIAL_CUDA(synth_table_fill(t + nq + nk, nk, seed, layer_stream(l, kPv), 0, tb, s));
    build(L.qkv, t, e->QKV, H, 0);
    DIAL_CUDA(synth_table_fill(t, static_cast<int64_t>(H) * QH * D, seed, layer_stream(l, kPo), 0, tb, s));
    build(L.o, t, H, QH * D, 0);
    const int64_t ng = static_cast<int64_t>(I) * H;
    DIAL_CUDA(synth_table_fill(t, ng, seed, layer_stream(l, kPgate), 0, tb, s));
    DIAL_CUDA(synth_table_fill(t + ng, ng, seed, layer_stream(l, kPup), 0, tb, s));
    build(L.gate_up, t, 2 * I, H, 1);
    DIAL_CUDA(synth_table_fill(t, static_cast<int64_t>(H) * I, seed, layer_stream(l, kPdown), 0, tb, s));
    build(L.down, t, H, I, 0);
    fill_ones(L.input_norm, H, s, act);
    fill_ones(L.post_norm, H, s, act);
    fill_ones(L.q_norm, D, s, act);
    fill_ones(L.k_norm, D, s, act);
  }
  tmp.release();
  if (e->cfg.has_embed)
    DIAL_CUDA(synth_table_fill(e->embed.as<uint16_t>(), static_cast<int64_t>(e->V) * H, seed,
                               kStreamEmbed, 0, tb, s));
  if (e->cfg.has_head) {
    fill_ones(e->final_norm, H, s, act);
    DevBuf w(static_cast<size_t>(e->V) * H * 2);
    DIAL_CUDA(synth_table_fill(w.as<uint16_t>(), static_cast<int64_t>(e->V) * H, seed,
                               kStreamLmHead, 0, tb, s));
    build_dense_from_device(e->lm_head, w.p, act, e->V, H, s);
  }
  DIAL_CUDA(cudaStreamSynchronize(s));
}

// ----------------------------------------------------------- forward pieces
void set_rows_decode(dial_b200_engine* e, int M, const int32_t* sids, const int32_t* pos,
                     cudaStream_t s) {
  // small per-call arrays travel by pageable copy ordered on the stream
  std::vector<int32_t> buf(2 * static_cast<size_t>(M));
  for (int i = 0; i < M; ++i) {
    DIAL_CHECK(sids[i] >= 0 && sids[i] < e->cfg.max_sessions, "session %d out of range [0,%d)",
               sids[i], e->cfg.max_sessions);
    DIAL_CHECK(pos[i] >= 0 && pos[i] < e->cfg.max_seq_len,
               "position %d outside the KV capacity %d", pos[i], e->cfg.max_seq_len);
    buf[i] = sids[i];
    buf[M + i] = pos[i];
  }
  DIAL_CUDA(cudaMemcpyAsync(e->sid.p, buf.data(), M * 4, cudaMemcpyHostToDevice, s));
  DIAL_CUDA(cudaMemcpyAsync(e->pos.p, buf.data() + M, M * 4, cudaMemcpyHostToDevice, s));
  DIAL_CUDA(cudaStreamSynchronize(s));
}

AttnDecodeArgs decode_attn_args(dial_b200_engine* e, LayerW& L, int M, int row0 = 0) {
  AttnDecodeArgs a{};
  a.sh = e->shape();
  a.qkv = e->qkv.p;
  a.qkv_ld = e->QKV;
  a.q_norm_w = L.q_norm.p;
  a.k_norm_w = L.k_norm.p;
  a.cos = e->cos.p;
  a.sin = e->sin.p;
  a.kv = KvLayer{L.kpool.p, L.vpool.p};
  a.block_table = e->block_table.as<int32_t>();
  a.sid = e->sid.as<int32_t>() + row0;
  a.pos = e->pos.as<int32_t>() + row0;
  a.out = e->attn.p;
  a.out_ld = e->QH * e->D;
  a.M = M;
  a.splits = e->part_o.p ? e->splits_for(M) : 1;
  a.part_o = e->part_o.as<float>();
  a.part_ml = e->part_ml.as<float>();
  a.counters = e->counters.as<int>();
  a.status = e->status;
  a.min_split_tokens = g_tuning().attn_min_split;
  // every caller of layer_decode starts from completed sessions, positions
  // and KV: a graph launch (root node), or an eager call after a host sync
  a.rows_ready = 1;
  // opt-in page ring for steps of few rows (measured: +2 % on the 8B decoder
  // at 2048-token context, -11 % on the 27B shapes; with many rows the
  // register form packs more CTAs per SM)
  a.page_ring = g_tuning().attn_ring && M <= 4 ? 1 : 0;
  a.tok_split = g_tuning().attn_tok_split;
  a.num_blocks = g_tuning().attn_mma ? e->cfg.max_sessions * e->max_blocks : 0;
  if (a.num_blocks && M > 4 && g_tuning().attn_mma_min_split > 0)
    a.min_split_tokens = g_tuning().attn_mma_min_split;
  a.mma_ring = g_tuning().attn_mma_ring;
  a.trace = e->trace.as<unsigned long long>();
  return a;
}

// One decoder layer for M decode rows whose sessions / positions are the
// engine's rows [row0, row0 + M).
void layer_decode(dial_b200_engine* e, LayerW& L, void* hidden, int M, cudaStream_t s,
                  int row0 = 0) {
  const float eps = e->cfg.rms_norm_eps;
  const GemmScratch gsv = e->scratch();
  const GemmScratch* gs = &gsv;
  unsigned long long* tr = e->trace.as<unsigned long long>();
  const int tag = static_cast<int>(&L - e->layers.data() + e->cfg.first_layer) << 8;
  run_linear(L.qkv, hidden, e->H, L.input_norm.p, eps, e->qkv.p, e->QKV, M, kEpiStore, s,
             e->status, gs, tr, tag | 0);
  AttnDecodeArgs a = decode_attn_args(e, L, M, row0);
  a.trace_tag = tag | 1;
  DIAL_CUDA(attn_decode_launch(a, e->cfg.act, s, g_tuning().pdl));
  run_linear(L.o, e->attn.p, e->QH * e->D, nullptr, eps, hidden, e->H, M, kEpiResidual, s, e->status,
             gs, tr, tag | 2);
  run_linear(L.gate_up, hidden, e->H, L.post_norm.p, eps, e->inter.p, e->I, M, kEpiSwiglu, s,
             e->status, gs, tr, tag | 3);
  run_linear(L.down, e->inter.p, e->I, nullptr, eps, hidden, e->H, M, kEpiResidual, s, e->status,
             gs, tr, tag | 4);
}

void layer_prefill(dial_b200_engine* e, LayerW& L, void* hidden, int M, int session, int p0,
                   cudaStream_t s) {
  const float eps = e->cfg.rms_norm_eps;
  const GemmScratch gsv = e->scratch();
  const GemmScratch* gs = &gsv;
  run_linear(L.qkv, hidden, e->H, L.input_norm.p, eps, e->qkv.p, e->QKV, M, kEpiStore, s, e->status,
             gs);
  AttnPrefillArgs a{};
  a.sh = e->shape();
  a.qkv = e->qkv.p;
  a.qkv_ld = e->QKV;
  a.q_norm_w = L.q_norm.p;
  a.k_norm_w = L.k_norm.p;
  a.cos = e->cos.p;
  a.sin = e->sin.p;
  a.kv = KvLayer{L.kpool.p, L.vpool.p};
  a.block_table = e->block_table.as<int32_t>() + static_cast<size_t>(session) * e->max_blocks;
  a.p0 = p0;
  a.M = M;
  a.rows_scratch = e->rows_scratch.as<int32_t>();
  a.out = e->attn.p;
  a.out_ld = e->QH * e->D;
  a.status = e->status;
  if (g_tuning().attn_tc) {
    a.q_rot = e->gemm_scratch.p;  // free between the QKV and o_proj GEMMs
    a.num_blocks = e->cfg.max_sessions * e->max_blocks;
  }
  DIAL_CUDA(attn_prefill_launch(a, e->cfg.act, s, g_tuning().pdl));
  run_linear(L.o, e->attn.p, e->QH * e->D, nullptr, eps, hidden, e->H, M, kEpiResidual, s, e->status,
             gs);
  run_linear(L.gate_up, hidden, e->H, L.post_norm.p, eps, e->inter.p, e->I, M, kEpiSwiglu, s,
             e->status, gs);
  run_linear(L.down, e->inter.p, e->I, nullptr, eps, hidden, e->H, M, kEpiResidual, s, e->status,
             gs);
}

void check_weights(dial_b200_engine* e, int first, int count) {
  for (int l = first; l < first + count; ++l) {
    LayerW& L = e->layer(l);
    DIAL_CHECK(L.qkv.ready() && L.o.ready() && L.gate_up.ready() && L.down.ready(),
               "layer %d has no weights loaded", l);
  }
}

void range_forward(dial_b200_engine* e, int first, int count, void* hidden, int64_t seq_len,
                   int session, int64_t index_pos, cudaStream_t s) {
  DIAL_CHECK(count >= 0, "negative layer count");
  DIAL_CHECK(seq_len >= 1 && seq_len <= e->cfg.max_tokens, "seq_len %lld outside [1, %d]",
             (long long)seq_len, e->cfg.max_tokens);
  DIAL_CHECK(session >= 0 && session < e->cfg.max_sessions, "session %d out of range", session);
  DIAL_CHECK(index_pos >= 0 && index_pos + seq_len <= e->cfg.max_seq_len,
             "positions [%lld, %lld) exceed the KV capacity %d", (long long)index_pos,
             (long long)(index_pos + seq_len), e->cfg.max_seq_len);
  DIAL_CHECK(hidden != nullptr, "hidden pointer is null");
  for (int l = first; l < first + count; ++l) (void)e->layer(l);  // validate before mutating
  check_weights(e, first, count);
  const int M = static_cast<int>(seq_len);
  if (M == 1 && index_pos > 0) {
    const int32_t sid = session, p = static_cast<int32_t>(index_pos);
    set_rows_decode(e, 1, &sid, &p, s);
    for (int l = first; l < first + count; ++l) layer_decode(e, e->layer(l), hidden, 1, s);
  } else {
    for (int l = first; l < first + count; ++l)
      layer_prefill(e, e->layer(l), hidden, M, session, static_cast<int>(index_pos), s);
  }
}

void head_forward(dial_b200_engine* e, const void* hidden, int rows, void* logits, int32_t* toks,
                  cudaStream_t s) {
  DIAL_CHECK(e->cfg.has_head, "this engine does not own the head");
  DIAL_CHECK(e->lm_head.ready(), "lm_head weights not loaded");
  DIAL_CHECK(rows <= e->max_rows_decode, "too many head rows (%d > %d)", rows,
             e->max_rows_decode);
  // ln_f + lm_head GEMV with the greedy argmax in its epilogue; the logits are
  // written only when the caller asks for them.
  GemvArgs a{};
  a.w = e->lm_head.d;
  a.x = hidden;
  a.x_ld = e->H;
  a.norm_w = e->final_norm.p;
  a.eps = e->cfg.rms_norm_eps;
  a.out = logits;
  a.out_ld = e->V;
  a.M = rows;
  a.status = e->status;
  a.amax_key = e->amax_key.as<unsigned long long>();
  a.amax_count = e->amax_count.as<int>();
  a.amax_tok = toks;
  a.trace = e->trace.as<unsigned long long>();
  a.trace_tag = (0xFFFF << 8) | 5;
  DIAL_CUDA(gemv_launch(a, e->lm_head.act, kEpiArgmax, true, s, g_tuning()));
}

// Write the trace records taken since the last dump as CSV (layer, op, cta,
// entry, wait released, staged, end in ns; 0 = not taken) and start over.
void dump_trace(dial_b200_engine* e) {
  if (!e->trace.p) return;
  unsigned long long hdr[2] = {0ull, 0ull};
  DIAL_CUDA(cudaMemcpy(hdr, e->trace.p, sizeof(hdr), cudaMemcpyDeviceToHost));
  const unsigned long long n = std::min(hdr[0], hdr[1]);
  std::vector<unsigned long long> r(n * kTraceWords);
  if (n)
    DIAL_CUDA(cudaMemcpy(r.data(), e->trace.as<unsigned long long>() + kTraceHeader, r.size() * 8,
                         cudaMemcpyDeviceToHost));
  FILE* f = std::fopen(e->trace_path.c_str(), "w");
  if (f) {
    std::fprintf(f, "layer,op,cta,entry,released,staged,end\n");
    for (unsigned long long i = 0; i < n; ++i) {
      const unsigned long long* q = &r[i * kTraceWords];
      const unsigned tag = static_cast<unsigned>(q[0] >> 32);
      std::fprintf(f, "%d,%u,%u,%llu,%llu,%llu,%llu\n", static_cast<int>(tag >> 8) == 0xFFFF ? -1
                   : static_cast<int>(tag >> 8), tag & 0xFF, static_cast<unsigned>(q[0] & 0xFFFFFFFFu),
                   q[1], q[2], q[3], q[4]);
    }
    std::fclose(f);
  }
  const unsigned long long zero = 0ull;
  DIAL_CUDA(cudaMemcpy(e->trace.p, &zero, 8, cudaMemcpyHostToDevice));
}

// Whole decode step on device buffers (tok_in, sid, pos -> tok_out).
void step_body(dial_b200_engine* e, int M, cudaStream_t s) {
  DIAL_CUDA(embed_launch(e->embed.p, e->tok_in.as<int32_t>(), M, e->V, e->H, e->hidden.p, e->H,
                         e->status, s, g_tuning().pdl));
  for (int li = 0; li < e->cfg.num_layers; ++li) layer_decode(e, e->layers[li], e->hidden.p, M, s);
  head_forward(e, e->hidden.p, M, nullptr, e->tok_out.as<int32_t>(), s);
}

void require_full_model(dial_b200_engine* e) {
  DIAL_CHECK(e->cfg.has_embed && e->cfg.has_head && e->cfg.first_layer == 0 &&
                 e->cfg.num_layers == e->cfg.num_hidden_layers,
             "this entry point needs an engine that owns the whole model");
  check_weights(e, 0, e->cfg.num_layers);
  DIAL_CHECK(e->lm_head.ready(), "lm_head weights not loaded");
}

void drop_graphs(dial_b200_engine* e) {
  cudaStreamSynchronize(e->stream);
  e->step_graphs.clear();
  e->loop_graphs.clear();
  e->stage_graphs.clear();
}

// Step graph of M rows (loop: tokens fed back on the device).
Graph* get_graph(dial_b200_engine* e, int M, bool loop) {
  auto& map = loop ? e->loop_graphs : e->step_graphs;
  auto it = map.find(M);
  if (it != map.end()) return it->second.get();
  cudaStream_t s = e->stream;
  auto g = std::make_unique<Graph>();
  DIAL_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  try {
    if (!loop) {
      DIAL_CUDA(cudaMemcpyAsync(e->tok_in.p, e->h_in, M * 4, cudaMemcpyHostToDevice, s));
      DIAL_CUDA(cudaMemcpyAsync(e->sid.p, e->h_in + M, M * 4, cudaMemcpyHostToDevice, s));
      DIAL_CUDA(cudaMemcpyAsync(e->pos.p, e->h_in + 2 * M, M * 4, cudaMemcpyHostToDevice, s));
    }
    step_body(e, M, s);
    if (loop)
      DIAL_CUDA(advance_launch(e->tok_out.as<int32_t>(), e->tok_in.as<int32_t>(),
                               e->pos.as<int32_t>(), M, s, g_tuning().pdl));
    if (!loop) {
      DIAL_CUDA(cudaMemcpyAsync(e->h_out, e->tok_out.p, M * 4, cudaMemcpyDeviceToHost, s));
      DIAL_CUDA(cudaMemcpyAsync(e->h_out + M, e->status, 4, cudaMemcpyDeviceToHost, s));
    }
  } catch (...) {
    cudaGraph_t tmp = nullptr;
    cudaStreamEndCapture(s, &tmp);
    if (tmp) cudaGraphDestroy(tmp);
    throw;
  }
  DIAL_CUDA(cudaStreamEndCapture(s, &g->g));
  DIAL_CUDA(cudaGraphInstantiate(&g->exec, g->g, 0));
  Graph* raw = g.get();
  map[M] = std::move(g);
  return raw;
}

void check_status(dial_b200_engine* e, int st) {
  if (st != 0)
    throw Error{DIAL_ERR_DEVICE, fmtstr("device status 0x%x recorded by a kernel", st)};
}

void decode_step_host(dial_b200_engine* e, int M, const int32_t* toks, const int32_t* sids,
                      const int32_t* pos, int32_t* next) {
  require_full_model(e);
  DIAL_CHECK(M >= 1 && M <= e->max_rows_decode && M <= 256, "rows %d outside [1, %d]", M,
             std::min(e->max_rows_decode, 256));
  for (int i = 0; i < M; ++i) {
    DIAL_CHECK(toks[i] >= 0 && toks[i] < e->V, "token %d outside the vocabulary", toks[i]);
    DIAL_CHECK(sids[i] >= 0 && sids[i] < e->cfg.max_sessions, "session %d out of range", sids[i]);
    DIAL_CHECK(pos[i] >= 0 && pos[i] < e->cfg.max_seq_len, "position %d outside the KV capacity",
               pos[i]);
  }
  Graph* g = get_graph(e, M, false);
  std::memcpy(e->h_in, toks, M * 4);
  std::memcpy(e->h_in + M, sids, M * 4);
  std::memcpy(e->h_in + 2 * M, pos, M * 4);
  DIAL_CUDA(cudaGraphLaunch(g->exec, e->stream));
  DIAL_CUDA(cudaStreamSynchronize(e->stream));
  std::memcpy(next, e->h_out, M * 4);
  check_status(e, e->h_out[M]);
}

}  // namespace

// ============================================================ C entry points
extern "C" {

uint32_t dial_b200_abi_version(void) { return DIAL_B200_ABI_VERSION; }

int dial_b200_device_status(int* status_out, int clear, char* err, size_t n) {
  return guarded(err, n, [&] {
    int dev = 0;
    DIAL_CUDA(cudaGetDevice(&dev));
    int* w = device_status_word(false);
    int v = 0;
    if (w) {
      DIAL_CUDA(cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost));
      if (clear) DIAL_CUDA(cudaMemset(w, 0, 4));
    }
    int v_noalloc = 0;
    DIAL_CUDA(noalloc_status(dev, clear != 0, &v_noalloc));
    if (status_out) *status_out = v != 0 ? v : v_noalloc;
  });
}

int dial_b200_w8a16_quantize(const void* weight, int dtype, int64_t out_dim, int64_t in_dim,
                             int8_t* q, float* scale, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(weight && q && scale, "null pointer argument");
    DIAL_CHECK(out_dim > 0 && in_dim > 0, "shape must be positive");
    DIAL_CHECK(dtype == DIAL_ACT_BF16 || dtype == DIAL_ACT_F16 || dtype == DIAL_ACT_F32,
               "unsupported weight dtype %d", dtype);
    const size_t wb = static_cast<size_t>(out_dim * in_dim) * act_size(dtype);
    DevBuf w(wb), dq(static_cast<size_t>(out_dim * in_dim)), ds(static_cast<size_t>(out_dim) * 4);
    DIAL_CUDA(cudaMemcpy(w.p, weight, wb, cudaMemcpyHostToDevice));
    const int src = dtype == DIAL_ACT_BF16 ? kSrcBf16 : (dtype == DIAL_ACT_F16 ? kSrcF16 : kSrcF32);
    DIAL_CUDA(quantize_rows(w.p, src, static_cast<int>(out_dim), static_cast<int>(in_dim),
                            dq.as<int8_t>(), ds.as<float>(), nullptr));
    DIAL_CUDA(cudaMemcpy(q, dq.p, dq.bytes, cudaMemcpyDeviceToHost));
    DIAL_CUDA(cudaMemcpy(scale, ds.p, ds.bytes, cudaMemcpyDeviceToHost));
  });
}

int dial_b200_w8a16_from_dense(const void* weight, int dtype, int64_t out_dim, int64_t in_dim,
                               int act, dial_b200_qlinear** out, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(weight && out, "null pointer argument");
    DIAL_CHECK(dtype == DIAL_ACT_BF16 || dtype == DIAL_ACT_F16 || dtype == DIAL_ACT_F32,
               "unsupported weight dtype %d", dtype);
    DIAL_CHECK(act == DIAL_ACT_BF16 || act == DIAL_ACT_F16, "W8A16 expects F16 or BF16 activations");
    DIAL_CHECK(out_dim > 0 && in_dim > 0, "shape must be positive");
    auto lin = std::make_unique<dial_b200_qlinear>();
    DIAL_CUDA(cudaGetDevice(&lin->device));
    const size_t wb = static_cast<size_t>(out_dim * in_dim) * act_size(dtype);
    DevBuf w(wb);
    DIAL_CUDA(cudaMemcpy(w.p, weight, wb, cudaMemcpyHostToDevice));
    const int src = dtype == DIAL_ACT_BF16 ? kSrcBf16 : (dtype == DIAL_ACT_F16 ? kSrcF16 : kSrcF32);
    build_w8a16_from_device_dense(lin->L, w.p, src, act, out_dim, in_dim, 0, nullptr);
    *out = lin.release();
  });
}

int dial_b200_qlinear_create(int fmt, int act, const void* codes, const void* scales,
                             float global_scale, int64_t in_dim, int64_t out_dim,
                             dial_b200_qlinear** out, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(out != nullptr, "null output handle");
    auto lin = std::make_unique<dial_b200_qlinear>();
    DIAL_CUDA(cudaGetDevice(&lin->device));
    cudaStream_t s = nullptr;
    build_linear_host(lin->L, fmt, act, codes, scales, global_scale, out_dim, in_dim, 0, s);
    *out = lin.release();
  });
}

void dial_b200_qlinear_destroy(dial_b200_qlinear* lin) { delete lin; }

int dial_b200_qlinear_forward(dial_b200_qlinear* lin, const void* x, void* y, int64_t rows,
                              void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(lin && x && y, "null pointer argument");
    DIAL_CHECK(rows >= 1 && rows < (1 << 24), "row count %lld out of range", (long long)rows);
    const int M = static_cast<int>(rows);
    GemmScratch sc;
    if (use_gemm(lin->L, M, true)) {
      const size_t need = gemm_scratch_bytes(M, lin->L.d.K_pad);
      if (lin->scratch.bytes < need) {
        DIAL_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
        lin->scratch.alloc(need);
      }
      sc.stage = lin->scratch.p;
    }
    run_linear(lin->L, x, static_cast<int>(lin->L.in_dim), nullptr, 0.f, y,
               static_cast<int>(lin->L.out_dim), M, kEpiStore, static_cast<cudaStream_t>(stream),
               device_status_word(), sc.stage ? &sc : nullptr);
  });
}

int64_t dial_b200_qlinear_in_dim(const dial_b200_qlinear* lin) { return lin ? lin->L.in_dim : -1; }
int64_t dial_b200_qlinear_out_dim(const dial_b200_qlinear* lin) { return lin ? lin->L.out_dim : -1; }
int64_t dial_b200_qlinear_resident_bytes(const dial_b200_qlinear* lin) {
  return lin ? lin->L.resident : -1;
}

int64_t dial_b200_attention_scratch_bytes(const dial_b200_attn_shape* sh, int64_t rows,
                                          int32_t splits) {
  if (!sh || rows < 1 || splits < 1) return -1;
  AttnShape a{};
  a.q_heads = sh->q_heads;
  a.kv_heads = sh->kv_heads;
  a.head_dim = sh->head_dim;
  return static_cast<int64_t>(attn_decode_scratch_bytes(a, static_cast<int>(rows), splits));
}

int dial_b200_attention_decode(const dial_b200_attn_shape* sh, const void* qkv, int64_t qkv_ld,
                               const void* q_norm_w, const void* k_norm_w, const void* cos,
                               const void* sin, void* k_pages, void* v_pages,
                               const int32_t* block_table, const int32_t* sids,
                               const int32_t* positions, void* out, int64_t out_ld, int64_t rows,
                               int32_t splits, void* scratch, void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(sh && qkv && q_norm_w && k_norm_w && cos && sin && k_pages && v_pages &&
                   block_table && sids && positions && out,
               "null pointer argument");
    DIAL_CHECK(sh->head_dim == 128, "head_dim must be 128 (got %d)", sh->head_dim);
    DIAL_CHECK(sh->q_heads > 0 && sh->kv_heads > 0 && sh->q_heads % sh->kv_heads == 0,
               "q_heads must be a positive multiple of kv_heads");
    const int rep = sh->q_heads / sh->kv_heads;
    DIAL_CHECK(rep == 1 || rep == 2 || rep == 4 || rep == 5 || rep == 8,
               "q_heads / kv_heads must be 1, 2, 4, 5 or 8 (got %d)", rep);
    DIAL_CHECK(sh->act == DIAL_ACT_BF16 || sh->act == DIAL_ACT_F16, "act must be BF16 or F16");
    DIAL_CHECK(rows >= 1 && rows <= 65535, "rows %lld outside [1, 65535]", (long long)rows);
    DIAL_CHECK(splits >= 1 && splits <= 32, "splits %d outside [1, 32]", splits);
    DIAL_CHECK(splits == 1 || scratch, "splits > 1 needs scratch");
    AttnDecodeArgs a{};
    a.sh.q_heads = sh->q_heads;
    a.sh.kv_heads = sh->kv_heads;
    a.sh.head_dim = sh->head_dim;
    a.sh.max_blocks = sh->max_blocks;
    a.sh.max_pos = sh->max_pos;
    a.sh.eps = sh->eps;
    a.qkv = qkv;
    a.qkv_ld = static_cast<int>(qkv_ld);
    a.q_norm_w = q_norm_w;
    a.k_norm_w = k_norm_w;
    a.cos = cos;
    a.sin = sin;
    a.kv = KvLayer{k_pages, v_pages};
    a.block_table = block_table;
    a.sid = sids;
    a.pos = positions;
    a.out = out;
    a.out_ld = static_cast<int>(out_ld);
    a.M = static_cast<int>(rows);
    a.splits = splits;
    if (splits > 1) {
      const size_t prow = static_cast<size_t>(rows) * sh->q_heads * splits;
      a.part_o = static_cast<float*>(scratch);
      a.part_ml = a.part_o + prow * 128;
      a.counters = reinterpret_cast<int*>(a.part_ml + prow * 2);
    }
    a.status = device_status_word();
    a.page_ring = 1;
    // token split as the engine: on by default, the cluster-merge variant for
    // steps of up to 4 rows with DIAL_B200_ATTN_TOKSPLIT=2, off with 0
    a.tok_split = g_tuning().attn_tok_split;
    DIAL_CHECK(sh->num_blocks >= 0, "num_blocks %d is negative", sh->num_blocks);
    a.num_blocks = sh->num_blocks;
    DIAL_CUDA(attn_decode_launch(a, sh->act, static_cast<cudaStream_t>(stream), false));
  });
}

int dial_b200_engine_create(const dial_b200_model_config* cfg, int device, dial_b200_engine** out,
                            char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(cfg && out, "null pointer argument");
    auto e = std::make_unique<dial_b200_engine>();
    engine_init(e.get(), *cfg, device);
    *out = e.release();
  });
}

void dial_b200_engine_destroy(dial_b200_engine* eng) {
  if (!eng) return;
  cudaSetDevice(eng->device);
  cudaStreamSynchronize(eng->stream);
  eng->step_graphs.clear();
  eng->loop_graphs.clear();
  eng->stage_graphs.clear();
  eng->link_graphs.clear();
  if (eng->link_next) cudaIpcCloseMemHandle(eng->link_next);
  if (eng->link_first && eng->link_first != eng->link_next) cudaIpcCloseMemHandle(eng->link_first);
  if (eng->h_in) cudaFreeHost(eng->h_in);
  if (eng->h_out) cudaFreeHost(eng->h_out);
  cudaStream_t s = eng->stream;
  delete eng;
  if (s) cudaStreamDestroy(s);
}

int dial_b200_engine_load_synthetic(dial_b200_engine* eng, uint64_t seed, const uint16_t* table,
                                    char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    drop_graphs(eng);
    engine_load_synthetic(eng, seed, table);
  });
}

int dial_b200_engine_set_linear(dial_b200_engine* eng, int layer, int which, int fmt,
                                const void* codes, const void* scales, float global_scale,
                                int64_t out_dim, int64_t in_dim, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    drop_graphs(eng);
    const int H = eng->H, I = eng->I;
    if (which == 4) {
      DIAL_CHECK(eng->cfg.has_head, "this engine does not own the head");
      DIAL_CHECK(out_dim == eng->V && in_dim == H, "lm_head must be [%d, %d]", eng->V, H);
      build_linear_host(eng->lm_head, fmt, eng->cfg.act, codes, scales, global_scale, out_dim,
                        in_dim, 0, eng->stream);
      return;
    }
    LayerW& L = eng->layer(layer);
    int64_t en = 0, ek = 0;
    Linear* dst = nullptr;
    int swiglu = 0;
    switch (which) {
      case 0: en = eng->QKV; ek = H; dst = &L.qkv; break;
      case 1: en = H; ek = eng->QH * eng->D; dst = &L.o; break;
      case 2: en = 2 * I; ek = H; dst = &L.gate_up; swiglu = 1; break;
      case 3: en = H; ek = I; dst = &L.down; break;
      default: DIAL_CHECK(false, "unknown linear slot %d", which);
    }
    DIAL_CHECK(out_dim == en && in_dim == ek, "linear slot %d must be [%lld, %lld], got [%lld, %lld]",
               which, (long long)en, (long long)ek, (long long)out_dim, (long long)in_dim);
    build_linear_host(*dst, fmt, eng->cfg.act, codes, scales, global_scale, out_dim, in_dim, swiglu,
                      eng->stream);
  });
}

int dial_b200_engine_set_tensor(dial_b200_engine* eng, int layer, int which, const void* host,
                                int64_t numel, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && host, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    drop_graphs(eng);
    DevBuf* dst = nullptr;
    int64_t expect = 0;
    if (which == 4) {
      DIAL_CHECK(eng->cfg.has_head, "this engine does not own the head");
      dst = &eng->final_norm;
      expect = eng->H;
    } else if (which == 5) {
      DIAL_CHECK(eng->cfg.has_embed, "this engine does not own the embedding");
      dst = &eng->embed;
      expect = static_cast<int64_t>(eng->V) * eng->H;
    } else {
      LayerW& L = eng->layer(layer);
      switch (which) {
        case 0: dst = &L.input_norm; expect = eng->H; break;
        case 1: dst = &L.post_norm; expect = eng->H; break;
        case 2: dst = &L.q_norm; expect = eng->D; break;
        case 3: dst = &L.k_norm; expect = eng->D; break;
        default: DIAL_CHECK(false, "unknown tensor slot %d", which);
      }
    }
    DIAL_CHECK(numel == expect, "tensor slot %d expects %lld elements, got %lld", which,
               (long long)expect, (long long)numel);
    DIAL_CUDA(cudaMemcpy(dst->p, host, numel * 2, cudaMemcpyHostToDevice));
  });
}

int dial_b200_layer_forward(dial_b200_engine* eng, int layer, void* hidden, int64_t seq_len,
                            int32_t session, int64_t index_pos, void* stream, char* err, size_t n) {
  return dial_b200_range_forward(eng, layer, 1, hidden, seq_len, session, index_pos, stream, err, n);
}

int dial_b200_range_forward(dial_b200_engine* eng, int first_layer, int count, void* hidden,
                            int64_t seq_len, int32_t session, int64_t index_pos, void* stream,
                            char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    range_forward(eng, first_layer, count, hidden, seq_len, session, index_pos,
                  static_cast<cudaStream_t>(stream));
  });
}

int dial_b200_batch_decode_forward(dial_b200_engine* eng, int first_layer, int count, void* hidden,
                                   int64_t rows, const int32_t* sids, const int32_t* positions,
                                   void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && hidden && sids && positions, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(rows >= 1 && rows <= eng->max_rows_decode, "rows %lld outside [1, %d]",
               (long long)rows, eng->max_rows_decode);
    for (int l = first_layer; l < first_layer + count; ++l) (void)eng->layer(l);
    check_weights(eng, first_layer, count);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    set_rows_decode(eng, static_cast<int>(rows), sids, positions, s);
    for (int l = first_layer; l < first_layer + count; ++l)
      layer_decode(eng, eng->layer(l), hidden, static_cast<int>(rows), s);
  });
}

int dial_b200_session_reset(dial_b200_engine* eng, int32_t session, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CHECK(session >= 0 && session < eng->cfg.max_sessions, "session %d out of range", session);
    // Paged KV: a session's context is defined by its positions; restarting
    // at index_pos 0 overwrites from the first page, so nothing to free.
  });
}

int dial_b200_embed(dial_b200_engine* eng, const int32_t* tokens_dev, int64_t rows, void* hidden,
                    void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && tokens_dev && hidden, "null pointer argument");
    DIAL_CHECK(eng->cfg.has_embed, "this engine does not own the embedding");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CUDA(embed_launch(eng->embed.p, tokens_dev, static_cast<int>(rows), eng->V, eng->H, hidden,
                           eng->H, eng->status, static_cast<cudaStream_t>(stream), false));
  });
}

int dial_b200_head(dial_b200_engine* eng, const void* hidden, int64_t rows, void* logits_dev,
                   int32_t* tokens_dev, void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && hidden && tokens_dev, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(rows >= 1 && rows <= 256, "head rows %lld outside [1, 256]", (long long)rows);
    head_forward(eng, hidden, static_cast<int>(rows), logits_dev, tokens_dev,
                 static_cast<cudaStream_t>(stream));
  });
}

int dial_b200_decode_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens,
                          const int32_t* sids, const int32_t* positions, int32_t* next, char* err,
                          size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && tokens && sids && positions && next, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    decode_step_host(eng, static_cast<int>(rows), tokens, sids, positions, next);
  });
}

int dial_b200_generate(dial_b200_engine* eng, int32_t session, const int32_t* prompt,
                       int64_t n_prompt, int64_t n_gen, int32_t* out_tokens, double* ttft_s,
                       double* decode_s, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && prompt && out_tokens, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    require_full_model(eng);
    DIAL_CHECK(n_prompt >= 1 && n_prompt <= eng->cfg.max_tokens, "prompt length %lld outside [1, %d]",
               (long long)n_prompt, eng->cfg.max_tokens);
    DIAL_CHECK(n_gen >= 1 && n_prompt + n_gen <= eng->cfg.max_seq_len,
               "prompt + generation exceeds the KV capacity %d", eng->cfg.max_seq_len);
    for (int64_t i = 0; i < n_prompt; ++i)
      DIAL_CHECK(prompt[i] >= 0 && prompt[i] < eng->V, "prompt token %d outside the vocabulary",
                 prompt[i]);
    cudaStream_t s = eng->stream;
    const auto t0 = std::chrono::steady_clock::now();
    DIAL_CUDA(cudaMemcpyAsync(eng->tok_in.p, prompt, n_prompt * 4, cudaMemcpyHostToDevice, s));
    DIAL_CUDA(embed_launch(eng->embed.p, eng->tok_in.as<int32_t>(), static_cast<int>(n_prompt),
                           eng->V, eng->H, eng->hidden.p, eng->H, eng->status, s, false));
    range_forward(eng, 0, eng->cfg.num_layers, eng->hidden.p, n_prompt, session, 0, s);
    head_forward(eng, static_cast<char*>(eng->hidden.p) + (n_prompt - 1) * eng->H * 2, 1, nullptr,
                 eng->tok_out.as<int32_t>(), s);
    int32_t first = 0;
    DIAL_CUDA(cudaMemcpyAsync(&first, eng->tok_out.p, 4, cudaMemcpyDeviceToHost, s));
    DIAL_CUDA(cudaStreamSynchronize(s));
    const auto t1 = std::chrono::steady_clock::now();
    int st = 0;
    DIAL_CUDA(cudaMemcpy(&st, eng->status, 4, cudaMemcpyDeviceToHost));
    check_status(eng, st);
    out_tokens[0] = first;
    int32_t tok = first;
    for (int64_t i = 1; i < n_gen; ++i) {
      const int32_t p = static_cast<int32_t>(n_prompt + i - 1);
      int32_t next = 0;
      decode_step_host(eng, 1, &tok, &session, &p, &next);
      out_tokens[i] = next;
      tok = next;
    }
    const auto t2 = std::chrono::steady_clock::now();
    if (ttft_s) *ttft_s = std::chrono::duration<double>(t1 - t0).count();
    if (decode_s) *decode_s = std::chrono::duration<double>(t2 - t1).count();
  });
}

int dial_b200_decode_loop_prepare(dial_b200_engine* eng, int64_t rows, const int32_t* toks,
                                  const int32_t* sids, const int32_t* pos, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && toks && sids && pos, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    require_full_model(eng);
    const int M = static_cast<int>(rows);
    DIAL_CHECK(M >= 1 && M <= eng->max_rows_decode && M <= 256, "rows %d out of range", M);
    for (int i = 0; i < M; ++i) {
      DIAL_CHECK(toks[i] >= 0 && toks[i] < eng->V, "token out of range");
      DIAL_CHECK(sids[i] >= 0 && sids[i] < eng->cfg.max_sessions, "session out of range");
      DIAL_CHECK(pos[i] >= 0 && pos[i] < eng->cfg.max_seq_len, "position out of range");
    }
    // loop replays still in flight on the engine stream read these buffers
    DIAL_CUDA(cudaStreamSynchronize(eng->stream));
    DIAL_CUDA(cudaMemcpy(eng->tok_in.p, toks, M * 4, cudaMemcpyHostToDevice));
    DIAL_CUDA(cudaMemcpy(eng->sid.p, sids, M * 4, cudaMemcpyHostToDevice));
    DIAL_CUDA(cudaMemcpy(eng->pos.p, pos, M * 4, cudaMemcpyHostToDevice));
    (void)get_graph(eng, M, true);
  });
}

int dial_b200_decode_loop_run(dial_b200_engine* eng, int64_t rows, int64_t n_steps, char* err,
                              size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    auto it = eng->loop_graphs.find(rows);
    DIAL_CHECK(it != eng->loop_graphs.end(), "decode loop for %lld rows not prepared",
               (long long)rows);
    for (int64_t i = 0; i < n_steps; ++i) DIAL_CUDA(cudaGraphLaunch(it->second->exec, eng->stream));
  });
}

int dial_b200_decode_loop_state(dial_b200_engine* eng, int64_t rows, int32_t* toks, int32_t* pos,
                                char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CUDA(cudaStreamSynchronize(eng->stream));
    if (toks) DIAL_CUDA(cudaMemcpy(toks, eng->tok_in.p, rows * 4, cudaMemcpyDeviceToHost));
    if (pos) DIAL_CUDA(cudaMemcpy(pos, eng->pos.p, rows * 4, cudaMemcpyDeviceToHost));
    int st = 0;
    DIAL_CUDA(cudaMemcpy(&st, eng->status, 4, cudaMemcpyDeviceToHost));
    dump_trace(eng);
    check_status(eng, st);
  });
}

int dial_b200_stage_prepare(dial_b200_engine* eng, int64_t rows, const int32_t* sids,
                            const int32_t* positions, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && sids && positions, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    const int M = static_cast<int>(rows);
    DIAL_CHECK(M >= 1 && M <= eng->max_rows_decode && M <= 256, "rows %d out of range", M);
    for (int i = 0; i < M; ++i) {
      DIAL_CHECK(sids[i] >= 0 && sids[i] < eng->cfg.max_sessions, "session %d out of range",
                 sids[i]);
      DIAL_CHECK(positions[i] >= 0 && positions[i] < eng->cfg.max_seq_len,
                 "position %d outside the KV capacity %d", positions[i], eng->cfg.max_seq_len);
    }
    DIAL_CUDA(cudaStreamSynchronize(eng->stream));
    DIAL_CUDA(cudaMemcpy(eng->sid.p, sids, M * 4, cudaMemcpyHostToDevice));
    DIAL_CUDA(cudaMemcpy(eng->pos.p, positions, M * 4, cudaMemcpyHostToDevice));
  });
}

int dial_b200_stage_step_rows(dial_b200_engine* eng, int64_t row_offset, int64_t rows,
                              const int32_t* tokens_dev, void* hidden, int32_t* tokens_out_dev,
                              void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && hidden, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    const int M = static_cast<int>(rows);
    const int r0 = static_cast<int>(row_offset);
    DIAL_CHECK(M >= 1 && M <= 256, "rows %d out of range", M);
    DIAL_CHECK(r0 >= 0 && r0 + M <= eng->max_rows_decode,
               "rows [%d, %d) outside the %d decode rows", r0, r0 + M, eng->max_rows_decode);
    DIAL_CHECK(!eng->cfg.has_embed || tokens_dev, "the first stage needs device token ids");
    DIAL_CHECK(!eng->cfg.has_head || tokens_out_dev, "the last stage needs a token output");
    check_weights(eng, eng->cfg.first_layer, eng->cfg.num_layers);
    if (eng->cfg.has_head) DIAL_CHECK(eng->lm_head.ready(), "lm_head weights not loaded");
    const auto key = std::make_tuple(rows | (static_cast<int64_t>(r0) << 32),
                                     static_cast<const void*>(tokens_dev),
                                     static_cast<const void*>(hidden),
                                     static_cast<const void*>(tokens_out_dev));
    auto it = eng->stage_graphs.find(key);
    if (it == eng->stage_graphs.end()) {
      cudaStream_t s = eng->stream;
      auto g = std::make_unique<Graph>();
      DIAL_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        if (eng->cfg.has_embed)
          DIAL_CUDA(embed_launch(eng->embed.p, tokens_dev, M, eng->V, eng->H, hidden, eng->H,
                                 eng->status, s, g_tuning().pdl));
        for (int li = 0; li < eng->cfg.num_layers; ++li)
          layer_decode(eng, eng->layers[li], hidden, M, s, r0);
        if (eng->cfg.has_head) head_forward(eng, hidden, M, nullptr, tokens_out_dev, s);
        DIAL_CUDA(advance_launch(nullptr, nullptr, eng->pos.as<int32_t>() + r0, M, s,
                                 g_tuning().pdl));
      } catch (...) {
        cudaGraph_t tmp = nullptr;
        cudaStreamEndCapture(s, &tmp);
        if (tmp) cudaGraphDestroy(tmp);
        throw;
      }
      DIAL_CUDA(cudaStreamEndCapture(s, &g->g));
      DIAL_CUDA(cudaGraphInstantiate(&g->exec, g->g, 0));
      it = eng->stage_graphs.emplace(key, std::move(g)).first;
    }
    DIAL_CUDA(cudaGraphLaunch(it->second->exec, static_cast<cudaStream_t>(stream)));
  });
}

int dial_b200_stage_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_dev,
                         void* hidden, int32_t* tokens_out_dev, void* stream, char* err,
                         size_t n) {
  return dial_b200_stage_step_rows(eng, 0, rows, tokens_dev, hidden, tokens_out_dev, stream, err,
                                   n);
}

int dial_b200_stage_link_handle(dial_b200_engine* eng, void* handle_out, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && handle_out, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    if (!eng->link_in.p) {
      eng->link_in.alloc(link_inbox_bytes(eng->max_rows_decode, eng->H));
      DIAL_CUDA(cudaMemset(eng->link_in.p, 0, eng->link_in.bytes));
      eng->link_cnt.alloc(4 * sizeof(uint64_t));
      DIAL_CUDA(cudaMemset(eng->link_cnt.p, 0, eng->link_cnt.bytes));
    }
    cudaIpcMemHandle_t h;
    DIAL_CUDA(cudaIpcGetMemHandle(&h, eng->link_in.p));
    std::memcpy(handle_out, &h, sizeof(h));
  });
}

int dial_b200_stage_link_open(dial_b200_engine* eng, const void* next_handle,
                              const void* first_handle, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(eng->link_in.p, "call dial_b200_stage_link_handle first");
    DIAL_CHECK(!eng->link_next && !eng->link_first, "the stage link is already open");
    DIAL_CHECK(eng->cfg.has_head || next_handle, "a stage without the head needs the next stage");
    DIAL_CHECK(!eng->cfg.has_head || eng->cfg.has_embed || first_handle,
               "the last stage needs the first stage's inbox");
    auto open = [&](const void* hp) -> uint8_t* {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, hp, sizeof(h));
      void* p = nullptr;
      DIAL_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
      return static_cast<uint8_t*>(p);
    };
    if (!eng->cfg.has_head) eng->link_next = open(next_handle);
    if (eng->cfg.has_head && !eng->cfg.has_embed) eng->link_first = open(first_handle);
  });
}

int dial_b200_stage_link_step(dial_b200_engine* eng, int64_t rows, const int32_t* tokens_dev,
                              void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    const int M = static_cast<int>(rows);
    DIAL_CHECK(M >= 1 && M <= eng->max_rows_decode && M <= 256, "rows %d out of range", M);
    DIAL_CHECK(!(eng->cfg.has_embed && eng->cfg.has_head),
               "an engine that owns the whole model has no stage link");
    DIAL_CHECK((eng->cfg.has_head ? eng->link_first : eng->link_next) != nullptr,
               "the stage link is not open");
    DIAL_CHECK(eng->cfg.has_embed || !tokens_dev, "only the first stage takes token ids");
    check_weights(eng, eng->cfg.first_layer, eng->cfg.num_layers);
    if (eng->cfg.has_head) DIAL_CHECK(eng->lm_head.ready(), "lm_head weights not loaded");
    // tokens_dev (first stage): this step's tokens come from the caller (the
    // first step after a prepare or a finish); null: from the last stage
    const auto key = std::make_tuple(rows, static_cast<const void*>(tokens_dev));
    auto it = eng->link_graphs.find(key);
    if (it == eng->link_graphs.end()) {
      cudaStream_t s = eng->stream;
      auto g = std::make_unique<Graph>();
      uint64_t* cnt = eng->link_cnt.as<uint64_t>();
      const uint8_t* inbox = eng->link_in.as<uint8_t>();
      const int mr = eng->max_rows_decode;
      const bool pdl = g_tuning().pdl;
      DIAL_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        if (eng->cfg.has_embed) {
          const int32_t* toks = tokens_dev;
          if (!toks) {
            DIAL_CUDA(link_recv_launch(inbox, kLinkTokens, mr, cnt + 1, eng->tok_in.p, M * 4,
                                       eng->status, s));
            toks = eng->tok_in.as<int32_t>();
          }
          DIAL_CUDA(embed_launch(eng->embed.p, toks, M, eng->V, eng->H, eng->hidden.p, eng->H,
                                 eng->status, s, pdl));
        } else {
          DIAL_CUDA(link_recv_launch(inbox, kLinkHidden, mr, cnt + 0, eng->hidden.p,
                                     static_cast<size_t>(M) * eng->H * 2, eng->status, s));
        }
        for (int li = 0; li < eng->cfg.num_layers; ++li)
          layer_decode(eng, eng->layers[li], eng->hidden.p, M, s);
        if (eng->cfg.has_head) {
          head_forward(eng, eng->hidden.p, M, nullptr, eng->tok_out.as<int32_t>(), s);
          DIAL_CUDA(link_send_launch(eng->link_first, kLinkTokens, mr, cnt + 3, eng->tok_out.p,
                                     M * 4, eng->status, s, pdl));
        } else {
          DIAL_CUDA(link_send_launch(eng->link_next, kLinkHidden, mr, cnt + 2, eng->hidden.p,
                                     static_cast<size_t>(M) * eng->H * 2, eng->status, s, pdl));
        }
        DIAL_CUDA(advance_launch(nullptr, nullptr, eng->pos.as<int32_t>(), M, s, pdl));
      } catch (...) {
        cudaGraph_t tmp = nullptr;
        cudaStreamEndCapture(s, &tmp);
        if (tmp) cudaGraphDestroy(tmp);
        throw;
      }
      DIAL_CUDA(cudaStreamEndCapture(s, &g->g));
      DIAL_CUDA(cudaGraphInstantiate(&g->exec, g->g, 0));
      it = eng->link_graphs.emplace(key, std::move(g)).first;
    }
    DIAL_CUDA(cudaGraphLaunch(it->second->exec, static_cast<cudaStream_t>(stream)));
  });
}

int dial_b200_stage_link_finish(dial_b200_engine* eng, int64_t rows, int32_t* tokens_host,
                                void* stream, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(eng->cfg.has_embed && !eng->cfg.has_head, "only the first stage finishes a run");
    DIAL_CHECK(eng->link_in.p, "the stage link is not open");
    const int M = static_cast<int>(rows);
    DIAL_CHECK(M >= 1 && M <= eng->max_rows_decode, "rows %d out of range", M);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DIAL_CUDA(link_recv_launch(eng->link_in.as<uint8_t>(), kLinkTokens, eng->max_rows_decode,
                               eng->link_cnt.as<uint64_t>() + 1, eng->tok_in.p, M * 4, eng->status,
                               s));
    if (tokens_host) {
      DIAL_CUDA(cudaMemcpyAsync(tokens_host, eng->tok_in.p, M * 4, cudaMemcpyDeviceToHost, s));
      DIAL_CUDA(cudaStreamSynchronize(s));
      int st = 0;
      DIAL_CUDA(cudaMemcpy(&st, eng->status, 4, cudaMemcpyDeviceToHost));
      check_status(eng, st);
    }
  });
}

void* dial_b200_engine_stream(dial_b200_engine* eng) { return eng ? eng->stream : nullptr; }

int dial_b200_session_fill_random(dial_b200_engine* eng, int32_t session, int64_t length,
                                  uint64_t seed, const uint16_t* table_host, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng && table_host, "null pointer argument");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(session >= 0 && session < eng->cfg.max_sessions, "session out of range");
    DIAL_CHECK(length >= 0 && length <= eng->cfg.max_seq_len, "length outside the KV capacity");
    DevBuf table(65536 * 2);
    DIAL_CUDA(cudaMemcpy(table.p, table_host, table.bytes, cudaMemcpyHostToDevice));
    const int64_t nblk = (length + kPageTokens - 1) / kPageTokens;
    const int64_t per_block = static_cast<int64_t>(eng->KVH) * kPageTokens * eng->D;
    const int64_t off = static_cast<int64_t>(session) * eng->max_blocks * per_block;
    for (int li = 0; li < eng->cfg.num_layers; ++li) {
      LayerW& L = eng->layers[li];
      const uint64_t st = (static_cast<uint64_t>(eng->cfg.first_layer + li) << 20) ^
                          (static_cast<uint64_t>(session) << 4) ^ 0xCA;
      DIAL_CUDA(synth_table_fill(L.kpool.as<uint16_t>() + off, nblk * per_block, seed, st, 0,
                                 table.as<uint16_t>(), eng->stream));
      DIAL_CUDA(synth_table_fill(L.vpool.as<uint16_t>() + off, nblk * per_block, seed, st + 1, 0,
                                 table.as<uint16_t>(), eng->stream));
    }
    DIAL_CUDA(cudaStreamSynchronize(eng->stream));
  });
}

namespace {

int64_t kernel_nodes(cudaGraph_t g) {
  size_t n = 0;
  DIAL_CUDA(cudaGraphGetNodes(g, nullptr, &n));
  std::vector<cudaGraphNode_t> nodes(n);
  DIAL_CUDA(cudaGraphGetNodes(g, nodes.data(), &n));
  int64_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    DIAL_CUDA(cudaGraphNodeGetType(nodes[i], &t));
    if (t == cudaGraphNodeTypeKernel) ++k;
  }
  return k;
}

}  // namespace

int64_t dial_b200_step_kernel_count(dial_b200_engine* eng, int64_t rows) {
  if (!eng || rows < 1) return -1;
  try {
    DIAL_CUDA(cudaSetDevice(eng->device));
    require_full_model(eng);
    DIAL_CHECK(rows <= eng->max_rows_decode && rows <= 256, "rows out of range");
    return kernel_nodes(get_graph(eng, static_cast<int>(rows), true)->g);
  } catch (...) {
    return -1;
  }
}

int64_t dial_b200_prefill_kernel_count(dial_b200_engine* eng, int64_t n_prompt) {
  if (!eng || n_prompt < 1) return -1;
  try {
    DIAL_CUDA(cudaSetDevice(eng->device));
    require_full_model(eng);
    DIAL_CHECK(n_prompt <= eng->cfg.max_tokens && n_prompt <= eng->cfg.max_seq_len,
               "prompt length out of range");
    // capture (never launched) the device work of dial_b200_generate's
    // prefill: embed, every layer at positions [0, n_prompt) of session 0, head
    cudaStream_t s = eng->stream;
    DIAL_CUDA(cudaStreamSynchronize(s));
    Graph g;
    DIAL_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      DIAL_CUDA(embed_launch(eng->embed.p, eng->tok_in.as<int32_t>(), static_cast<int>(n_prompt),
                             eng->V, eng->H, eng->hidden.p, eng->H, eng->status, s, false));
      for (int l = 0; l < eng->cfg.num_layers; ++l)
        layer_prefill(eng, eng->layers[l], eng->hidden.p, static_cast<int>(n_prompt), 0, 0, s);
      head_forward(eng, eng->hidden.p, 1, nullptr, eng->tok_out.as<int32_t>(), s);
    } catch (...) {
      cudaGraph_t tmp = nullptr;
      cudaStreamEndCapture(s, &tmp);
      if (tmp) cudaGraphDestroy(tmp);
      throw;
    }
    DIAL_CUDA(cudaStreamEndCapture(s, &g.g));
    return kernel_nodes(g.g);
  } catch (...) {
    return -1;
  }
}

int dial_b200_engine_linear_replay(dial_b200_engine* eng, int layer, int which, int64_t rows,
                                   int64_t iters, char* err, size_t n) {
  return guarded(err, n, [&] {
    DIAL_CHECK(eng, "null engine");
    DIAL_CUDA(cudaSetDevice(eng->device));
    DIAL_CHECK(rows >= 1 && rows <= eng->cfg.max_tokens, "rows out of range");
    const float eps = eng->cfg.rms_norm_eps;
    cudaStream_t s = eng->stream;
    const int M = static_cast<int>(rows);
    // the GEMM scratch of the decode step: rows >= 16 take the tcgen05 GEMM
    // exactly as layer_decode does
    const GemmScratch gsv = eng->scratch();
    const GemmScratch* gs = &gsv;
    // layer < 0: rotate over every owned layer so that no launch finds its
    // weights in L2
    for (int64_t i = 0; i < iters; ++i) {
      const int layer_i = layer >= 0 ? layer
                                     : eng->cfg.first_layer +
                                           static_cast<int>(i % eng->cfg.num_layers);
      if (which == 4) {
        DIAL_CHECK(eng->lm_head.ready(), "lm_head not loaded");
        head_forward(eng, eng->hidden.p, M, nullptr, eng->tok_out.as<int32_t>(), s);
        continue;
      }
      LayerW& L = eng->layer(layer_i);
      switch (which) {
        case 0: run_linear(L.qkv, eng->hidden.p, eng->H, L.input_norm.p, eps, eng->qkv.p, eng->QKV,
                           M, kEpiStore, s, eng->status, gs); break;
        case 1: run_linear(L.o, eng->attn.p, eng->QH * eng->D, nullptr, eps, eng->hidden.p, eng->H,
                           M, kEpiResidual, s, eng->status, gs); break;
        case 2: run_linear(L.gate_up, eng->hidden.p, eng->H, L.post_norm.p, eps, eng->inter.p,
                           eng->I, M, kEpiSwiglu, s, eng->status, gs); break;
        case 3: run_linear(L.down, eng->inter.p, eng->I, nullptr, eps, eng->hidden.p, eng->H, M,
                           kEpiResidual, s, eng->status, gs); break;
        default: DIAL_CHECK(false, "unknown linear slot %d", which);
      }
    }
  });
}

int64_t dial_b200_engine_linear_bytes(dial_b200_engine* eng, int layer, int which, int64_t rows) {
  if (!eng || rows < 1) return -1;
  try {
    const Linear* L = nullptr;
    if (which == 4) {
      L = &eng->lm_head;
    } else {
      LayerW& lw = eng->layer(layer);
      L = which == 0 ? &lw.qkv : which == 1 ? &lw.o : which == 2 ? &lw.gate_up : &lw.down;
    }
    if (!L->ready()) return -1;
    const int64_t N = L->out_dim, K = L->in_dim;
    const int64_t out_cols = L->d.swiglu ? N / 2 : N;
    int64_t bytes = L->resident;                 // weights + scales
    bytes += rows * K * 2;                       // activations in
    bytes += rows * out_cols * 2;                // activations out
    if (which == 1 || which == 3) bytes += rows * out_cols * 2;  // residual read
    return bytes;
  } catch (...) {
    return -1;
  }
}

}  // extern "C"
