// dial_b200_attention_decode_noalloc: the fused decode attention op with its
// split-KV scratch in a file-scope device array instead of caller memory.
//
// Who needs it: callers that may not allocate device memory at all on the
// call path -- code running inside a CUDA stream capture (a cudaMalloc there
// breaks the capture), a serving loop that pins its memory budget up front
// and treats any later allocation as a failure, and foreign-language hosts
// (the reference's Rust side binds through FFI) that cannot easily own and
// zero a device buffer with the right lifetime.  The dial_b200_attention_decode
// entry point needs such a buffer for splits > 1; this one needs none.
//
// The scratch lives in `g_scratch` below, one copy per device (every CUDA
// context gets its own instance of a __device__ variable).  The first call on
// a device looks up its address with cudaGetSymbolAddress and zero-fills the
// split counters and the status word (cudaMemset, which allocates nothing);
// the kernels then leave the counters at zero after every call.  That setup
// can load the module and synchronizes, so the first call on each device
// belongs before any stream capture.  Calls that overlap in time on one
// device (two streams, two host threads) share the one scratch and race;
// serialize them.
//
// Device-side status (a position outside the KV capacity, a bounded wait that
// expired) goes to the status word inside the scratch; dial_b200_device_status
// reports it (noalloc_status below) and, when asked to clear it, also
// re-zeroes the split counters, since a call that gave up early can leave
// them non-zero.  The call uses the same kernel forms as
// dial_b200_attention_decode (page ring for steps of up to 4 rows, token split
// for more rows in groups of 4 query heads).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/dial_b200.h"
#include "attention.h"

namespace dialb200 {
namespace {

// Partial rows (rows * q_heads * splits) and per-(row, kv head) counters the
// static scratch holds: 2048 partial rows cover Qwen3-8B (32 q heads) at 4
// rows x 16 splits or 1 row x 32 splits; about 1.07 MB of device memory.
constexpr int kMaxPartRows = DIAL_B200_NOALLOC_MAX_PART_ROWS;
constexpr int kMaxCounters = DIAL_B200_NOALLOC_MAX_COUNTERS;

struct NoAllocScratch {
  float part_o[kMaxPartRows * 128];  // [rows][q_heads][splits][128]
  float part_ml[kMaxPartRows * 2];   // [rows][q_heads][splits][2]
  int counters[kMaxCounters];        // [rows][kv_heads]; zero between calls
  int status;                        // device status of this entry point
};

static __device__ __align__(256) NoAllocScratch g_scratch;

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
NoAllocScratch* g_addr[kMaxDevices] = {nullptr};

int fail(char* err, size_t n, int code, const char* f, ...) {
  if (err && n) {
    va_list ap;
    va_start(ap, f);
    std::vsnprintf(err, n, f, ap);
    va_end(ap);
  }
  return code;
}

// Address of this device's scratch; on the first call per device, looks it up
// and clears the counters and the status word.
cudaError_t scratch_for_device(int dev, NoAllocScratch** out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    NoAllocScratch* s = static_cast<NoAllocScratch*>(p);
    e = cudaMemset(s->counters, 0, sizeof(s->counters) + sizeof(s->status));
    if (e != cudaSuccess) return e;
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    g_addr[dev] = s;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace

cudaError_t noalloc_status(int dev, bool clear, int* out) {
  *out = 0;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  NoAllocScratch* s = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    s = g_addr[dev];
  }
  if (!s) return cudaSuccess;
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, &s->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return e;
  *out = v;
  if (clear && v != 0) {
    e = cudaMemset(s->counters, 0, sizeof(s->counters) + sizeof(s->status));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
  }
  return e;
}

}  // namespace dialb200

using namespace dialb200;

extern "C" int dial_b200_attention_decode_noalloc(
    const dial_b200_attn_shape* sh, const void* qkv, int64_t qkv_ld, const void* q_norm_w,
    const void* k_norm_w, const void* cos, const void* sin, void* k_pages, void* v_pages,
    const int32_t* block_table, const int32_t* sids, const int32_t* positions, void* out,
    int64_t out_ld, int64_t rows, int32_t splits, void* stream, char* err, size_t n) {
  if (!(sh && qkv && q_norm_w && k_norm_w && cos && sin && k_pages && v_pages && block_table &&
        sids && positions && out))
    return fail(err, n, DIAL_ERR_INVALID, "null pointer argument");
  if (sh->head_dim != 128)
    return fail(err, n, DIAL_ERR_INVALID, "head_dim must be 128 (got %d)", sh->head_dim);
  if (sh->q_heads <= 0 || sh->kv_heads <= 0 || sh->q_heads % sh->kv_heads != 0)
    return fail(err, n, DIAL_ERR_INVALID, "q_heads must be a positive multiple of kv_heads");
  const int rep = sh->q_heads / sh->kv_heads;
  if (!(rep == 1 || rep == 2 || rep == 4 || rep == 5 || rep == 8))
    return fail(err, n, DIAL_ERR_INVALID, "q_heads / kv_heads must be 1, 2, 4, 5 or 8 (got %d)",
                rep);
  if (sh->act != DIAL_ACT_BF16 && sh->act != DIAL_ACT_F16)
    return fail(err, n, DIAL_ERR_INVALID, "act must be BF16 or F16");
  if (rows < 1 || rows > 65535)
    return fail(err, n, DIAL_ERR_INVALID, "rows %lld outside [1, 65535]", (long long)rows);
  if (splits < 1 || splits > 32)
    return fail(err, n, DIAL_ERR_INVALID, "splits %d outside [1, 32]", splits);
  const long long part_rows = static_cast<long long>(rows) * sh->q_heads * splits;
  const long long counters = static_cast<long long>(rows) * sh->kv_heads;
  if (splits > 1 && part_rows > kMaxPartRows)
    return fail(err, n, DIAL_ERR_INVALID,
                "rows * q_heads * splits = %lld exceeds the static scratch limit of %d partial "
                "rows; lower splits or rows, or use dial_b200_attention_decode",
                part_rows, kMaxPartRows);
  if (splits > 1 && counters > kMaxCounters)
    return fail(err, n, DIAL_ERR_INVALID,
                "rows * kv_heads = %lld exceeds the static scratch limit of %d counters; lower "
                "rows, or use dial_b200_attention_decode",
                counters, kMaxCounters);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(err, n, DIAL_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(err, n, DIAL_ERR_INVALID, "device index %d out of range", dev);
  NoAllocScratch* s = nullptr;
  e = scratch_for_device(dev, &s);
  if (e != cudaSuccess)
    return fail(err, n, DIAL_ERR_CUDA, "static scratch setup failed: %s", cudaGetErrorString(e));

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
  a.part_o = s->part_o;
  a.part_ml = s->part_ml;
  a.counters = s->counters;
  a.status = &s->status;
  a.page_ring = 1;
  a.tok_split = 1;
  e = attn_decode_launch(a, sh->act, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess)
    return fail(err, n, DIAL_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
  return DIAL_OK;
}
