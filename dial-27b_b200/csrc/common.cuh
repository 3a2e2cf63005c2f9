// Shared device helpers for the DIAL B200 kernels (sm_100a only).
//
// PTX wrappers for mbarriers, 1-D bulk async copies (the TMA engine's
// untiled form), programmatic dependent launch and the register-fed
// m16n8k16 tensor-core MMA used by the decode GEMV, plus bounded waits that
// report a status word instead of hanging.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "trace.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "dial_b200 kernels target sm_100a only"
#endif

namespace dialb200 {

// Status codes written to the library's device status word.
enum DevStatus : int {
  kStatusOk = 0,
  kStatusFullWaitTimeout = 0x101,   // consumer gave up waiting for a weight stage
  kStatusEmptyWaitTimeout = 0x102,  // producer gave up waiting for a free ring slot
  kStatusDrainTimeout = 0x103,      // in-flight copies did not land during error drain
  kStatusBadArgs = 0x104,
  kStatusAttnCounter = 0x201,
  kStatusAttnRing = 0x202,          // decode-attention page ring wait timed out
  kStatusLinkTimeout = 0x301,       // a stage link receive waited past the bound
};

// Wall-clock bound (ns) on any spin-wait; well above any legitimate wait.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Opt-in timeline of the decode step (DIAL_B200_TRACE=<csv> on the engine):
// thread 0 of every CTA appends one record (trace.h), [tag << 32 | CTA] and
// four %globaltimer stamps (0 = not taken), after the header words
// trace[0] = records written, trace[1] = capacity.
__device__ __forceinline__ void trace_record(unsigned long long* trace, int tag,
                                             const unsigned long long (&t)[4]) {
  if (!trace) return;
  const unsigned long long i = atomicAdd(trace, 1ull);
  if (i >= trace[1]) return;
  unsigned long long* r = trace + kTraceHeader + i * kTraceWords;
  const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  r[0] = (static_cast<unsigned long long>(static_cast<unsigned>(tag)) << 32) | cta;
  r[1] = t[0];
  r[2] = t[1];
  r[3] = t[2];
  r[4] = t[3];
}

__device__ __forceinline__ void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `ns` nanoseconds pass, instead of spinning on the issue
// slots the other warps of the SM need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// mbar_wait whose retries sleep in the barrier (mbar_try_wait_sleep).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* status,
                                                int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((it & 15u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      set_status(status, code);
      return false;
    }
  }
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in
// the status word) once kWaitLimitNs has elapsed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      set_status(status, code);
      return false;
    }
  }
}

// Orders this thread's generic shared-memory accesses before later
// async-proxy ones (a bulk or TMA copy that refills a ring slot the thread
// has just read, or an MMA that reads what it has just written).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------ bulk async copies
// 1-D global -> shared copy on the TMA engine, completing on an mbarrier.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read once per pass (streamed weights): evicted first,
// so that the small tensors every layer re-reads stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* src_gmem, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}

// ------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ----------------------------------------------------------- tensor MMA
// D = A(16x16, row) * B(16x8, col) + D with f32 accumulation.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// --------------------------------------------------- weight conversions
// Weight bytes are stored offset by 0x80 (u = q + 128).  Building the f16
// bit pattern 0x6400|u gives 1024+u exactly; subtracting 1152 leaves q.
__device__ __forceinline__ uint32_t u8pair_to_f16x2(uint32_t word, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(word), "r"(0x64646464u), "r"(sel));
  const __half2 h = __hsub2(*reinterpret_cast<__half2*>(&r), __half2(__float2half_rn(1152.f),
                                                                    __float2half_rn(1152.f)));
  return *reinterpret_cast<const uint32_t*>(&h);
}
// bytes 0,1 -> (lo, hi) halves ; bytes 2,3 -> (lo, hi) halves
__device__ __forceinline__ uint32_t i8_lo_pair(uint32_t w) { return u8pair_to_f16x2(w, 0x5140u); }
__device__ __forceinline__ uint32_t i8_hi_pair(uint32_t w) { return u8pair_to_f16x2(w, 0x7362u); }

// Two e4m3 codes (low byte -> low half) to f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// Eight e2m1 codes (one 32-bit word, byte j -> o[j], low nibble -> low
// half) to four f16x2, exact.
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// -------------------------------------------------------- act helpers
template <typename T>
struct ActTraits;
template <>
struct ActTraits<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};
template <>
struct ActTraits<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

// 2^e for small integer e, exact.
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace dialb200
