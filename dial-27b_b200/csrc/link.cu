// Stage link kernels: the hidden state (and the sampled tokens) move between
// pipeline stages on different GPUs of one box through peer memory, as nodes
// of the stages' decode graphs, with no host involvement per token.
//
// Protocol per channel (one message in flight: the next message of a channel
// can only exist after the ring of stages has consumed the previous one):
//   sender   payload stores -> fence.sc.sys -> block barrier ->
//            st.release.sys seq = n + 1   (its local count n -> n + 1)
//   receiver spin ld.acquire.sys seq >= n + 1 (bounded by %globaltimer) ->
//            block barrier -> payload loads through L2 (ld.global.cg) ->
//            local count n -> n + 1
// A wait that runs past kWaitLimitNs records kStatusLinkTimeout and skips the
// copy; the host sees the status through dial_b200_device_status.
#include "common.cuh"
#include "link.h"

namespace dialb200 {
namespace {

constexpr int kLinkThreads = 256;

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kLinkThreads) link_recv_kernel(const uint8_t* inbox, int channel,
                                                                 size_t payload_off,
                                                                 uint64_t* count, uint32_t* dst,
                                                                 size_t n4, int* status) {
  pdl_launch_dependents();
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const uint64_t want = *count + 1;
    const uint64_t* seq = reinterpret_cast<const uint64_t*>(inbox) + channel;
    const unsigned long long t0 = global_ns();
    int good = 1;
    while (ld_acquire_sys(seq) < want) {
      if (global_ns() - t0 > kWaitLimitNs) {
        set_status(status, kStatusLinkTimeout);
        good = 0;
        break;
      }
      __nanosleep(64);
    }
    ok = good;
    if (good) *count = want;
  }
  __syncthreads();
  if (!ok) return;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(inbox + payload_off);
  for (size_t i = threadIdx.x; i < n4; i += kLinkThreads) dst[i] = __ldcg(src + i);
}

__global__ void __launch_bounds__(kLinkThreads) link_send_kernel(uint8_t* peer_inbox, int channel,
                                                                 size_t payload_off,
                                                                 uint64_t* count,
                                                                 const uint32_t* src, size_t n4) {
  pdl_launch_dependents();
  pdl_wait();  // the payload is the previous kernel's output
  uint32_t* dst = reinterpret_cast<uint32_t*>(peer_inbox + payload_off);
  for (size_t i = threadIdx.x; i < n4; i += kLinkThreads) dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t next = *count + 1;
    st_release_sys(reinterpret_cast<uint64_t*>(peer_inbox) + channel, next);
    *count = next;
  }
}

cudaLaunchConfig_t link_cfg(cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kLinkThreads);
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

cudaError_t link_recv_launch(const uint8_t* inbox, int channel, int max_rows, uint64_t* count,
                             void* dst, size_t bytes, int* status, cudaStream_t s) {
  if (!inbox || !count || !dst || bytes % 4 != 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  // the receive waits on another GPU, not on the previous kernel of this
  // stream: it is launched without programmatic overlap of its own start
  const cudaLaunchConfig_t cfg = link_cfg(s, false, attr);
  return cudaLaunchKernelEx(&cfg, link_recv_kernel, inbox, channel,
                            link_payload_off(channel, max_rows), count,
                            static_cast<uint32_t*>(dst), bytes / 4, status);
}

cudaError_t link_send_launch(uint8_t* peer_inbox, int channel, int max_rows, uint64_t* count,
                             const void* src, size_t bytes, int* status, cudaStream_t s,
                             bool pdl) {
  (void)status;
  if (!peer_inbox || !count || !src || bytes % 4 != 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = link_cfg(s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, link_send_kernel, peer_inbox, channel,
                            link_payload_off(channel, max_rows), count,
                            static_cast<const uint32_t*>(src), bytes / 4);
}

}  // namespace dialb200
