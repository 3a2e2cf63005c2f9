// Host interface of the stage link kernels (link.cu): the in-box replacement
// of the Master -> Worker TCP hop between pipeline stages on different GPUs
// of one box (spm/client.rs:391-453 send, spm/worker.rs:740-796 receive),
// over peer memory instead of NCCL.
//
// Every stage owns an inbox in its own HBM, exported to the other stage
// processes by CUDA IPC.  Layout: kLinkHeader bytes of sequence words
// (word 0: hidden-state messages delivered, word 1: token messages delivered,
// each written last by the sender with a system-scope release), then the
// token payload (int32 [max_rows]) and the hidden payload (act [max_rows][H]).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dialb200 {

constexpr size_t kLinkHeader = 256;
enum LinkChannel : int { kLinkHidden = 0, kLinkTokens = 1 };

inline size_t link_tokens_off() { return kLinkHeader; }
inline size_t link_hidden_off(int max_rows) {
  return kLinkHeader + (static_cast<size_t>(max_rows) * 4 + 255) / 256 * 256;
}
inline size_t link_inbox_bytes(int max_rows, int H) {
  return link_hidden_off(max_rows) + static_cast<size_t>(max_rows) * H * 2;
}
inline size_t link_payload_off(int channel, int max_rows) {
  return channel == kLinkHidden ? link_hidden_off(max_rows) : link_tokens_off();
}

// Wait (bounded) until the local inbox's `channel` sequence word reaches
// *count + 1, copy `bytes` of its payload to dst, then *count += 1.  Launches
// its dependents at once (programmatic dependent launch), so the next kernel
// starts streaming its weights while this one waits.
cudaError_t link_recv_launch(const uint8_t* inbox, int channel, int max_rows, uint64_t* count,
                             void* dst, size_t bytes, int* status, cudaStream_t s);

// After the previous kernel completes: copy `bytes` from src into the peer
// inbox's `channel` payload with plain stores over NVLink, fence at system
// scope, then store *count + 1 into the peer's sequence word (release) and
// *count += 1.
cudaError_t link_send_launch(uint8_t* peer_inbox, int channel, int max_rows, uint64_t* count,
                             const void* src, size_t bytes, int* status, cudaStream_t s,
                             bool pdl);

}  // namespace dialb200
