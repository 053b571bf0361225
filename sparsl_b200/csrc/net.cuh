// The spike-vector exchange of the multi-GPU network tick (net.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

constexpr uint32_t kNetMaxRanks = 32;
constexpr uint32_t kNetSlots = 4;  // per-tick count slots (a peer is at most one tick ahead)

// One rank's exchange area, written by its peers over NVLink: peer r stores
// its spike count for tick t in count[t % kNetSlots][r], then t + 1 in flag[r].
struct NetMailbox {
  uint32_t flag[kNetMaxRanks];
  uint32_t count[kNetSlots][kNetMaxRanks];
};

// One exchange step after a tick (see net.cu).
struct NetExchange {
  uint32_t self = 0, nranks = 1;
  // This rank's slice of the new spike vector, and the same slice in every
  // peer's copy (null for this rank); copied here when `push` is set (the
  // tick kernels did not store to the peers themselves).
  const uint32_t* local_words = nullptr;
  uint32_t nwords = 0;
  uint32_t* const* peer_words = nullptr;
  bool push = false;
  // The tick kernels' count of this rank's spikes (read, then reset to 0),
  // or null: the step counts the slice itself.
  uint32_t* count = nullptr;
  NetMailbox* const* peer_box = nullptr;  // [nranks], null for this rank
  NetMailbox* my_box = nullptr;
  uint32_t tick = 0;
  uint64_t wait_ns = 0;  // bound of the wait for the peers (skipped once one expired)
  uint32_t* trace_slot = nullptr;
  uint32_t* err = nullptr;
};

cudaError_t launch_net_exchange(const NetExchange& x, cudaStream_t s);

}  // namespace sparsl
