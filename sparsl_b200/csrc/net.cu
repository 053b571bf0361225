// Spike-vector exchange of the multi-GPU network tick, over peer memory.
//
// Every rank holds the whole spike vector (two ping-pong copies) and computes
// the words of its own rows.  On the TMA path the tick kernel itself stores
// each packed word into every peer's copy as it is produced (ell.cu), so the
// NVLink transfer overlaps the streaming fold; other engines leave the copy
// to this step.  What remains after the tick is one small kernel per rank:
//
//   1. (push) copy this rank's slice into every peer's copy;
//   2. publish: store this rank's spike count into each peer's mailbox, then
//      -- after a system-scope fence that orders every earlier store to that
//      peer, the tick kernels' included -- the tick number into its flag;
//   3. wait until every peer's flag for this tick has arrived (bounded by
//      %globaltimer: on expiry the device error word records it and the step
//      returns instead of hanging);
//   4. the tick's global spike count = this rank's count + the peers' counts.
//
// Ping-pong safety: tick t + 1 writes the copy that tick t - 1 read.  A rank
// starts tick t + 1 only after every peer's flag for tick t, i.e. after every
// peer has finished tick t (and so tick t - 1), so no word is overwritten
// while a peer can still read it.
#include "common.cuh"
#include "net.cuh"

namespace sparsl {
namespace {

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kXchgThreads = 1024;

__global__ void __launch_bounds__(kXchgThreads) net_exchange_kernel(const NetExchange x) {
  __shared__ uint32_t s_warp[kXchgThreads / 32];
  __shared__ uint32_t s_peer[kNetMaxRanks];
  const uint32_t t = threadIdx.x;
  // 1. push this rank's slice to the peers (16-byte stores when aligned)
  if (x.push) {
    const bool vec = (x.nwords % 4 == 0) && ((uintptr_t)x.local_words % 16 == 0);
    for (uint32_t r = 0; r < x.nranks; ++r) {
      uint32_t* q = x.peer_words[r];
      if (!q) continue;
      if (vec && (uintptr_t)q % 16 == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(x.local_words);
        uint4* dst = reinterpret_cast<uint4*>(q);
        for (uint32_t i = t; i < x.nwords / 4; i += blockDim.x) dst[i] = src[i];
      } else {
        for (uint32_t i = t; i < x.nwords; i += blockDim.x) q[i] = x.local_words[i];
      }
    }
    __threadfence_system();
  }
  // 2. this rank's spike count for the tick
  uint32_t c = 0;
  if (x.count) {
    if (t == 0) c = *x.count;
  } else {
    for (uint32_t i = t; i < x.nwords; i += blockDim.x) c += __popc(x.local_words[i]);
  }
  c = __reduce_add_sync(0xffffffffu, c);
  if ((t & 31) == 0) s_warp[t >> 5] = c;
  __syncthreads();
  uint32_t mine = 0;
  for (int w = 0; w < kXchgThreads / 32; ++w) mine += s_warp[w];
  const uint32_t slot = x.tick % kNetSlots;
  const uint32_t want = x.tick + 1;
  // 3. publish to every peer, then wait for every peer (not again once a
  //    wait of this call has expired: the call fails fast)
  const bool failed = (*reinterpret_cast<volatile uint32_t*>(x.err) & DEVERR_PEER_TIMEOUT) != 0;
  if (t < x.nranks && t != x.self) {
    NetMailbox* pb = x.peer_box[t];
    st_relaxed_sys(&pb->count[slot][x.self], mine);
    __threadfence_system();
    st_release_sys(&pb->flag[x.self], want);
    const uint64_t t0 = globaltimer();
    bool ok = !failed;
    while (ok && (int32_t)(ld_acquire_sys(&x.my_box->flag[t]) - want) < 0) {
      if (globaltimer() - t0 > x.wait_ns) {
        ok = false;
        break;
      }
      __nanosleep(256);
    }
    if (!ok && !failed) set_err(x.err, DEVERR_PEER_TIMEOUT);
    s_peer[t] = ok ? ld_acquire_sys(&x.my_box->count[slot][t]) : 0u;
  }
  __syncthreads();
  // 4. the global count of the tick
  if (t == 0) {
    uint32_t total = mine;
    for (uint32_t r = 0; r < x.nranks; ++r)
      if (r != x.self) total += s_peer[r];
    *x.trace_slot = total;
    if (x.count) *x.count = 0;
  }
}

}  // namespace

cudaError_t launch_net_exchange(const NetExchange& x, cudaStream_t s) {
  net_exchange_kernel<<<1, kXchgThreads, 0, s>>>(x);
  return cudaGetLastError();
}

}  // namespace sparsl
