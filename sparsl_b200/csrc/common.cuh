// Shared device helpers for the sparsl CUDA library (sm_100a).
//
// Every floating-point step on the hot path is an explicit round-to-nearest
// multiply or add (__fmul_rn / __fadd_rn): the reference's CPU fold never
// contracts `a * b + c` into an FMA (src/backend/mod.rs:2259-2267), and the
// library is also compiled with -fmad=false and without FTZ so subnormals
// survive (tests/stress.rs:366-384).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SPARSL_WARP 32

namespace sparsl {

// Device error word bits, written to host-mapped memory so the host reads
// them after completion without a copy.
enum DevErr : uint32_t {
  DEVERR_LOOKBACK_TIMEOUT = 1u << 0,  // a bounded look-back spin gave up
  DEVERR_CANARY = 1u << 1,            // a canary tail was overwritten
  DEVERR_REPAIR_LIMIT = 1u << 2,      // scan repair hit its iteration cap
  DEVERR_PEER_TIMEOUT = 1u << 3,      // a peer GPU's tick did not arrive in time
};

// Iteration cap for every device-side spin.  At ~100 ns per poll this bounds a
// wait at well under a second; a wait that runs out records DEVERR_* and
// returns instead of hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }

// binary16 bits -> f32 by the hardware conversion (cvt.f32.f16, no flush):
// every binary16 value, subnormals included, is an f32 value, so for every
// non-NaN pattern the result is the one half.rs:49-90 constructs bit for bit.
// A NaN stays a NaN (its payload may differ, which the parity rule allows).
__device__ __forceinline__ float widen_f16(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// bfloat16 bits -> f32: the top half of an f32 (src/half.rs:187-189).
__device__ __forceinline__ float widen_bf16(uint32_t h) { return __uint_as_float(h << 16); }

// Weight element types.
enum WeightKind : int { W_F32 = 0, W_F16 = 1, W_BF16 = 2 };

template <int WK>
__device__ __forceinline__ float load_weight(const void* w, uint64_t i) {
  if constexpr (WK == W_F32) {
    return __ldg(reinterpret_cast<const float*>(w) + i);
  } else if constexpr (WK == W_F16) {
    return widen_f16(__ldg(reinterpret_cast<const unsigned short*>(w) + i));
  } else {
    return widen_bf16(__ldg(reinterpret_cast<const unsigned short*>(w) + i));
  }
}

__device__ __forceinline__ void set_err(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

// Relaxed-but-coherent 64-bit flag access for decoupled look-back.
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Relaxed coherent 64-bit flag access, for look-backs whose flag words carry
// all the data they publish (no other memory is ordered by them).
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Decoupled look-back over integer tile counts (exact, so the result is the
// same whichever predecessors are summed).  Run by one thread per tile.
__device__ inline uint32_t lookback_count(unsigned long long* flags, uint32_t tile, uint32_t agg,
                                   uint32_t* err) {
  if (tile == 0) {
    st_release_u64(flags, (2ull << 32) | agg);
    return 0;
  }
  st_release_u64(flags + tile, (1ull << 32) | agg);
  uint32_t excl = 0;
  int64_t j = (int64_t)tile - 1;
  uint32_t spins = 0;
  while (j >= 0) {
    unsigned long long f = ld_acquire_u64(flags + j);
    uint32_t st = (uint32_t)(f >> 32);
    if (st == 0) {
      if (++spins > kSpinLimit) {
        set_err(err, DEVERR_LOOKBACK_TIMEOUT);
        break;
      }
      __nanosleep(64);
      continue;
    }
    excl += (uint32_t)f;
    if (st == 2) break;
    --j;
  }
  st_release_u64(flags + tile, (2ull << 32) | (excl + agg));
  return excl;
}

}  // namespace sparsl
