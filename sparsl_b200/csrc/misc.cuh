// Launchers for SpMM, standalone LIF, packing, counting and canary checks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// Sentinel tail written after every device buffer a kernel writes, checked
// after each host-facing dispatch (the reference's Metal canaries,
// src/backend/metal.rs:321-344, use the same pattern and length).
constexpr uint32_t kCanaryBits = 0x7FA5C0DEu;
constexpr uint32_t kCanaryWords = 64;

struct CanarySet {
  static constexpr int kMax = 16;
  const uint32_t* ptr[kMax];
  int count = 0;
};

cudaError_t launch_spmm(const uint32_t* ptr, const uint32_t* idx, const void* w, int wkind, const float* x,
                        float* y, uint32_t nrows, uint32_t n_vec, int sm_count, cudaStream_t s);
cudaError_t launch_lif_integrate(float* v, float* theta, const float* cur, uint8_t* spk, uint64_t n,
                                 float decay, float v_reset, float dtheta, cudaStream_t s);
cudaError_t launch_pack(const uint8_t* spk, uint64_t n, uint32_t* out, uint64_t out_words, cudaStream_t s);
// Writes popcount(words) into *slot (zeroed first).
cudaError_t launch_popcount(const uint32_t* words, uint64_t nwords, uint32_t* slot, cudaStream_t s);
cudaError_t launch_canary_check(const CanarySet& set, uint32_t* err, cudaStream_t s);
cudaError_t launch_fill(uint32_t* p, uint64_t n, uint32_t v, cudaStream_t s);

}  // namespace sparsl
