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

// One SpMM launch, Y += A X (batch-minor X[ncols][n_vec], Y[nrows][n_vec]).
// Rows are handed out in work units: unit u covers positions
// [unit_start[u], unit_start[u+1]) of `order` (rows by descending length, so
// the long rows start first and the short ones fill the tail), or, with no
// order, the natural rows [u*rows_per_unit, ...).  `ctr` is two words, zero
// on entry and left zero; launches sharing it must be stream-ordered.
struct SpmmLaunch {
  const uint32_t* ptr = nullptr;
  const uint32_t* idx = nullptr;
  const void* w = nullptr;
  int wkind = 0;
  const float* x = nullptr;
  float* y = nullptr;
  uint32_t nrows = 0, n_vec = 0;
  const uint32_t* order = nullptr;       // nrows entries, or null
  const uint32_t* unit_start = nullptr;  // nunits + 1 entries when order is set
  uint32_t nunits = 0, rows_per_unit = 1;
  uint32_t* ctr = nullptr;
  uint32_t unit_base = 0;  // the launch takes units [unit_base, unit_base + nunits)
};

// Work units over rows sorted by descending length: each unit holds at least
// kSpmmUnitNnz entries or is a single row, and at most kSpmmUnitRows rows.
constexpr uint32_t kSpmmUnitNnz = 512, kSpmmUnitRows = 256;
// Row ranges of the host-buffer SpMM pipeline: operators of at least
// kSpmmRangeMinRows rows also get work units per range of consecutive rows,
// so range k's Y rows can be copied in, folded and copied out while the
// next range's rows are copied in.
constexpr uint32_t kSpmmRanges = 8, kSpmmRangeMinRows = 1u << 16;

cudaError_t launch_spmm(const SpmmLaunch& p, int sm_count, cudaStream_t s);
cudaError_t launch_lif_integrate(float* v, float* theta, const float* cur, uint8_t* spk, uint64_t n,
                                 float decay, float v_reset, float dtheta, cudaStream_t s);
cudaError_t launch_pack(const uint8_t* spk, uint64_t n, uint32_t* out, uint64_t out_words, cudaStream_t s);
// idx[0..) = idx_base + the ascending positions of the set bits of words
// (bit b of word w is position 32w + b); *count = their number.
cudaError_t launch_compact_bits(const uint32_t* words, uint64_t nwords, uint32_t* idx, uint32_t* count,
                                uint32_t idx_base, cudaStream_t s);
// Writes popcount(words) into *slot (zeroed first).
cudaError_t launch_popcount(const uint32_t* words, uint64_t nwords, uint32_t* slot, cudaStream_t s);
cudaError_t launch_canary_check(const CanarySet& set, uint32_t* err, cudaStream_t s);
cudaError_t launch_fill(uint32_t* p, uint64_t n, uint32_t v, cudaStream_t s);
// A look-back over a predecessor that never publishes, in 32 zeroed bytes of
// `scratch32`: the bounded wait expires and sets DEVERR_LOOKBACK_TIMEOUT in
// *err (failure-detection tests).
cudaError_t launch_expired_wait(void* scratch32, uint32_t* err, cudaStream_t s);
// out[k] = w[idx[k]] for k < n, elements of `wbytes` (4 or 2) bytes.
cudaError_t launch_gather_weights(const void* w, const uint32_t* idx, uint64_t n, int wbytes, void* out,
                                  cudaStream_t s);

}  // namespace sparsl
