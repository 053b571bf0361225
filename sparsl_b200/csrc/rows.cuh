// Launch interface of the row-fold kernel family (rows.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// How the right-hand operand is read.
enum XMode : int {
  X_DENSE = 0,      // f32 vector, gathered through L1/L2
  X_BITS_SMEM = 1,  // LSB-first spike bitmask, copied to shared memory per block
  X_BITS_GLOBAL = 2 // spike bitmask too large for shared memory, read through L1/L2
};

// Per-line epilogue.
enum Epilogue : int {
  EPI_ACCUM = 0,  // y[l] = y[l] + fold
  EPI_LIF = 1     // LIF membrane step on the fold (src/backend/mod.rs:2461-2472)
};

// One launch of the row-fold engine.  A "line" is a CSR row (forward) or a
// CSC column (transpose); every line is folded left to right, from 0.0, by a
// single lane, so each output is bit-identical to the reference's sequential
// row_dot / col_dot (src/backend/mod.rs:2259-2288).
struct RowLaunch {
  const uint32_t* ptr = nullptr;   // nlines + 1 offsets
  const uint32_t* idx = nullptr;   // column (CSR) or row (CSC) per entry
  const uint32_t* eidx = nullptr;  // CSC: weight slot per entry; null for CSR
  const void* w = nullptr;         // weights: f32, or u16 binary16 / bfloat16 bits
  int wkind = 0;                   // WeightKind
  const float* x = nullptr;        // dense operand
  const uint32_t* xbits = nullptr; // spike operand
  uint32_t xbits_words = 0;
  uint32_t nlines = 0;
  // Optional line order (CSR rows by descending length, ties by index): warp
  // slot k folds line order[k], so the 32 lines of a warp have similar
  // lengths and no lane idles behind a long neighbour.  Packed spike words,
  // compaction and the transpose are not produced by ordered launches.
  const uint32_t* order = nullptr;
  int xmode = X_DENSE;
  int epilogue = EPI_ACCUM;
  float* y = nullptr;              // EPI_ACCUM output
  // EPI_LIF state
  float* v = nullptr;
  float* theta = nullptr;
  uint8_t* spikes = nullptr;
  // Optional state in pinned, mapped host memory (a tick that takes its
  // state from the host or returns it there): when set, v / theta are read
  // from v_src / theta_src instead, and the new values are written to
  // v_mirror / theta_mirror as well as to v / theta.
  const float* v_src = nullptr;
  const float* theta_src = nullptr;
  float* v_mirror = nullptr;
  float* theta_mirror = nullptr;
  uint32_t* out_bits = nullptr;    // optional packed spike words (word = line / 32)
  // Network ticks across GPUs (TMA path): each packed word is also stored
  // into every peer's copy of the spike vector (peer_out[r] is peer r's
  // words at the same offset as out_bits, null for this rank), the spikes
  // are counted into *tick_count, and every warp that stored to a peer
  // fences those stores system-wide before it exits.
  uint32_t* const* peer_out = nullptr;
  uint32_t npeers = 0;
  uint32_t* tick_count = nullptr;
  float decay = 0.f, v_reset = 0.f, dtheta = 0.f;
  // Optional spike compaction (requires EPI_LIF): ascending index list.
  uint32_t* idx_list = nullptr;
  uint32_t* idx_count = nullptr;   // total spikes written here by the last tile
  uint32_t idx_base = 0;           // added to every emitted line index
  unsigned long long* tile_flags = nullptr;  // >= tiles(nlines), zero on entry
  uint32_t* tile_ticket = nullptr;           // 2 words, zero on entry
  uint32_t epoch = 0;              // TMA path: tag of this launch's compaction flags
  uint32_t* err = nullptr;         // device error word (host mapped)
};

constexpr int kRowWarps = 8;                 // warps per block
constexpr int kRowLines = kRowWarps * 32;    // lines per block (one tile)

__host__ __device__ inline uint32_t row_tiles(uint32_t nlines) { return (nlines + kRowLines - 1) / kRowLines; }

cudaError_t launch_rows(const RowLaunch& p, cudaStream_t stream);

// Largest bitmask (in 32-bit words) staged in shared memory per block.
constexpr uint32_t kBitsSmemMaxWords = 16384;  // 64 KiB = 524,288 columns

}  // namespace sparsl
