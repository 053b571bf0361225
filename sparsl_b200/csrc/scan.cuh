// Launch interface of the exact affine-map scan (scan.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// Sub-chunks of 32 maps with a 160-map warm-up replay (the replay is
// amortised over 32 maps of output).
#ifndef SPARSL_SCAN_K
#define SPARSL_SCAN_K 32
#endif
#ifndef SPARSL_SCAN_WARM_SUB
#define SPARSL_SCAN_WARM_SUB 5
#endif
constexpr int kScanThreads = 256;  // sub-chunk threads per tile (8 warps)
constexpr int kScanBlock = kScanThreads + 32;  // plus one look-back warp
constexpr int kScanK = SPARSL_SCAN_K;  // elements per thread (one sub-chunk)
constexpr int kScanTile = kScanThreads * kScanK;
constexpr int kScanWarmSub = SPARSL_SCAN_WARM_SUB;  // warm-up of an in-tile guess, in sub-chunks
#ifndef SPARSL_SCAN_HALO_SUB
#define SPARSL_SCAN_HALO_SUB 16
#endif
// Rows of the previous tile staged with a tile for its first warp's warm-up,
// in sub-chunks (the look-back warp composes the 32 - kScanHaloSub before
// them from global memory).
constexpr int kScanHaloSub = SPARSL_SCAN_HALO_SUB;
static_assert(kScanHaloSub >= 1 && kScanHaloSub <= 32, "halo rows (one per lane of warp 0)");
#ifndef SPARSL_SCAN_T0_SUB
#define SPARSL_SCAN_T0_SUB 10
#endif
// Warm-up of a tile's thread 0, in sub-chunks (less than the halo): a miss
// there is only caught by the cross-tile check and repaired serially.
constexpr int kScanT0Sub = SPARSL_SCAN_T0_SUB;
static_assert(kScanT0Sub >= kScanWarmSub && kScanT0Sub < kScanHaloSub, "thread 0 warm-up");
constexpr int kScanHalo = kScanHaloSub * kScanK;
// Maps per chunk of the pipelined host-buffer scan (32 MiB each way).
constexpr uint64_t kScanPipeChunk = 1ull << 22;

// Scratch the scan needs, sized by scan_scratch_bytes(n).  All of it is
// left in its zero state (or self-resetting) after each call.
struct ScanScratch {
  unsigned long long* flags;  // ntiles look-back words: [33:32] status, [31:0] payload
  uint32_t* ticket;         // [0] tile ticket
  float* assumed;           // 2 * ntiles: thread 0's assumed incoming state
  float* last;              // 2 * ntiles: each tile's last output state
  uint32_t* mis_bits;       // ntiles * 8 words: in-tile sub-chunk mismatches
  uint32_t* xmis;           // ntiles: tile-boundary mismatch
  uint32_t* tile_bits;      // ceil(ntiles / 32) words: any mismatch in tile
  uint32_t* repair_stats;   // [0] repaired elements, [1] repair segments
  unsigned long long* timeline = nullptr;  // optional: 16 words per tile (phase stamps, counters)
};

size_t scan_scratch_bytes(uint64_t n);
ScanScratch scan_scratch_carve(void* base, uint64_t n);

// out[i] = in[0] o in[1] o ... o in[i] as an exact sequential left fold
// (src/scan.rs:298-313).  `in` and `out` hold n (a, b) pairs and must not
// alias.  scratch must be zeroed once before first use.
// `entry` (host pointer to an (a, b) pair, or null): the run continues a
// longer sequence whose state before in[0] is *entry, so out[0] is
// entry o in[0] rather than a copy of in[0].
cudaError_t launch_scan(const float* in, float* out, uint64_t n, const ScanScratch& s,
                        uint32_t* err, cudaStream_t stream, const float* entry = nullptr,
                        const float* entry_dev = nullptr);

// Serial single-thread walks for runs split across devices (see scan.cu):
// fold in[0..n) into state[2] (device memory), or repair out[0..n) from an
// exact entry state until it rejoins the stored trajectory.
// repair: 0 = fold, 1 = rejoin, 2 = settle (the multiplier chain from a copy
// of in[0] until it is one of {0..7} * 2^-149; stats[0] = maps folded).
cudaError_t launch_scan_walk(const float* in, float* out, uint64_t n, const float* entry, int repair,
                             float* state, unsigned long long* stats, cudaStream_t stream);

// Transfer table of in[0..n) for the multiplier chain (nibble m: the
// multiplier leaving the run when m * 2^-149 entered it; 8 = outside that
// set), into *out (device).  blk_scratch holds nblk_max words.
cudaError_t launch_scan_table(const float* in, uint64_t n, uint32_t* blk_scratch, uint32_t nblk_max, uint32_t* out,
                              cudaStream_t stream, const unsigned long long* start = nullptr);

// A run's part of a split scan with no host round trip (see scan.cu):
// publish writes blob = [last `halo` maps, identity-padded | len, table,
// first run's exit multiplier, 0] (2*halo + 4 floats); entry reads every
// run's blob (gathered, in run order) and writes the run's guessed entry
// state (2 floats).  Scratch: tab_scratch (nblk_max + 1 words), walk_state
// (2 floats), walk_stats (1 word).
cudaError_t launch_scan_publish(const float* in, uint64_t n, int first, uint32_t halo, float* blob,
                                uint32_t* tab_scratch, uint32_t nblk_max, float* walk_state,
                                unsigned long long* walk_stats, cudaStream_t stream);
cudaError_t launch_scan_entry(const float* gathered, uint32_t world, uint32_t rank, uint32_t halo, float* entry,
                              cudaStream_t stream);

}  // namespace sparsl
