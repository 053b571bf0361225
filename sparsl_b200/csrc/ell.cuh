// TMA-pipelined row-fold for operators with a uniform row length (ell.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rows.cuh"

namespace sparsl {

#ifndef SPARSL_ELL_WARPS
#define SPARSL_ELL_WARPS 12
#endif
constexpr int kEllWarps = SPARSL_ELL_WARPS;  // warps per persistent CTA

// Compaction tiles of the TMA path: one warp's 32 rows.
__host__ __device__ inline uint32_t ell_tiles(uint32_t nlines) { return (nlines + 31) / 32; }

// Two encoded CUtensorMaps (column and weight matrices viewed as [nrows x L]).
struct EllMaps {
  alignas(64) unsigned char idx[128];
  alignas(64) unsigned char w[128];
  uint32_t L = 0;
  bool ok = false;
};

// Builds the tensor maps; false when the shape or alignment does not allow
// 2-D TMA boxes (the caller keeps the generic row-fold path).
bool ell_encode(EllMaps& m, const uint32_t* col, const void* w, int wkind, uint64_t nrows, uint32_t L);

// Same contract as launch_rows for a forward (CSR) launch; p.ptr is unused
// and p.tile_ticket (two words, zero on entry, left zero) is required: tiles
// are handed out by ticket.  Launches sharing it must be stream-ordered.
// Compaction flags are tagged with p.epoch (nonzero, below 2^30, different
// from the previous launch's) instead of being cleared between launches.
cudaError_t launch_ell(const EllMaps& m, const RowLaunch& p, cudaStream_t stream);

}  // namespace sparsl
