// Sliced-ELL fold for the transpose product (sell.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// The reverse index (CSC) in slices of 32 consecutive lines (columns of the
// operator).  Slice s holds its lines' entries column-major: entry k of line
// 32s + l sits at slice_ptr[s] + 32k + l, for k below the slice's longest
// line; shorter lines are padded (row 0, never added).
struct SellLaunch {
  const uint64_t* slice_ptr = nullptr;  // nslices + 1 entry offsets
  const uint32_t* line_ptr = nullptr;   // nlines + 1: the CSC col_ptr (line lengths)
  const uint32_t* idx = nullptr;        // row index per entry
  const void* w = nullptr;              // weights per entry (f32 or u16 bits)
  int wkind = 0;
  const float* x = nullptr;             // length nrows
  float* y = nullptr;                   // length nlines
  uint32_t nlines = 0, nslices = 0;
  uint32_t* ctr = nullptr;              // 2 words, zero on entry and left zero
};

// y[l] = y[l] + (((0 + w0 x[r0]) + w1 x[r1]) + ...) over line l's entries in
// order, one lane per line: the reference's col_dot (src/backend/mod.rs:2277-2304).
cudaError_t launch_sell(const SellLaunch& p, int sm_count, cudaStream_t s);

}  // namespace sparsl
