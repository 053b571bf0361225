// Stable reverse index (CSC) built on the GPU (csc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// Device scratch for csc_build, in bytes, for `nnz` edges.
size_t csc_scratch_bytes(uint64_t nnz);

// Csc::from_csr_slices (src/sparse.rs:361-427) for a validated CSR in device
// memory: col_ptr[ncols + 1], and for each slot of column c, in CSR order,
// the edge's row and its index into col / weights.  The order within a
// column is the stable counting sort's: by edge index.  Computed as a stable
// LSD radix sort of (column, edge) pairs, 8 bits per pass, followed by a pass
// that derives col_ptr and the rows.  `keys_out`, if not null, receives the
// column of every slot (nnz entries).  `scratch` holds csc_scratch_bytes(nnz)
// bytes; `err` is the device error word (a look-back that gave up sets
// DEVERR_LOOKBACK_TIMEOUT).  Requires nnz, nrows, ncols < 2^32.
cudaError_t csc_build(const uint32_t* row_ptr, uint64_t nrows, const uint32_t* col, uint64_t nnz, uint64_t ncols,
                      uint32_t* col_ptr, uint32_t* row, uint32_t* edge_idx, uint32_t* keys_out, void* scratch,
                      uint32_t* err, cudaStream_t s);

// Sliced-ELL layout from a CSC: the depth (longest column) of each slice of
// 32 columns.
cudaError_t launch_slice_depth(const uint32_t* col_ptr, uint64_t ncols, uint32_t* depth, cudaStream_t s);

// Places CSC slot k of column c at slice_ptr[c / 32] + c % 32 + (k - col_ptr[c]) * 32
// (rows and edge indices); padding slots must already be zero.
cudaError_t launch_sell_fill(const uint32_t* col_ptr, const uint32_t* keys, const uint32_t* row,
                             const uint32_t* edge_idx, uint64_t nnz, const unsigned long long* slice_ptr,
                             uint32_t* sell_row, uint32_t* sell_eidx, cudaStream_t s);

}  // namespace sparsl
