// Dense-x SpMV for operators with a uniform row length, with x staged in
// shared memory one column panel at a time (panel.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sparsl {

// A panel is at most 216 KiB of x (one CTA per SM holds it); an operator
// takes this path when x fits in kPanelMaxPanels of them and its rows have
// at most kPanelMaxRowLen entries.
constexpr uint32_t kPanelMaxFloats = 55296;
constexpr uint32_t kPanelMaxPanels = 4;
constexpr uint32_t kPanelMaxRowLen = 65535;

// Tile-interleaved copy of a uniform-length CSR operator, built at prepare.
// Rows go in tiles of 32 (one per lane of a warp); within a tile, entry
// positions go in groups of 16 bytes per lane, so a lane reads 8 columns or
// 16 bytes of weights with one load and a warp reads 512 contiguous bytes.
//   col16[((T * Lc + j / 8) * 32 + lane) * 8 + j % 8]      Lc = ceil(L / 8)
//     the column minus the start of its panel (below kPanelMaxFloats < 2^16)
//   w[((T * Lw + j / G) * 32 + lane) * G + j % G]            G = 16 / weight bytes,
//                                                            Lw = 8 * Lc / G
//   split[(T * (npanels + 1) + k) * 32 + lane]
//     the row's first entry in panel k (0 for k = 0, L for k = npanels)
// Rows past nrows in the last tile and positions past L are padding: their
// split points are all 0, so no pass folds them.
//
// The same layout serves lines of different lengths (the transpose product
// over the sliced-ELL reverse index: a line is a column, its entries are its
// rows in ascending order, x is indexed by row): tile T then holds
// toff[T + 1] - toff[T] groups of 8 positions (its longest line, padded), at
// group offset toff[T] instead of T * Lc.
struct PanelOp {
  const uint16_t* col16 = nullptr;
  const void* w = nullptr;    // f32, or binary16 / bfloat16 bits
  const uint16_t* split = nullptr;
  const uint64_t* toff = nullptr;  // ragged lines: 8-position groups before tile T
  int wkind = 0;              // WeightKind
  uint32_t nrows = 0, L = 0, ncols = 0;  // lines, uniform line length (0 when ragged), x length
  uint32_t width = 0;         // panel width in floats (a multiple of 4)
  uint32_t npanels = 0;
  bool ok = false;
};

// Panel geometry for ncols columns: false when x needs more than
// kPanelMaxPanels panels.
bool panel_geometry(uint64_t ncols, uint32_t& width, uint32_t& npanels);

// Elements of each interleaved array.
inline uint64_t panel_tiles(uint64_t nrows) { return (nrows + 31) / 32; }
inline uint64_t panel_col_elems(uint64_t nrows, uint32_t L) { return panel_tiles(nrows) * 32 * 8 * ((L + 7) / 8); }
// Positions are padded to a multiple of 8 in both arrays (one batch).
inline uint64_t panel_w_elems(uint64_t nrows, uint32_t L) { return panel_tiles(nrows) * 32 * 8 * ((L + 7) / 8); }
inline uint64_t panel_split_elems(uint64_t nrows, uint32_t npanels) { return panel_tiles(nrows) * 32 * (npanels + 1); }

// Builds col16 and split from the row-major [nrows x L] column array.
cudaError_t launch_panel_build(const uint32_t* col, uint64_t nrows, uint32_t L, uint32_t width, uint32_t npanels,
                               uint16_t* col16, uint16_t* split, cudaStream_t stream);
// Interleaves the row-major [nrows x L] weights (esize bytes each: 4 or 2).
cudaError_t launch_panel_weights(const void* w, uint64_t nrows, uint32_t L, int esize, void* out,
                                 cudaStream_t stream);

// The same copy of a sliced-ELL operator (slices of 32 lines; entry j of
// line 32 * T + l at slice_ptr[T] + 32 * j + l; line lengths from line_ptr;
// the entries' gathered index, here a row, ascending within a line): col16
// and split from the rows, and (separately, for new weights) the weights
// from the sliced-ELL weight array.  toff holds nslices + 1 group offsets.
cudaError_t launch_panel_build_sell(const unsigned long long* slice_ptr, const uint32_t* line_ptr,
                                    const uint32_t* sell_idx, uint64_t nlines, uint32_t nslices, const uint64_t* toff,
                                    uint32_t width, uint32_t npanels, uint16_t* col16, uint16_t* split,
                                    cudaStream_t stream);
cudaError_t launch_panel_weights_sell(const unsigned long long* slice_ptr, const uint32_t* line_ptr,
                                      const void* w_sell, uint64_t nlines, uint32_t nslices, const uint64_t* toff,
                                      int esize, void* out, cudaStream_t stream);

// Skewed operators (rows of very different lengths): the rows in
// descending-length order.  The first nlong rows (kOrderedLongRow entries or
// more) are folded one warp per row straight from the CSR arrays, 32
// consecutive entries per load.  The rest are copied 32 per tile, each tile
// padded to its longest row (a multiple of 8 positions), with 32-bit
// columns, and folded one lane per row.
//   col[((toff[T] * 2 + j / 4) * 32 + lane) * 4 + j % 4]
//   w  as in the panel copy, with gbase = toff[T]
//   len[32 * T + lane]: the row's length; the row is order[nlong + 32 * T + lane]
#ifndef SPARSL_ORDERED_LONG_ROW
#define SPARSL_ORDERED_LONG_ROW 1024
#endif
constexpr uint32_t kOrderedLongRow = SPARSL_ORDERED_LONG_ROW;
struct OrderedOp {
  const uint32_t* col = nullptr;
  const void* w = nullptr;
  const uint32_t* len = nullptr;
  const uint64_t* toff = nullptr;     // 8-position groups before tile T
  const uint32_t* order = nullptr;    // all rows by descending length
  const uint32_t* row_ptr = nullptr;  // the CSR arrays, for the long rows
  const uint32_t* csr_col = nullptr;
  const void* csr_w = nullptr;
  int wkind = 0;
  uint32_t nrows = 0;  // all rows
  uint32_t nlong = 0;  // rows folded one warp each
  bool ok = false;
};

// Builds col, w and len from the CSR arrays (row_ptr, col, w of esize bytes)
// and the order; toff holds ntiles + 1 group offsets.
cudaError_t launch_ordered_build(const uint32_t* row_ptr, const uint32_t* col, const void* w, int esize,
                                 const uint32_t* order, uint64_t nrows, const uint64_t* toff, uint32_t* ocol,
                                 void* ow, uint32_t* olen, cudaStream_t stream);
// Rebuilds only the weights (new weights after prepare).
cudaError_t launch_ordered_weights(const uint32_t* row_ptr, const void* w, int esize, const uint32_t* order,
                                   uint64_t nrows, const uint64_t* toff, void* ow, cudaStream_t stream);
// y[r] = y[r] + fold_r over the ordered copy (same fold as below).
cudaError_t launch_ordered_spmv(const OrderedOp& op, const float* x, float* y, cudaStream_t stream);

// The same fold with a dense x or a spike bitmask (staged in shared memory,
// at most kOrderedBitsMaxBytes), then either y[r] = y[r] + fold_r (v null) or
// the LIF step on row r's v, theta and spike byte (src/backend/mod.rs:
// 2461-2472).  The spike bytes are the whole output: the caller packs them.
constexpr uint64_t kOrderedBitsMaxBytes = 200 * 1024;
// Optional LIF state in pinned, mapped host memory: read from v_src /
// theta_src instead of v / theta when set, and the new values written to
// v_mirror / theta_mirror too when set.
struct LifHostState {
  const float* v_src = nullptr;
  const float* theta_src = nullptr;
  float* v_mirror = nullptr;
  float* theta_mirror = nullptr;
};
cudaError_t launch_ordered_fold(const OrderedOp& op, const float* x, const uint32_t* xbits, uint32_t xbits_words,
                                float* y, float* v, float* theta, uint8_t* spikes, float decay, float v_reset,
                                float dtheta, cudaStream_t stream, const LifHostState& hs = LifHostState{});

// y[r] = y[r] + fold_r, fold_r the strict left fold from 0.0 of w * x over
// row r's entries in stored order (src/backend/mod.rs:2259-2267), for a
// dense x of op.ncols floats.  The columns of a row are non-decreasing, so
// its entries in panel k follow those in panel k - 1: panel by panel, a
// lane folds each entry of its row once, in order.
cudaError_t launch_panel_spmv(const PanelOp& op, const float* x, float* y, cudaStream_t stream);

}  // namespace sparsl
