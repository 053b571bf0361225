// Stable reverse index on the GPU: the counting sort of Csc::from_csr_slices
// (src/sparse.rs:361-427) restated as a stable LSD radix sort of
// (column, edge index) pairs.  A stable sort keyed on the column alone puts
// each column's edges in edge-index order, which is the order the
// reference's row-by-row cursor walk produces, so the result is identical.
//
// Per 8-bit digit: a tile histogram (radix_hist_kernel), one exclusive scan
// of the digit-major histogram table with a decoupled look-back
// (scan_excl_kernel), and a stable scatter (radix_scatter_kernel) that ranks
// each tile's keys with warp match masks.  Integer work, HBM-bound.
#include <algorithm>

#include "common.cuh"
#include "csc.cuh"

namespace sparsl {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 16;
constexpr int kTile = kThreads * kItems;  // keys per tile
constexpr int kRadix = 256;

uint64_t tiles_of(uint64_t n) { return std::max<uint64_t>(1, (n + kTile - 1) / kTile); }
size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

struct Carve {
  uint32_t* keys[2];
  uint32_t* vals[2];
  uint32_t* hist;
  unsigned long long* flags;
  uint32_t* ticket;
  uint64_t tiles, hist_n, scan_tiles;
};

Carve carve(void* base, uint64_t nnz) {
  Carve c{};
  char* p = static_cast<char*>(base);
  const size_t kb = align256(nnz * 4 + 16);
  for (int i = 0; i < 2; ++i) {
    c.keys[i] = reinterpret_cast<uint32_t*>(p);
    p += kb;
    c.vals[i] = reinterpret_cast<uint32_t*>(p);
    p += kb;
  }
  c.tiles = tiles_of(nnz);
  c.hist_n = c.tiles * kRadix;
  c.scan_tiles = tiles_of(c.hist_n);
  c.hist = reinterpret_cast<uint32_t*>(p);
  p += align256(c.hist_n * 4);
  c.flags = reinterpret_cast<unsigned long long*>(p);
  p += align256((c.scan_tiles + 1) * 8);
  c.ticket = reinterpret_cast<uint32_t*>(p);
  return c;
}

// hist[d * tiles + t] = number of keys of tile t whose digit is d.
__global__ void __launch_bounds__(kThreads) radix_hist_kernel(const uint32_t* __restrict__ keys, uint64_t n,
                                                              int shift, uint32_t* __restrict__ hist,
                                                              uint64_t tiles) {
  __shared__ uint32_t h[kRadix];
  h[threadIdx.x] = 0;
  __syncthreads();
  const uint64_t base = (uint64_t)blockIdx.x * kTile;
#pragma unroll 4
  for (int j = 0; j < kItems; ++j) {
    const uint64_t i = base + (uint64_t)j * kThreads + threadIdx.x;
    if (i < n) atomicAdd(&h[(__ldg(keys + i) >> shift) & (kRadix - 1)], 1u);
  }
  __syncthreads();
  hist[(uint64_t)threadIdx.x * tiles + blockIdx.x] = h[threadIdx.x];
}

// In-place exclusive prefix sum of n u32 values (the totals fit in u32: they
// count edges).  Tiles take ids from a ticket, so every predecessor a tile
// waits on is already running.
__global__ void __launch_bounds__(kThreads) scan_excl_kernel(uint32_t* data, uint64_t n,
                                                             unsigned long long* flags, uint32_t* ticket,
                                                             uint32_t* err) {
  __shared__ uint32_t s_tile, s_excl, s_warp[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1u);
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint64_t base = (uint64_t)tile * kTile + (uint64_t)threadIdx.x * kItems;
  uint32_t v[kItems];
  uint32_t t = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    v[j] = base + j < n ? data[base + j] : 0u;
    t += v[j];
  }
  uint32_t incl = t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c = s_warp[w];
      s_warp[w] = run;
      run += c;
    }
    s_excl = lookback_count(flags, tile, run, err);
  }
  __syncthreads();
  uint32_t run = s_excl + s_warp[warp] + incl - t;
#pragma unroll
  for (int j = 0; j < kItems; ++j)
    if (base + j < n) {
      data[base + j] = run;
      run += v[j];
    }
}

// Stable scatter of one digit pass.  Tile order is warp-major, then round,
// then lane; each key's rank counts the earlier keys of its digit in that
// order (warp match masks within a round, per-warp counters across rounds,
// an exclusive prefix over warps, then the tile's global digit offset).
template <bool kFirst>
__global__ void __launch_bounds__(kThreads) radix_scatter_kernel(const uint32_t* __restrict__ keys_in,
                                                                 const uint32_t* __restrict__ vals_in, uint64_t n,
                                                                 int shift, const uint32_t* __restrict__ offs,
                                                                 uint64_t tiles, uint32_t* __restrict__ keys_out,
                                                                 uint32_t* __restrict__ vals_out) {
  __shared__ uint32_t cnt[kWarps][kRadix];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < kWarps * kRadix; k += kThreads) cnt[k / kRadix][k % kRadix] = 0;
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  const uint64_t base = (uint64_t)blockIdx.x * kTile + (uint64_t)warp * (kTile / kWarps);
  uint32_t key[kItems], val[kItems], rank[kItems];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const uint64_t i = base + (uint64_t)j * 32 + lane;
    const bool valid = i < n;
    key[j] = valid ? __ldg(keys_in + i) : 0u;
    val[j] = valid ? (kFirst ? (uint32_t)i : __ldg(vals_in + i)) : 0u;
    const uint32_t d = valid ? (key[j] >> shift) & (kRadix - 1) : (uint32_t)kRadix;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    rank[j] = valid ? cnt[warp][d] + __popc(peers & lt) : 0u;
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) cnt[warp][d] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {
    const int d = threadIdx.x;
    uint32_t run = __ldg(offs + (uint64_t)d * tiles + blockIdx.x);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c = cnt[w][d];
      cnt[w][d] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const uint64_t i = base + (uint64_t)j * 32 + lane;
    if (i < n) {
      const uint32_t pos = cnt[warp][(key[j] >> shift) & (kRadix - 1)] + rank[j];
      keys_out[pos] = key[j];
      vals_out[pos] = val[j];
    }
  }
}

// col_ptr[c] = first slot whose column is >= c (sorted keys); row[k] = the
// CSR row holding edge edge_idx[k] (the last r with row_ptr[r] <= e).
__global__ void col_ptr_kernel(const uint32_t* __restrict__ keys, uint64_t nnz, uint64_t ncols,
                               uint32_t* __restrict__ col_ptr) {
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c <= ncols;
       c += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const uint64_t mid = (lo + hi) >> 1;
      if ((uint64_t)__ldg(keys + mid) < c)
        lo = mid + 1;
      else
        hi = mid;
    }
    col_ptr[c] = (uint32_t)lo;
  }
}

__global__ void row_of_edge_kernel(const uint32_t* __restrict__ row_ptr, uint64_t nrows,
                                   const uint32_t* __restrict__ edge_idx, uint64_t nnz, uint32_t* __restrict__ row) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nnz; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = __ldg(edge_idx + k);
    uint64_t lo = 0, hi = nrows;  // row_ptr[lo] <= e < row_ptr[hi]
    while (hi - lo > 1) {
      const uint64_t mid = (lo + hi) >> 1;
      if (__ldg(row_ptr + mid) <= e)
        lo = mid;
      else
        hi = mid;
    }
    row[k] = (uint32_t)lo;
  }
}

__global__ void slice_depth_kernel(const uint32_t* __restrict__ col_ptr, uint64_t ncols, uint32_t* __restrict__ depth) {
  const uint64_t nslices = (ncols + 31) / 32;
  for (uint64_t sl = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; sl < nslices;
       sl += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t d = 0;
    const uint64_t end = sl * 32 + 32 < ncols ? sl * 32 + 32 : ncols;
    for (uint64_t c = sl * 32; c < end; ++c) d = max(d, __ldg(col_ptr + c + 1) - __ldg(col_ptr + c));
    depth[sl] = d;
  }
}

__global__ void sell_fill_kernel(const uint32_t* __restrict__ col_ptr, const uint32_t* __restrict__ keys,
                                 const uint32_t* __restrict__ row, const uint32_t* __restrict__ edge_idx, uint64_t nnz,
                                 const unsigned long long* __restrict__ slice_ptr, uint32_t* __restrict__ sell_row,
                                 uint32_t* __restrict__ sell_eidx) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nnz; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = __ldg(keys + k);
    const uint64_t pos = __ldg(slice_ptr + (c >> 5)) + (c & 31) + (uint64_t)(k - __ldg(col_ptr + c)) * 32;
    sell_row[pos] = __ldg(row + k);
    sell_eidx[pos] = __ldg(edge_idx + k);
  }
}

unsigned grid_for(uint64_t items, unsigned block) {
  const uint64_t g = (items + block - 1) / block;
  return (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(g, 148ull * 16));
}

}  // namespace

size_t csc_scratch_bytes(uint64_t nnz) {
  const uint64_t tiles = tiles_of(nnz), hist_n = tiles * kRadix, scan_tiles = tiles_of(hist_n);
  return 4 * align256(nnz * 4 + 16) + align256(hist_n * 4) + align256((scan_tiles + 1) * 8) + 256;
}

cudaError_t csc_build(const uint32_t* row_ptr, uint64_t nrows, const uint32_t* col, uint64_t nnz, uint64_t ncols,
                      uint32_t* col_ptr, uint32_t* row, uint32_t* edge_idx, uint32_t* keys_out, void* scratch,
                      uint32_t* err, cudaStream_t s) {
  cudaError_t e;
  if (nnz == 0) {
    col_ptr_kernel<<<grid_for(ncols + 1, 256), 256, 0, s>>>(col, 0, ncols, col_ptr);
    return cudaGetLastError();
  }
  const Carve c = carve(scratch, nnz);
  int bits = 0;
  while (bits < 32 && (ncols - 1) >> bits) ++bits;
  const int passes = std::max(1, (bits + 7) / 8);
  const uint32_t* kin = col;
  const uint32_t* vin = nullptr;
  uint32_t* kout = nullptr;
  for (int p = 0; p < passes; ++p) {
    const bool last = p == passes - 1;
    kout = last && keys_out ? keys_out : c.keys[p & 1];
    uint32_t* vout = last ? edge_idx : c.vals[p & 1];
    radix_hist_kernel<<<(unsigned)c.tiles, kThreads, 0, s>>>(kin, nnz, 8 * p, c.hist, c.tiles);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(c.flags, 0, (c.scan_tiles + 1) * 8, s)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(c.ticket, 0, 4, s)) != cudaSuccess) return e;
    scan_excl_kernel<<<(unsigned)c.scan_tiles, kThreads, 0, s>>>(c.hist, c.hist_n, c.flags, c.ticket, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (p == 0)
      radix_scatter_kernel<true><<<(unsigned)c.tiles, kThreads, 0, s>>>(kin, nullptr, nnz, 0, c.hist, c.tiles, kout,
                                                                        vout);
    else
      radix_scatter_kernel<false><<<(unsigned)c.tiles, kThreads, 0, s>>>(kin, vin, nnz, 8 * p, c.hist, c.tiles,
                                                                         kout, vout);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    kin = kout;
    vin = vout;
  }
  col_ptr_kernel<<<grid_for(ncols + 1, 256), 256, 0, s>>>(kout, nnz, ncols, col_ptr);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  row_of_edge_kernel<<<grid_for(nnz, 256), 256, 0, s>>>(row_ptr, nrows, edge_idx, nnz, row);
  return cudaGetLastError();
}

cudaError_t launch_slice_depth(const uint32_t* col_ptr, uint64_t ncols, uint32_t* depth, cudaStream_t s) {
  const uint64_t nslices = (ncols + 31) / 32;
  if (nslices == 0) return cudaSuccess;
  slice_depth_kernel<<<grid_for(nslices, 256), 256, 0, s>>>(col_ptr, ncols, depth);
  return cudaGetLastError();
}

cudaError_t launch_sell_fill(const uint32_t* col_ptr, const uint32_t* keys, const uint32_t* row,
                             const uint32_t* edge_idx, uint64_t nnz, const unsigned long long* slice_ptr,
                             uint32_t* sell_row, uint32_t* sell_eidx, cudaStream_t s) {
  if (nnz == 0) return cudaSuccess;
  sell_fill_kernel<<<grid_for(nnz, 256), 256, 0, s>>>(col_ptr, keys, row, edge_idx, nnz, slice_ptr, sell_row,
                                                      sell_eidx);
  return cudaGetLastError();
}

}  // namespace sparsl
