// Device-side CSR gate: the O(nnz) checks of validate_csr on the GPU, so an
// operator whose arrays already live in device memory is validated without
// copying them to the host.  Integer work only; each check reports its first
// failing index (an atomic minimum), exactly as the host gate does.
#include <algorithm>
#include <vector>

#include "codec.cuh"
#include "common.cuh"
#include "validate.cuh"

namespace sparsl {
namespace {

constexpr unsigned long long kNone = ~0ull;

// First e with col[e] >= ncols.
__global__ void col_range_kernel(const uint32_t* __restrict__ col, uint64_t n, uint64_t ncols,
                                 unsigned long long* first) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n; e += (uint64_t)gridDim.x * blockDim.x)
    if ((uint64_t)__ldg(col + e) >= ncols) {
      atomicMin(first, (unsigned long long)e);
      return;
    }
}

// First row whose columns decrease somewhere, and (in a second word) the
// first decreasing edge of the rows found: a warp per row, 32 edges at once.
__global__ void unsorted_rows_kernel(const uint32_t* __restrict__ row_ptr, uint64_t nrows,
                                     const uint32_t* __restrict__ col, unsigned long long* first_row) {
  const int lane = threadIdx.x & 31;
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t r = warp; r < nrows; r += nwarps) {
    const uint64_t b = __ldg(row_ptr + r), e = __ldg(row_ptr + r + 1);
    for (uint64_t k0 = b + 1; k0 < e; k0 += 32) {
      const uint64_t k = k0 + lane;
      const bool bad = k < e && __ldg(col + k) < __ldg(col + k - 1);
      if (__ballot_sync(0xffffffffu, bad)) {
        if (lane == 0) atomicMin(first_row, (unsigned long long)r);
        break;
      }
    }
  }
}

__global__ void encode_kernel(int precision, const float* __restrict__ in, uint16_t* __restrict__ out,
                              uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = precision == 1 ? encode_f16(__ldg(in + i)) : encode_bf16(__ldg(in + i));
}

unsigned grid_of(uint64_t items, unsigned block) {
  const uint64_t g = (items + block - 1) / block;
  return (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(g, 148ull * 32));
}

}  // namespace

cudaError_t validate_csr_device(const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* d_row_ptr,
                                const uint32_t* d_col, uint64_t col_len, uint64_t csr_ncols, uint64_t ncols,
                                unsigned long long* scratch, cudaStream_t s, PlanResult* out) {
  PlanResult r{};
  // The row_ptr checks, in order, on the host copy.
  if (row_ptr_len == 0) {
    r.code = PLAN_EMPTY_ROW_PTR;
    *out = r;
    return cudaSuccess;
  }
  if (row_ptr[0] != 0) {
    r.code = PLAN_NONZERO_START;
    r.a = row_ptr[0];
    *out = r;
    return cudaSuccess;
  }
  for (uint64_t i = 1; i < row_ptr_len; ++i)
    if (row_ptr[i] < row_ptr[i - 1]) {
      r.code = PLAN_NOT_MONOTONIC;
      r.a = i;
      *out = r;
      return cudaSuccess;
    }
  const uint32_t end = row_ptr[row_ptr_len - 1];
  if ((uint64_t)end != col_len) {
    r.code = PLAN_NNZ_MISMATCH;
    r.a = end;
    r.b = col_len;
    *out = r;
    return cudaSuccess;
  }
  if (csr_ncols != ncols) {
    r.code = PLAN_NCOLS_MISMATCH;
    r.a = csr_ncols;
    r.b = ncols;
    *out = r;
    return cudaSuccess;
  }
  const uint64_t nrows = row_ptr_len - 1;
  // The column checks on the GPU.
  unsigned long long h[2] = {kNone, kNone};
  cudaError_t e = cudaMemcpyAsync(scratch, h, sizeof h, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return e;
  if (col_len) {
    col_range_kernel<<<grid_of(col_len, 256), 256, 0, s>>>(d_col, col_len, ncols, scratch);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    unsorted_rows_kernel<<<grid_of(nrows * 32, 256), 256, 0, s>>>(d_row_ptr, nrows, d_col, scratch + 1);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if ((e = cudaMemcpyAsync(h, scratch, sizeof h, cudaMemcpyDeviceToHost, s)) != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return e;
  if (h[0] != kNone) {
    uint32_t c = 0;
    if ((e = cudaMemcpy(&c, d_col + h[0], 4, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
    r.code = PLAN_COLUMN_OUT_OF_RANGE;
    r.a = h[0];
    r.b = c;
    r.c = ncols;
    *out = r;
    return cudaSuccess;
  }
  if (h[1] != kNone) {
    // The first decreasing edge of that row, from a copy of the row.
    const uint64_t row = h[1], b = row_ptr[row], en = row_ptr[row + 1];
    std::vector<uint32_t> seg(en - b);
    if ((e = cudaMemcpy(seg.data(), d_col + b, (en - b) * 4, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
    r.code = PLAN_ROW_UNSORTED;
    r.a = row;
    for (uint64_t k = 1; k < seg.size(); ++k)
      if (seg[k] < seg[k - 1]) {
        r.b = b + k;
        break;
      }
    *out = r;
    return cudaSuccess;
  }
  uint64_t mx = 0;
  for (uint64_t row = 0; row < nrows; ++row) mx = std::max<uint64_t>(mx, row_ptr[row + 1] - row_ptr[row]);
  const uint64_t vals[3] = {nrows, ncols, col_len};
  for (int k = 0; k < 3; ++k)
    if (vals[k] > 0xffffffffull) {
      r.code = PLAN_TOO_LARGE;
      r.a = (uint64_t)k;
      r.b = vals[k];
      *out = r;
      return cudaSuccess;
    }
  r.code = PLAN_OK;
  r.nrows = nrows;
  r.ncols = ncols;
  r.nnz = col_len;
  r.max_row_nnz = mx;
  *out = r;
  return cudaSuccess;
}

cudaError_t launch_encode_narrow(int precision, const float* in, uint16_t* out, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  encode_kernel<<<grid_of(n, 256), 256, 0, s>>>(precision, in, out, n);
  return cudaGetLastError();
}

}  // namespace sparsl
