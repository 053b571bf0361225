// Sliced-ELL fold for the transpose product.
//
// The reverse index has ragged lines (a column's nonzeros), so the 2-D TMA
// boxes of the uniform-row engine do not apply.  In sliced-ELL order the k-th
// entries of a slice's 32 lines are 128 contiguous bytes, so a warp reads them
// with one coalesced load per array and needs no shared-memory staging: each
// lane folds its own line, eight entries' loads and gathers in flight before
// their dependent adds.  Warps are persistent and take slices from a counter.
// With no shared memory in use, all of the SM's L1 caches x.
#include "common.cuh"
#include "sell.cuh"

namespace sparsl {
namespace {

constexpr int kSellWarps = 8;
constexpr int kSellDepth = 8;

template <int WK>
__device__ __forceinline__ float weight_at(const void* w, uint64_t i) {
  if constexpr (WK == W_F32) {
    return __ldg(reinterpret_cast<const float*>(w) + i);
  } else if constexpr (WK == W_F16) {
    return widen_f16(__ldg(reinterpret_cast<const unsigned short*>(w) + i));
  } else {
    return widen_bf16(__ldg(reinterpret_cast<const unsigned short*>(w) + i));
  }
}

template <int WK>
__global__ void __launch_bounds__(kSellWarps * 32) sell_fold_kernel(const SellLaunch p) {
  const int lane = threadIdx.x & 31;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  while (true) {
    uint32_t s = 0;
    if (lane == 0) s = atomicAdd(p.ctr, 1u);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (s >= p.nslices) break;
    const uint64_t base = __ldg(p.slice_ptr + s);
    const uint32_t depth = (uint32_t)((__ldg(p.slice_ptr + s + 1) - base) >> 5);
    const uint32_t line = s * 32 + lane;
    uint32_t len = 0;
    if (line < p.nlines) len = __ldg(p.line_ptr + line + 1) - __ldg(p.line_ptr + line);
    float sum = 0.0f;
    for (uint32_t k = 0; k < depth; k += kSellDepth) {
      uint32_t c[kSellDepth];
      float wv[kSellDepth], xv[kSellDepth];
#pragma unroll
      for (int j = 0; j < kSellDepth; ++j) {
        const bool in = k + j < depth;  // padding rows are row 0: always in bounds
        const uint64_t e = base + (uint64_t)(in ? k + j : 0) * 32 + lane;
        c[j] = __ldg(p.idx + e);
        wv[j] = weight_at<WK>(p.w, e);
      }
#pragma unroll
      for (int j = 0; j < kSellDepth; ++j) xv[j] = __ldg(p.x + c[j]);
#pragma unroll
      for (int j = 0; j < kSellDepth; ++j)
        if (k + j < len) sum = fadd(sum, fmul(wv[j], xv[j]));
    }
    if (line < p.nlines) p.y[line] = fadd(p.y[line], sum);
  }
  // The last warp out rewinds the counters for the next launch.
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(p.ctr + 1, 1u) == nwarps - 1) {
      atomicExch(p.ctr, 0u);
      atomicExch(p.ctr + 1, 0u);
    }
  }
}

template <int WK>
cudaError_t launch_t(const SellLaunch& p, int sm_count, cudaStream_t s) {
  int per_sm = 0;
  cudaError_t e =
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sell_fold_kernel<WK>, kSellWarps * 32, 0);
  if (e != cudaSuccess) return e;
  const uint64_t want = ((uint64_t)p.nslices + kSellWarps - 1) / kSellWarps;
  const uint64_t cap = (uint64_t)sm_count * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  sell_fold_kernel<WK><<<grid, kSellWarps * 32, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_sell(const SellLaunch& p, int sm_count, cudaStream_t s) {
  if (p.nlines == 0 || p.nslices == 0) return cudaSuccess;
  switch (p.wkind) {
    case W_F16: return launch_t<W_F16>(p, sm_count, s);
    case W_BF16: return launch_t<W_BF16>(p, sm_count, s);
    default: return launch_t<W_F32>(p, sm_count, s);
  }
}

}  // namespace sparsl
