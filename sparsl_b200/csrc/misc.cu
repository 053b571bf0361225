// SpMM, standalone LIF, spike packing, trace counting and canary checks.
#include "common.cuh"
#include "misc.cuh"

namespace sparsl {
namespace {

// Y += A X for batch-minor X[ncols][n_vec] / Y[nrows][n_vec].  One warp owns
// one row; lane l folds vectors l and l + 32 of each 64-vector block, so every
// (row, vector) output is its own left fold in edge order, as row_dot_batched
// computes it (src/backend/mod.rs:2331-2360).  Each step loads one X row slice
// with a coalesced 128-byte access per 32 vectors.
template <int WK>
__global__ void __launch_bounds__(256) spmm_kernel(const uint32_t* __restrict__ ptr,
                                                   const uint32_t* __restrict__ idx, const void* w,
                                                   const float* __restrict__ x, float* __restrict__ y,
                                                   uint32_t nrows, uint32_t n_vec) {
  const int lane = threadIdx.x & 31;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t r = warp; r < nrows; r += nwarps) {
    const uint32_t s = __ldg(ptr + r), e = __ldg(ptr + r + 1);
    for (uint32_t vb = 0; vb < n_vec; vb += 64) {
      const uint32_t v0 = vb + lane, v1 = vb + 32 + lane;
      const bool ok0 = v0 < n_vec, ok1 = v1 < n_vec;
      float a0 = 0.0f, a1 = 0.0f;
      for (uint32_t e0 = s; e0 < e; e0 += 32) {
        const uint32_t ee = e0 + lane;
        uint32_t c = 0;
        float wv = 0.0f;
        if (ee < e) {
          c = __ldg(idx + ee);
          wv = load_weight<WK>(w, ee);
        }
        const uint32_t cnt = min(32u, e - e0);
        for (uint32_t j = 0; j < cnt; ++j) {
          const uint32_t cj = __shfl_sync(0xffffffffu, c, j);
          const float wj = __shfl_sync(0xffffffffu, wv, j);
          const float* xr = x + (uint64_t)cj * n_vec;
          if (ok0) a0 = fadd(a0, fmul(wj, __ldg(xr + v0)));
          if (ok1) a1 = fadd(a1, fmul(wj, __ldg(xr + v1)));
        }
      }
      float* yr = y + (uint64_t)r * n_vec;
      if (ok0) yr[v0] = fadd(yr[v0], a0);
      if (ok1) yr[v1] = fadd(yr[v1], a1);
    }
  }
}

// lif_step over dense currents (src/backend/mod.rs:2461-2501).
__global__ void lif_integrate_kernel(float* __restrict__ v, float* __restrict__ theta,
                                     const float* __restrict__ cur, uint8_t* __restrict__ spk, uint64_t n,
                                     float decay, float v_reset, float dtheta) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float vv = v[i];
    float th = theta[i];
    const float vol = fadd(fmul(vv, decay), cur[i]);
    uint8_t s = 0;
    if (vol >= th) {
      s = 1;
      vv = v_reset;
      th = fadd(th, dtheta);
    } else {
      vv = vol;
    }
    v[i] = vv;
    theta[i] = th;
    spk[i] = s;
  }
}

// pack_spikes_into (src/spikes.rs:237-262): LSB first, partial tail word
// zero-filled, words beyond packed_len(n) cleared.
__global__ void pack_kernel(const uint8_t* __restrict__ spk, uint64_t n, uint32_t* __restrict__ out,
                            uint64_t out_words) {
  for (uint64_t wi = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; wi < out_words;
       wi += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t word = 0;
    const uint64_t base = wi * 32;
    if (base < n) {
      const uint32_t lim = (uint32_t)min((uint64_t)32, n - base);
      for (uint32_t b = 0; b < lim; ++b) word |= (uint32_t)(spk[base + b] != 0) << b;
    }
    out[wi] = word;
  }
}

__global__ void popcount_kernel(const uint32_t* __restrict__ words, uint64_t nwords, uint32_t* slot) {
  uint32_t c = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nwords;
       i += (uint64_t)gridDim.x * blockDim.x)
    c += __popc(words[i]);
  c = __reduce_add_sync(0xffffffffu, c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(slot, c);
}

__global__ void canary_check_kernel(CanarySet set, uint32_t* err) {
  for (int d = blockIdx.x; d < set.count; d += gridDim.x) {
    const uint32_t* p = set.ptr[d];
    for (uint32_t i = threadIdx.x; i < kCanaryWords; i += blockDim.x)
      if (p[i] != kCanaryBits) set_err(err, DEVERR_CANARY);
  }
}

__global__ void fill_kernel(uint32_t* p, uint64_t n, uint32_t v) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

inline unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 148 * 16) {
  uint64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

}  // namespace

cudaError_t launch_spmm(const uint32_t* ptr, const uint32_t* idx, const void* w, int wkind, const float* x,
                        float* y, uint32_t nrows, uint32_t n_vec, int sm_count, cudaStream_t s) {
  if (nrows == 0) return cudaSuccess;
  const unsigned block = 256;
  uint64_t blocks = ((uint64_t)nrows * 32 + block - 1) / block;
  const uint64_t cap = (uint64_t)sm_count * 8;
  if (blocks > cap) blocks = cap;
  switch (wkind) {
    case W_F16: spmm_kernel<W_F16><<<(unsigned)blocks, block, 0, s>>>(ptr, idx, w, x, y, nrows, n_vec); break;
    case W_BF16: spmm_kernel<W_BF16><<<(unsigned)blocks, block, 0, s>>>(ptr, idx, w, x, y, nrows, n_vec); break;
    default: spmm_kernel<W_F32><<<(unsigned)blocks, block, 0, s>>>(ptr, idx, w, x, y, nrows, n_vec); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_lif_integrate(float* v, float* theta, const float* cur, uint8_t* spk, uint64_t n,
                                 float decay, float v_reset, float dtheta, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  lif_integrate_kernel<<<grid_for(n, 256), 256, 0, s>>>(v, theta, cur, spk, n, decay, v_reset, dtheta);
  return cudaGetLastError();
}

cudaError_t launch_pack(const uint8_t* spk, uint64_t n, uint32_t* out, uint64_t out_words, cudaStream_t s) {
  if (out_words == 0) return cudaSuccess;
  pack_kernel<<<grid_for(out_words, 256), 256, 0, s>>>(spk, n, out, out_words);
  return cudaGetLastError();
}

cudaError_t launch_popcount(const uint32_t* words, uint64_t nwords, uint32_t* slot, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(slot, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess || nwords == 0) return e;
  popcount_kernel<<<grid_for(nwords, 256, 148 * 2), 256, 0, s>>>(words, nwords, slot);
  return cudaGetLastError();
}

cudaError_t launch_canary_check(const CanarySet& set, uint32_t* err, cudaStream_t s) {
  if (set.count == 0) return cudaSuccess;
  canary_check_kernel<<<set.count, 64, 0, s>>>(set, err);
  return cudaGetLastError();
}

cudaError_t launch_fill(uint32_t* p, uint64_t n, uint32_t v, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(p, n, v);
  return cudaGetLastError();
}

}  // namespace sparsl
