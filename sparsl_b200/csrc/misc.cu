// SpMM, standalone LIF, spike packing, trace counting and canary checks.
#include "common.cuh"
#include "misc.cuh"

namespace sparsl {
namespace {

// Y += A X for batch-minor X[ncols][n_vec] / Y[nrows][n_vec].  One warp owns
// one row at a time and folds a 64-vector block per sweep of the row: lane l
// folds vectors 2l and 2l + 1 with one 8-byte load (V2: n_vec even, X and Y 8-byte
// aligned), else vectors l and l + 32.  Every (row, vector) output is its own
// left fold in edge order, as row_dot_batched computes it
// (src/backend/mod.rs:2331-2360).  Each step reads one X row slice with a
// coalesced 256-byte access per 64 vectors (Y rows alike); kSpmmDepth steps' gathers are
// issued before their dependent adds.  Warps are persistent and take work
// units from a counter, long rows first.
#ifndef SPARSL_SPMM_DEPTH
#define SPARSL_SPMM_DEPTH 4
#endif
constexpr int kSpmmDepth = SPARSL_SPMM_DEPTH;  // gathers in flight per lane and vector

template <int WK, bool V2>
__global__ void __launch_bounds__(256) spmm_kernel(const SpmmLaunch p) {
  const int lane = threadIdx.x & 31;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  const uint32_t nv = p.n_vec;
  const float* __restrict__ x = p.x;
  while (true) {
    uint32_t u = 0;
    if (lane == 0) u = atomicAdd(p.ctr, 1u);
    u = __shfl_sync(0xffffffffu, u, 0);
    if (u >= p.nunits) break;
    u += p.unit_base;
    uint32_t pb, pe;
    if (p.order) {
      pb = __ldg(p.unit_start + u);
      pe = __ldg(p.unit_start + u + 1);
    } else {
      pb = u * p.rows_per_unit;
      pe = min(p.nrows, pb + p.rows_per_unit);
    }
    for (uint32_t cb = pb; cb < pe; cb += 32) {
      // Lane l fetches the index and extent of the unit's row cb + l, so a
      // run of short rows does not wait on two dependent loads per row.
      uint32_t lr = 0, ls = 0, le = 0;
      if (cb + lane < pe) {
        lr = p.order ? __ldg(p.order + cb + lane) : cb + lane;
        ls = __ldg(p.ptr + lr);
        le = __ldg(p.ptr + lr + 1);
      }
      const uint32_t cn = min(32u, pe - cb);
      for (uint32_t q = 0; q < cn; ++q) {
        const uint32_t r = __shfl_sync(0xffffffffu, lr, q);
        const uint32_t s = __shfl_sync(0xffffffffu, ls, q), e = __shfl_sync(0xffffffffu, le, q);
        float* yr = p.y + (uint64_t)r * nv;
        for (uint32_t vb = 0; vb < nv; vb += 64) {
          const uint32_t v0 = V2 ? vb + 2 * lane : vb + lane, v1 = V2 ? v0 + 1 : vb + 32 + lane;
          const bool ok0 = v0 < nv, ok1 = V2 ? ok0 : v1 < nv;
          // Y is read before the fold, so its latency overlaps the gathers.
          float y0 = 0.0f, y1 = 0.0f;
          if (V2) {
            if (ok0) {
              const float2 t = *reinterpret_cast<const float2*>(yr + v0);
              y0 = t.x;
              y1 = t.y;
            }
          } else {
            if (ok0) y0 = yr[v0];
            if (ok1) y1 = yr[v1];
          }
          float a0 = 0.0f, a1 = 0.0f;
          for (uint32_t e0 = s; e0 < e; e0 += 32) {
            const uint32_t ee = e0 + lane;
            uint32_t c = 0;
            float wv = 0.0f;
            if (ee < e) {
              c = __ldg(p.idx + ee);
              wv = load_weight<WK>(p.w, ee);
            }
            const uint32_t cnt = min(32u, e - e0);
            uint32_t j = 0;
            for (; j + kSpmmDepth <= cnt; j += kSpmmDepth) {
              float xa[kSpmmDepth], xb[kSpmmDepth], wj[kSpmmDepth];
#pragma unroll
              for (int k = 0; k < kSpmmDepth; ++k) {
                const uint32_t cj = __shfl_sync(0xffffffffu, c, j + k);
                wj[k] = __shfl_sync(0xffffffffu, wv, j + k);
                const float* xr = x + (uint64_t)cj * nv;
                if (V2) {
                  const float2 t = ok0 ? __ldg(reinterpret_cast<const float2*>(xr + v0)) : make_float2(0.f, 0.f);
                  xa[k] = t.x;
                  xb[k] = t.y;
                } else {
                  xa[k] = ok0 ? __ldg(xr + v0) : 0.0f;
                  xb[k] = ok1 ? __ldg(xr + v1) : 0.0f;
                }
              }
#pragma unroll
              for (int k = 0; k < kSpmmDepth; ++k) {
                a0 = fadd(a0, fmul(wj[k], xa[k]));
                a1 = fadd(a1, fmul(wj[k], xb[k]));
              }
            }
            for (; j < cnt; ++j) {
              const uint32_t cj = __shfl_sync(0xffffffffu, c, j);
              const float wj = __shfl_sync(0xffffffffu, wv, j);
              const float* xr = x + (uint64_t)cj * nv;
              if (V2) {
                if (ok0) {
                  const float2 t = __ldg(reinterpret_cast<const float2*>(xr + v0));
                  a0 = fadd(a0, fmul(wj, t.x));
                  a1 = fadd(a1, fmul(wj, t.y));
                }
              } else {
                if (ok0) a0 = fadd(a0, fmul(wj, __ldg(xr + v0)));
                if (ok1) a1 = fadd(a1, fmul(wj, __ldg(xr + v1)));
              }
            }
          }
          // An empty row still adds its 0.0 fold: -0.0 + 0.0 is +0.0.
          if (V2) {
            if (ok0) *reinterpret_cast<float2*>(yr + v0) = make_float2(fadd(y0, a0), fadd(y1, a1));
          } else {
            if (ok0) yr[v0] = fadd(y0, a0);
            if (ok1) yr[v1] = fadd(y1, a1);
          }
        }
      }
    }
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

// The same four cells per thread with 16-byte loads and stores (v, theta and
// the currents 16-byte aligned, the spike bytes 4-byte aligned); a partial
// last quad is done cell by cell.
__device__ __forceinline__ uint8_t lif_cell(float& vv, float& th, float c, float decay, float v_reset,
                                            float dtheta) {
  const float vol = fadd(fmul(vv, decay), c);
  if (vol >= th) {
    vv = v_reset;
    th = fadd(th, dtheta);
    return 1;
  }
  vv = vol;
  return 0;
}

__global__ void lif_integrate4_kernel(float* __restrict__ v, float* __restrict__ theta,
                                      const float* __restrict__ cur, uint8_t* __restrict__ spk, uint64_t n,
                                      float decay, float v_reset, float dtheta) {
  const uint64_t quads = (n + 3) / 4;
  for (uint64_t q = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; q < quads;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = 4 * q;
    if (i + 4 <= n) {
      float4 vv = __ldcs(reinterpret_cast<const float4*>(v) + q);
      float4 th = __ldcs(reinterpret_cast<const float4*>(theta) + q);
      const float4 c = __ldcs(reinterpret_cast<const float4*>(cur) + q);
      uchar4 sp;
      sp.x = lif_cell(vv.x, th.x, c.x, decay, v_reset, dtheta);
      sp.y = lif_cell(vv.y, th.y, c.y, decay, v_reset, dtheta);
      sp.z = lif_cell(vv.z, th.z, c.z, decay, v_reset, dtheta);
      sp.w = lif_cell(vv.w, th.w, c.w, decay, v_reset, dtheta);
      __stcs(reinterpret_cast<float4*>(v) + q, vv);
      __stcs(reinterpret_cast<float4*>(theta) + q, th);
      reinterpret_cast<uchar4*>(spk)[q] = sp;
    } else {
      for (uint64_t k = i; k < n; ++k) {
        float vv = v[k], th = theta[k];
        spk[k] = lif_cell(vv, th, cur[k], decay, v_reset, dtheta);
        v[k] = vv;
        theta[k] = th;
      }
    }
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

// Ascending index list of the set bits of `words` (bit b of word w is line
// 32w + b): one block walks the words in order, 8 per thread per round, with
// a block-wide exclusive scan of the per-thread counts; *count receives the
// total.  Run after a tick kernel that wrote the packed spikes, it replaces a
// look-back inside the tick: the tick streams without waiting on other tiles.
constexpr int kCompactThreads = 1024;
constexpr int kCompactWords = 8;

__global__ void __launch_bounds__(kCompactThreads) compact_bits_kernel(const uint32_t* __restrict__ words,
                                                                      uint64_t nwords, uint32_t* __restrict__ idx,
                                                                      uint32_t* count, uint32_t idx_base) {
  __shared__ uint32_t s_warp[kCompactThreads / 32];
  __shared__ uint32_t s_carry;
  const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  constexpr uint64_t kRound = (uint64_t)kCompactThreads * kCompactWords;
  for (uint64_t r0 = 0; r0 < nwords; r0 += kRound) {
    const uint64_t w0 = r0 + (uint64_t)threadIdx.x * kCompactWords;
    uint32_t v[kCompactWords];
    uint32_t c = 0;
#pragma unroll
    for (int k = 0; k < kCompactWords; ++k) {
      v[k] = w0 + k < nwords ? __ldg(words + w0 + k) : 0u;
      c += __popc(v[k]);
    }
    uint32_t incl = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= (uint32_t)d) incl += o;
    }
    if (lane == 31) s_warp[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      uint32_t t = s_warp[lane];
      uint32_t ti = t;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, ti, d);
        if (lane >= (uint32_t)d) ti += o;
      }
      s_warp[lane] = ti - t;  // exclusive prefix of the warp totals
    }
    __syncthreads();
    uint32_t pos = s_carry + s_warp[wid] + incl - c;
#pragma unroll
    for (int k = 0; k < kCompactWords; ++k) {
      uint32_t b = v[k];
      while (b) {
        const uint32_t bit = __ffs(b) - 1;
        idx[pos++] = idx_base + (uint32_t)((w0 + k) * 32 + bit);
        b &= b - 1;
      }
    }
    __syncthreads();
    if (threadIdx.x == kCompactThreads - 1) s_carry = pos;  // the last thread ends at the round's total
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = s_carry;
}

__global__ void canary_check_kernel(CanarySet set, uint32_t* err) {
  for (int d = blockIdx.x; d < set.count; d += gridDim.x) {
    const uint32_t* p = set.ptr[d];
    for (uint32_t i = threadIdx.x; i < kCanaryWords; i += blockDim.x)
      if (p[i] != kCanaryBits) set_err(err, DEVERR_CANARY);
  }
}

// Tile 1 of a two-tile look-back whose tile 0 never publishes (its flag
// stays zero): the library's bounded wait runs out, records
// DEVERR_LOOKBACK_TIMEOUT and returns.  Only the failure-detection tests
// launch it.
__global__ void expired_wait_kernel(unsigned long long* flags, uint32_t* err, uint32_t* out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) out[0] = lookback_count(flags, 1, 1, err);
}

__global__ void fill_kernel(uint32_t* p, uint64_t n, uint32_t v) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ w, const uint32_t* __restrict__ idx, uint64_t n,
                              T* __restrict__ out) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n; k += (uint64_t)gridDim.x * blockDim.x)
    out[k] = w[__ldg(idx + k)];
}

inline unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 148 * 16) {
  uint64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

}  // namespace

template <bool V2>
static cudaError_t launch_spmm_t(const SpmmLaunch& p, int sm_count, cudaStream_t s) {
  const unsigned block = 256;
  int per_sm = 0;
  cudaError_t e;
  switch (p.wkind) {
    case W_F16: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, spmm_kernel<W_F16, V2>, block, 0); break;
    case W_BF16: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, spmm_kernel<W_BF16, V2>, block, 0); break;
    default: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, spmm_kernel<W_F32, V2>, block, 0); break;
  }
  if (e != cudaSuccess) return e;
  const uint64_t want = ((uint64_t)p.nunits * 32 + block - 1) / block;
  const uint64_t cap = (uint64_t)sm_count * (per_sm > 0 ? per_sm : 1);
  const unsigned blocks = (unsigned)(want < cap ? want : cap);
  switch (p.wkind) {
    case W_F16: spmm_kernel<W_F16, V2><<<blocks, block, 0, s>>>(p); break;
    case W_BF16: spmm_kernel<W_BF16, V2><<<blocks, block, 0, s>>>(p); break;
    default: spmm_kernel<W_F32, V2><<<blocks, block, 0, s>>>(p); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_spmm(const SpmmLaunch& p, int sm_count, cudaStream_t s) {
  if (p.nrows == 0 || p.nunits == 0) return cudaSuccess;
  const bool v2 = (p.n_vec % 2 == 0) && ((uintptr_t)p.x % 8 == 0) && ((uintptr_t)p.y % 8 == 0);
  return v2 ? launch_spmm_t<true>(p, sm_count, s) : launch_spmm_t<false>(p, sm_count, s);
}

cudaError_t launch_gather_weights(const void* w, const uint32_t* idx, uint64_t n, int wbytes, void* out,
                                  cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (wbytes == 4)
    gather_kernel<uint32_t><<<grid_for(n, 256), 256, 0, s>>>(static_cast<const uint32_t*>(w), idx, n,
                                                              static_cast<uint32_t*>(out));
  else
    gather_kernel<uint16_t><<<grid_for(n, 256), 256, 0, s>>>(static_cast<const uint16_t*>(w), idx, n,
                                                              static_cast<uint16_t*>(out));
  return cudaGetLastError();
}

cudaError_t launch_lif_integrate(float* v, float* theta, const float* cur, uint8_t* spk, uint64_t n,
                                 float decay, float v_reset, float dtheta, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const bool vec = ((uintptr_t)v % 16 == 0) && ((uintptr_t)theta % 16 == 0) && ((uintptr_t)cur % 16 == 0) &&
                   ((uintptr_t)spk % 4 == 0);
  if (vec) {
    const uint64_t quads = (n + 3) / 4;
    lif_integrate4_kernel<<<grid_for(quads, 256, 148 * 32), 256, 0, s>>>(v, theta, cur, spk, n, decay, v_reset,
                                                                          dtheta);
  } else {
    lif_integrate_kernel<<<grid_for(n, 256), 256, 0, s>>>(v, theta, cur, spk, n, decay, v_reset, dtheta);
  }
  return cudaGetLastError();
}

cudaError_t launch_pack(const uint8_t* spk, uint64_t n, uint32_t* out, uint64_t out_words, cudaStream_t s) {
  if (out_words == 0) return cudaSuccess;
  pack_kernel<<<grid_for(out_words, 256), 256, 0, s>>>(spk, n, out, out_words);
  return cudaGetLastError();
}

cudaError_t launch_compact_bits(const uint32_t* words, uint64_t nwords, uint32_t* idx, uint32_t* count,
                                uint32_t idx_base, cudaStream_t s) {
  compact_bits_kernel<<<1, kCompactThreads, 0, s>>>(words, nwords, idx, count, idx_base);
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

cudaError_t launch_expired_wait(void* scratch32, uint32_t* err, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(scratch32, 0, 32, s);
  if (e != cudaSuccess) return e;
  unsigned long long* flags = static_cast<unsigned long long*>(scratch32);
  expired_wait_kernel<<<1, 32, 0, s>>>(flags, err, reinterpret_cast<uint32_t*>(flags + 2));
  return cudaGetLastError();
}

cudaError_t launch_fill(uint32_t* p, uint64_t n, uint32_t v, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(p, n, v);
  return cudaGetLastError();
}

}  // namespace sparsl
