// Dense-x SpMV over a uniform-length operator with x in shared memory.
//
// The streaming row fold (ell.cu) gathers x through L1, one scattered sector
// per gathered entry, and that gather rate bounds it.  Here one CTA per SM
// stages a panel of x (up to 216 KiB) in shared memory, where a warp's 32
// random gathers cost a few bank cycles instead of 32 L1 sectors.  When x is
// wider than one panel the CTA walks the panels in order: every lane owns one
// row and keeps the row's running fold in a register, and in panel k folds
// the row's entries whose columns fall in that panel.  The columns of a row
// are non-decreasing (the CSR gate's rule, src/sparse.rs:31), so those
// entries are the positions [split_k, split_k+1) that follow the ones panel
// k - 1 folded: each entry is folded once, in stored order, and the result is
// the reference's row_dot bit for bit (src/backend/mod.rs:2259-2267).
//
// The operator is read from the tile-interleaved copy described in
// panel.cuh: 16-bit panel-relative columns and the weights in 16-byte groups
// per lane, so one load brings a lane 8 columns, and a warp's load is 512
// contiguous bytes.  Two batches of 8 positions are in flight while a third
// folds, and a pass's first two batches load while the panel is copied in.
//
// The file also holds the ordered fold for skewed operators (rows of very
// different lengths), which reads a copy in the same 16-byte-group layout
// but has no panels: see ordered_fold_kernel.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "panel.cuh"
#include "rows.cuh"

namespace sparsl {
namespace {

constexpr uint32_t kPanelMaxWarps = 24;

struct PanelLaunch {
  const uint4* col16;  // 16-byte groups of 8 columns
  const uint4* w;      // 16-byte groups of 4 (f32) or 8 (16-bit) weights
  const uint16_t* split;
  const uint64_t* toff;  // ragged lines: group offset of each tile (null: tile * Lg)
  const float* x;
  float* y;
  uint32_t nrows, L, ncols, width, npanels;
  uint32_t Lg;  // 8-position groups per row: ceil(L / 8)
};

__device__ __forceinline__ void cp_async16(float4* dst, const float4* src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// Entry positions jb .. jb + 7 (jb a multiple of 8) of one lane's row.
template <int WK>
struct Batch {
  uint4 c;
  uint4 w[WK == W_F32 ? 2 : 1];
  // gbase: the tile's first 8-position group.
  __device__ __forceinline__ void load(const PanelLaunch& p, uint64_t gbase, uint32_t lane, uint32_t jb) {
    const uint64_t g = (gbase + jb / 8) * 32 + lane;
    c = __ldg(p.col16 + g);
    if constexpr (WK == W_F32) {
      const uint64_t gw = (gbase * 2 + jb / 4) * 32 + lane;
      w[0] = __ldg(p.w + gw);
      w[1] = __ldg(p.w + gw + 32);
    } else {
      w[0] = __ldg(p.w + g);
    }
  }
  __device__ __forceinline__ uint32_t col(int u) const {
    const uint32_t h = u < 2 ? c.x : u < 4 ? c.y : u < 6 ? c.z : c.w;
    return (u & 1) ? h >> 16 : h & 0xffffu;
  }
  __device__ __forceinline__ float weight(int u) const {
    if constexpr (WK == W_F32) {
      const uint4& q = w[u / 4];
      const uint32_t b = (u & 3) == 0 ? q.x : (u & 3) == 1 ? q.y : (u & 3) == 2 ? q.z : q.w;
      return __uint_as_float(b);
    } else {
      const uint32_t h = u < 2 ? w[0].x : u < 4 ? w[0].y : u < 6 ? w[0].z : w[0].w;
      const uint32_t bits = (u & 1) ? h >> 16 : h & 0xffffu;
      return WK == W_F16 ? widen_f16(bits) : widen_bf16(bits);
    }
  }
};

template <int WK>
__global__ void __launch_bounds__(kPanelMaxWarps * 32, 1) panel_spmv_kernel(const PanelLaunch p) {
  extern __shared__ __align__(16) float xs[];
  const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const uint32_t ntiles = (p.nrows + 31) / 32;
  const uint32_t wave = gridDim.x * nw;  // tiles in flight: one per warp
  const bool x16 = ((uintptr_t)p.x & 15u) == 0;
  for (uint32_t t0 = 0; t0 < ntiles; t0 += wave) {
    const uint32_t tile = t0 + blockIdx.x * nw + wid;
    const bool has = tile < ntiles;  // warp-uniform
    const uint32_t row = tile * 32 + lane;
    const bool valid = has && row < p.nrows;
    const uint64_t gbase = !has ? 0 : p.toff ? __ldg(p.toff + tile) : (uint64_t)tile * p.Lg;
    float acc = 0.f;
    // y is loaded now and used after the last panel, so the load's latency
    // (a PCIe round trip when y is in host memory) hides under the folds.
    const float y_in = valid ? p.y[row] : 0.f;
    for (uint32_t pn = 0; pn < p.npanels; ++pn) {
      const uint32_t pbase = pn * p.width;
      const uint32_t pw = min(p.width, p.ncols - pbase);  // floats in this panel
      // This lane folds positions [lo, hi) in this panel; the warp walks
      // 8-position batches over the union of its lanes' ranges.
      uint32_t lo = 0, hi = 0, jb = 0, jend = 0;
      Batch<WK> cur, b1, b2;
      __syncthreads();  // the previous panel's gathers are done
      if (has) {
        const uint16_t* sp = p.split + ((uint64_t)tile * (p.npanels + 1) + pn) * 32 + lane;
        lo = sp[0];
        hi = sp[32];
        jb = __reduce_min_sync(0xffffffffu, lo < hi ? lo : 0xffffffffu) & ~7u;
        jend = __reduce_max_sync(0xffffffffu, lo < hi ? hi : 0u);
        // The pass's first positions do not depend on x: their loads are in
        // flight while the panel arrives.
        if (jb < jend) cur.load(p, gbase, lane, jb);
        if (jb + 8 < jend) b1.load(p, gbase, lane, jb + 8);
      }
      // Each CTA starts the panel copy at its own offset, so the SMs do not
      // all ask the same L2 slices for the same lines at once.
      if (x16) {
        const uint32_t n4 = pw / 4;
        const uint32_t off = n4 ? ((uint32_t)(((uint64_t)blockIdx.x * n4) / gridDim.x) & ~31u) % n4 : 0;
        const float4* src = reinterpret_cast<const float4*>(p.x + pbase);
        float4* dst = reinterpret_cast<float4*>(xs);
        for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) {
          uint32_t m = i + off;
          if (m >= n4) m -= n4;
          cp_async16(dst + m, src + m);  // every copy of the thread in flight at once
        }
        for (uint32_t i = (pw & ~3u) + threadIdx.x; i < pw; i += blockDim.x) xs[i] = __ldg(p.x + pbase + i);
        asm volatile("cp.async.wait_all;" ::: "memory");
      } else {
        for (uint32_t i = threadIdx.x; i < pw; i += blockDim.x) xs[i] = __ldg(p.x + pbase + i);
      }
      __syncthreads();
      if (!has || jb >= jend) continue;
      // Columns are panel-relative and below the panel width, so every
      // gather stays inside the staged panel; only positions in [lo, hi)
      // are folded.
      auto step = [&](Batch<WK>& f, Batch<WK>& l) {
        if (jb + 16 < jend) l.load(p, gbase, lane, jb + 16);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float xv = xs[f.col(u)];
          const uint32_t e = jb + u;
          if (e >= lo && e < hi) acc = fadd(acc, fmul(f.weight(u), xv));
        }
        jb += 8;
        return jb < jend;
      };
      while (step(cur, b2) && step(b1, cur) && step(b2, b1)) {
      }
    }
    if (valid) p.y[row] = fadd(y_in, acc);
  }
}

// One thread per row: the row's first entry in each panel, by binary search
// over its non-decreasing columns.
__global__ void panel_split_kernel(const uint32_t* __restrict__ col, uint64_t nrows, uint32_t L, uint32_t width,
                                   uint32_t npanels, uint16_t* __restrict__ split, uint64_t rows_pad) {
  for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < rows_pad;
       r += (uint64_t)gridDim.x * blockDim.x) {
    uint16_t* out = split + ((r / 32) * (npanels + 1)) * 32 + (r & 31);
    if (r >= nrows) {
      for (uint32_t k = 0; k <= npanels; ++k) out[(uint64_t)k * 32] = 0;
      continue;
    }
    const uint32_t* c = col + r * L;
    out[0] = 0;
    for (uint32_t k = 1; k < npanels; ++k) {
      const uint32_t bound = k * width;
      uint32_t a = 0, b = L;  // first position with c >= bound
      while (a < b) {
        const uint32_t m = (a + b) / 2;
        if (c[m] < bound) a = m + 1;
        else b = m;
      }
      out[(uint64_t)k * 32] = (uint16_t)a;
    }
    out[(uint64_t)npanels * 32] = (uint16_t)L;
  }
}

// Output element o of an interleaved array with g positions per 16-byte
// group: which row and entry position it holds.
__device__ __forceinline__ void panel_slot(uint64_t o, uint32_t g, uint32_t groups, uint64_t& row, uint32_t& j) {
  const uint32_t jj = (uint32_t)(o % g);
  const uint64_t q = o / g;  // (tile * groups + group) * 32 + lane
  const uint32_t lane = (uint32_t)(q & 31);
  const uint64_t tg = q >> 5;
  row = (tg / groups) * 32 + lane;
  j = (uint32_t)(tg % groups) * g + jj;
}

__global__ void panel_col_kernel(const uint32_t* __restrict__ col, uint64_t nrows, uint32_t L, uint32_t width,
                                 uint16_t* __restrict__ col16, uint64_t total) {
  const uint32_t groups = (L + 7) / 8;
  for (uint64_t o = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; o < total;
       o += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t row;
    uint32_t j;
    panel_slot(o, 8, groups, row, j);
    uint16_t v = 0;
    if (row < nrows && j < L) v = (uint16_t)(col[row * L + j] % width);
    col16[o] = v;
  }
}

template <typename T>
__global__ void panel_w_kernel(const T* __restrict__ w, uint64_t nrows, uint32_t L, T* __restrict__ out,
                               uint64_t total) {
  constexpr uint32_t g = 16 / sizeof(T);
  const uint32_t groups = (L + 7) / 8 * (8 / g);
  for (uint64_t o = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; o < total;
       o += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t row;
    uint32_t j;
    panel_slot(o, g, groups, row, j);
    out[o] = (row < nrows && j < L) ? w[row * L + j] : T(0);
  }
}

// ---- Ordered copy (skewed operators): no panels, x gathered from global ----

struct OrdLaunch {
  const uint4* col;  // 16-byte groups of 4 columns
  const uint4* w;    // 16-byte groups of 4 (f32) or 8 (16-bit) weights
  const uint32_t* len;
  const uint64_t* toff;
  const uint32_t* order;   // all rows by descending length
  const uint32_t* rp;      // CSR arrays, for the long rows
  const uint32_t* ccol;
  const void* cw;
  uint32_t nlong;          // rows folded one warp each (the first nlong of order)
  const float* x;          // dense operand
  const uint32_t* xbits;   // or the spike bitmask (staged in shared memory)
  uint32_t xbits_words;
  float* y;                // EPI_ACCUM
  float* v;                // EPI_LIF state and spike bytes
  float* theta;
  uint8_t* spikes;
  LifHostState hs;         // optional state in host memory
  float decay, v_reset, dtheta;
  uint32_t nrows;
};

template <int WK>
struct OBatch {
  uint4 c[2];
  uint4 w[WK == W_F32 ? 2 : 1];
  __device__ __forceinline__ void load(const OrdLaunch& p, uint64_t gbase, uint32_t lane, uint32_t jb) {
    const uint64_t g4 = (gbase * 2 + jb / 4) * 32 + lane;
    c[0] = __ldg(p.col + g4);
    c[1] = __ldg(p.col + g4 + 32);
    if constexpr (WK == W_F32) {
      w[0] = __ldg(p.w + g4);
      w[1] = __ldg(p.w + g4 + 32);
    } else {
      w[0] = __ldg(p.w + (gbase + jb / 8) * 32 + lane);
    }
  }
  __device__ __forceinline__ uint32_t col(int u) const {
    const uint4& q = c[u / 4];
    return (u & 3) == 0 ? q.x : (u & 3) == 1 ? q.y : (u & 3) == 2 ? q.z : q.w;
  }
  __device__ __forceinline__ float weight(int u) const {
    if constexpr (WK == W_F32) {
      const uint4& q = w[u / 4];
      return __uint_as_float((u & 3) == 0 ? q.x : (u & 3) == 1 ? q.y : (u & 3) == 2 ? q.z : q.w);
    } else {
      const uint32_t h = u < 2 ? w[0].x : u < 4 ? w[0].y : u < 6 ? w[0].z : w[0].w;
      const uint32_t bits = (u & 1) ? h >> 16 : h & 0xffffu;
      return WK == W_F16 ? widen_f16(bits) : widen_bf16(bits);
    }
  }
};

constexpr int kOrdWarps = 8;       // dense x: 8-warp CTAs, one tile per warp
constexpr int kOrdBitsWarps = 24;  // spike bitmask in shared memory: one 24-warp CTA per SM

// The ordered fold.  The first nlong rows of the descending order (the long
// ones) take a warp each: lane k loads entries k, k + 32, ... of a 128-entry
// chunk straight from the CSR arrays (coalesced), gathers and multiplies
// them, and the products reach the fold one by one through shuffles, in
// stored order, while the next chunk's loads are in flight.  The other rows
// take a lane each over the tile-interleaved copy, 32 rows of similar length
// per warp, with two batches of 8 positions loading while a third folds.
// Either way a row folds its entries in order from 0.0, so the sum is
// row_dot bit for bit; the epilogue (y + sum, or the LIF step of
// src/backend/mod.rs:2461-2472) goes to the row through the order.  A dense
// x is gathered from global memory with no shared memory, so many 8-warp
// CTAs share an SM; a spike bitmask is staged in shared memory by persistent
// CTAs, one per SM, whose warps stride over the rows and tiles.
template <int WK, int XM, int EPI>
__global__ void __launch_bounds__(XM == X_DENSE ? kOrdWarps * 32 : kOrdBitsWarps * 32, XM == X_DENSE ? 2 : 1)
    ordered_fold_kernel(const OrdLaunch p) {
  extern __shared__ __align__(16) uint32_t s_bits[];
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nw = blockDim.x >> 5;
  const uint32_t ntiles = (p.nrows - p.nlong + 31) / 32;
  if constexpr (XM == X_BITS_SMEM) {
    const uint32_t nvec = p.xbits_words >> 2;
    for (uint32_t i = threadIdx.x; i < nvec; i += blockDim.x)
      reinterpret_cast<uint4*>(s_bits)[i] = __ldg(reinterpret_cast<const uint4*>(p.xbits) + i);
    for (uint32_t i = (nvec << 2) + threadIdx.x; i < p.xbits_words; i += blockDim.x) s_bits[i] = __ldg(p.xbits + i);
    __syncthreads();
  }
  auto gather = [&](uint32_t c) -> float {
    if constexpr (XM == X_DENSE)
      return __ldg(p.x + c);
    else
      return (float)((s_bits[c >> 5] >> (c & 31)) & 1u);
  };
  auto epilogue = [&](uint32_t r, float acc) {
    if constexpr (EPI == EPI_ACCUM) {
      p.y[r] = fadd(p.y[r], acc);
    } else {
      // lif_step: two roundings, then >= theta.
      float vv = (p.hs.v_src ? p.hs.v_src : p.v)[r], th = (p.hs.theta_src ? p.hs.theta_src : p.theta)[r];
      const float vol = fadd(fmul(vv, p.decay), acc);
      uint8_t spike = 0;
      if (vol >= th) {
        spike = 1;
        vv = p.v_reset;
        th = fadd(th, p.dtheta);
      } else {
        vv = vol;
      }
      p.v[r] = vv;
      p.theta[r] = th;
      p.spikes[r] = spike;
      if (p.hs.v_mirror) {
        p.hs.v_mirror[r] = vv;
        p.hs.theta_mirror[r] = th;
      }
    }
  };
  const uint32_t gwarp = blockIdx.x * nw + (threadIdx.x >> 5), nwarps = gridDim.x * nw;
  for (uint32_t lr = gwarp; lr < p.nlong; lr += nwarps) {
    const uint32_t r = __ldg(p.order + lr);
    const uint32_t a = __ldg(p.rp + r), n = __ldg(p.rp + r + 1) - a;
    float acc = 0.f;
    uint32_t c[4], cn[4];
    float w[4], wn[4];
    auto load = [&](uint32_t k0, uint32_t* cc, float* ww) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t e = k0 + 32 * q + lane;
        cc[q] = 0;
        ww[q] = 0.f;
        if (e < n) {
          cc[q] = __ldg(p.ccol + a + e);
          ww[q] = load_weight<WK>(p.cw, (uint64_t)a + e);
        }
      }
    };
    load(0, c, w);
    for (uint32_t k0 = 0; k0 < n; k0 += 128) {
      if (k0 + 128 < n) load(k0 + 128, cn, wn);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float prod = fmul(w[q], gather(c[q]));
        const uint32_t base = k0 + 32 * q;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float t = __shfl_sync(0xffffffffu, prod, k);
          if (base + k < n) acc = fadd(acc, t);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        c[q] = cn[q];
        w[q] = wn[q];
      }
    }
    if (lane == 0) epilogue(r, acc);
  }
  for (uint32_t tile = gwarp; tile < ntiles; tile += nwarps) {
    const uint32_t line = tile * 32 + lane;
    const bool valid = line < p.nrows - p.nlong;
    const uint32_t hi = valid ? __ldg(p.len + line) : 0u;
    const uint32_t jend = __reduce_max_sync(0xffffffffu, hi);
    const uint64_t gbase = __ldg(p.toff + tile);
    float acc = 0.f;
    uint32_t jb = 0;
    OBatch<WK> cur, b1, b2;
    if (jend > 0) cur.load(p, gbase, lane, 0);
    if (jend > 8) b1.load(p, gbase, lane, 8);
    auto step = [&](OBatch<WK>& f, OBatch<WK>& l) {
      if (jb + 16 < jend) l.load(p, gbase, lane, jb + 16);
      float xv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) xv[u] = gather(f.col(u));  // padding positions hold column 0
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (jb + u < hi) acc = fadd(acc, fmul(f.weight(u), xv[u]));
      jb += 8;
      return jb < jend;
    };
    if (jend > 0) {
      while (step(cur, b2) && step(b1, cur) && step(b2, b1)) {
      }
    }
    if (valid) epilogue(__ldg(p.order + p.nlong + line), acc);
  }
}

// One CTA per tile: the tile's columns (groups of 4 positions) and lengths.
__global__ void ordered_col_kernel(const uint32_t* __restrict__ rp, const uint32_t* __restrict__ col,
                                   const uint32_t* __restrict__ order, uint64_t nrows, uint64_t ntiles,
                                   const uint64_t* __restrict__ toff, uint32_t* __restrict__ ocol,
                                   uint32_t* __restrict__ olen) {
  for (uint64_t T = blockIdx.x; T < ntiles; T += gridDim.x) {
    const uint64_t g0 = toff[T], n = (toff[T + 1] - g0) * 256;
    for (uint64_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t lane = (uint32_t)(e >> 2) & 31u;
      const uint32_t j = (uint32_t)(e >> 7) * 4 + (uint32_t)(e & 3);
      const uint64_t line = T * 32 + lane;
      uint32_t v = 0;
      if (line < nrows) {
        const uint32_t r = order[line], a = rp[r];
        if (j < rp[r + 1] - a) v = col[(uint64_t)a + j];
      }
      ocol[g0 * 256 + e] = v;
    }
    if (threadIdx.x < 32) {
      const uint64_t line = T * 32 + threadIdx.x;
      uint32_t l = 0;
      if (line < nrows) {
        const uint32_t r = order[line];
        l = rp[r + 1] - rp[r];
      }
      olen[line] = l;
    }
  }
}

template <typename T>
__global__ void ordered_w_kernel(const uint32_t* __restrict__ rp, const T* __restrict__ w,
                                 const uint32_t* __restrict__ order, uint64_t nrows, uint64_t ntiles,
                                 const uint64_t* __restrict__ toff, T* __restrict__ ow) {
  constexpr uint32_t g = 16 / sizeof(T);
  for (uint64_t S = blockIdx.x; S < ntiles; S += gridDim.x) {
    const uint64_t g0 = toff[S], n = (toff[S + 1] - g0) * 256;
    for (uint64_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t lane = (uint32_t)(e / g) & 31u;
      const uint32_t j = (uint32_t)(e / (g * 32)) * g + (uint32_t)(e % g);
      const uint64_t line = S * 32 + lane;
      T v = T(0);
      if (line < nrows) {
        const uint32_t r = order[line], a = rp[r];
        if (j < rp[r + 1] - a) v = w[(uint64_t)a + j];
      }
      ow[g0 * 256 + e] = v;
    }
  }
}

// One CTA per slice (tile of 32 lines): its lines' entries into the
// 16-byte-group layout.  Positions past a line's length are padding (0).
__global__ void panel_sell_col_kernel(const unsigned long long* __restrict__ slice_ptr,
                                      const uint32_t* __restrict__ line_ptr, const uint32_t* __restrict__ sell_idx,
                                      uint64_t nlines, uint32_t nslices, const uint64_t* __restrict__ toff,
                                      uint32_t width, uint16_t* __restrict__ col16) {
  for (uint32_t T = blockIdx.x; T < nslices; T += gridDim.x) {
    const uint64_t base = slice_ptr[T], g0 = toff[T], n = (toff[T + 1] - g0) * 256;
    for (uint64_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t lane = (uint32_t)(e >> 3) & 31u;
      const uint32_t j = (uint32_t)(e >> 8) * 8 + (uint32_t)(e & 7);
      const uint64_t line = (uint64_t)T * 32 + lane;
      const uint32_t len = line < nlines ? line_ptr[line + 1] - line_ptr[line] : 0u;
      col16[g0 * 256 + e] = j < len ? (uint16_t)(sell_idx[base + (uint64_t)j * 32 + lane] % width) : (uint16_t)0;
    }
  }
}

template <typename T>
__global__ void panel_sell_w_kernel(const unsigned long long* __restrict__ slice_ptr,
                                    const uint32_t* __restrict__ line_ptr, const T* __restrict__ w_sell,
                                    uint64_t nlines, uint32_t nslices, const uint64_t* __restrict__ toff,
                                    T* __restrict__ out) {
  constexpr uint32_t g = 16 / sizeof(T);  // positions per 16-byte group
  for (uint32_t S = blockIdx.x; S < nslices; S += gridDim.x) {
    const uint64_t base = slice_ptr[S], g0 = toff[S], n = (toff[S + 1] - g0) * 256;
    for (uint64_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t lane = (uint32_t)(e / g) & 31u;
      const uint32_t j = (uint32_t)(e / (g * 32)) * g + (uint32_t)(e % g);
      const uint64_t line = (uint64_t)S * 32 + lane;
      const uint32_t len = line < nlines ? line_ptr[line + 1] - line_ptr[line] : 0u;
      out[g0 * 256 + e] = j < len ? w_sell[base + (uint64_t)j * 32 + lane] : T(0);
    }
  }
}

// One thread per line (all 32 of every slice): the line's first entry in
// each panel, by binary search over its ascending indices.
__global__ void panel_sell_split_kernel(const unsigned long long* __restrict__ slice_ptr,
                                        const uint32_t* __restrict__ line_ptr, const uint32_t* __restrict__ sell_idx,
                                        uint64_t nlines, uint64_t lines_pad, uint32_t width, uint32_t npanels,
                                        uint16_t* __restrict__ split) {
  for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < lines_pad;
       r += (uint64_t)gridDim.x * blockDim.x) {
    uint16_t* out = split + ((r / 32) * (npanels + 1)) * 32 + (r & 31);
    const uint32_t len = r < nlines ? line_ptr[r + 1] - line_ptr[r] : 0u;
    const uint32_t* c = sell_idx + slice_ptr[r / 32] + (r & 31);  // entry j at c[32 * j]
    out[0] = 0;
    for (uint32_t k = 1; k < npanels; ++k) {
      const uint32_t bound = k * width;
      uint32_t a = 0, b = len;
      while (a < b) {
        const uint32_t m = (a + b) / 2;
        if (c[(uint64_t)m * 32] < bound) a = m + 1;
        else b = m;
      }
      out[(uint64_t)k * 32] = (uint16_t)a;
    }
    out[(uint64_t)npanels * 32] = (uint16_t)len;
  }
}

constexpr int kPanelDevSlots = 64;

// Per device: the SM count, and the kernels' shared-memory limit raised once
// (host calls inside the launch path would sit between a caller's events).
int panel_sms(int dev) {
  static std::atomic<int> sms[kPanelDevSlots];
  if (dev < 0 || dev >= kPanelDevSlots) {
    int v = 0;
    return cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess ? v : 0;
  }
  int v = sms[dev].load(std::memory_order_relaxed);
  if (v == 0 && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    sms[dev].store(v, std::memory_order_relaxed);
  return v;
}

template <int WK>
cudaError_t go(int dev, const PanelLaunch& p, uint32_t grid, uint32_t threads, size_t smem, cudaStream_t s) {
  static std::atomic<bool> ready[kPanelDevSlots];
  const bool cached = dev >= 0 && dev < kPanelDevSlots;
  if (!cached || !ready[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(panel_spmv_kernel<WK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kPanelMaxFloats * 4));
    if (e != cudaSuccess) return e;
    if (cached) ready[dev].store(true, std::memory_order_release);
  }
  panel_spmv_kernel<WK><<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

uint32_t grid_for(uint64_t total) { return (uint32_t)std::min<uint64_t>((total + 255) / 256, 148ull * 16); }

}  // namespace

bool panel_geometry(uint64_t ncols, uint32_t& width, uint32_t& npanels) {
  if (ncols == 0) return false;
  const uint64_t np = (ncols + kPanelMaxFloats - 1) / kPanelMaxFloats;
  if (np > kPanelMaxPanels) return false;
  const uint64_t w = ((ncols + np - 1) / np + 3) & ~3ull;
  width = (uint32_t)std::min<uint64_t>(w, kPanelMaxFloats);
  npanels = (uint32_t)((ncols + width - 1) / width);
  return npanels <= kPanelMaxPanels;
}

cudaError_t launch_panel_build(const uint32_t* col, uint64_t nrows, uint32_t L, uint32_t width, uint32_t npanels,
                               uint16_t* col16, uint16_t* split, cudaStream_t stream) {
  if (nrows == 0 || L == 0 || L > kPanelMaxRowLen || width == 0) return cudaErrorInvalidValue;
  const uint64_t rows_pad = panel_tiles(nrows) * 32;
  panel_split_kernel<<<grid_for(rows_pad), 256, 0, stream>>>(col, nrows, L, width, npanels, split, rows_pad);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const uint64_t total = panel_col_elems(nrows, L);
  panel_col_kernel<<<grid_for(total), 256, 0, stream>>>(col, nrows, L, width, col16, total);
  return cudaGetLastError();
}

cudaError_t launch_panel_weights(const void* w, uint64_t nrows, uint32_t L, int esize, void* out,
                                 cudaStream_t stream) {
  if (nrows == 0 || L == 0) return cudaSuccess;
  const uint64_t total = panel_w_elems(nrows, L);
  if (esize == 4)
    panel_w_kernel<uint32_t><<<grid_for(total), 256, 0, stream>>>(static_cast<const uint32_t*>(w), nrows, L,
                                                                   static_cast<uint32_t*>(out), total);
  else
    panel_w_kernel<uint16_t><<<grid_for(total), 256, 0, stream>>>(static_cast<const uint16_t*>(w), nrows, L,
                                                                   static_cast<uint16_t*>(out), total);
  return cudaGetLastError();
}

cudaError_t launch_panel_build_sell(const unsigned long long* slice_ptr, const uint32_t* line_ptr,
                                    const uint32_t* sell_idx, uint64_t nlines, uint32_t nslices, const uint64_t* toff,
                                    uint32_t width, uint32_t npanels, uint16_t* col16, uint16_t* split,
                                    cudaStream_t stream) {
  if (nslices == 0) return cudaSuccess;
  if (width == 0) return cudaErrorInvalidValue;
  const uint32_t blocks = std::min<uint32_t>(nslices, 148u * 8);
  panel_sell_col_kernel<<<blocks, 256, 0, stream>>>(slice_ptr, line_ptr, sell_idx, nlines, nslices, toff, width, col16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const uint64_t lines_pad = (uint64_t)nslices * 32;
  panel_sell_split_kernel<<<grid_for(lines_pad), 256, 0, stream>>>(slice_ptr, line_ptr, sell_idx, nlines, lines_pad,
                                                                    width, npanels, split);
  return cudaGetLastError();
}

cudaError_t launch_panel_weights_sell(const unsigned long long* slice_ptr, const uint32_t* line_ptr,
                                      const void* w_sell, uint64_t nlines, uint32_t nslices, const uint64_t* toff,
                                      int esize, void* out, cudaStream_t stream) {
  if (nslices == 0) return cudaSuccess;
  const uint32_t blocks = std::min<uint32_t>(nslices, 148u * 8);
  if (esize == 4)
    panel_sell_w_kernel<uint32_t><<<blocks, 256, 0, stream>>>(slice_ptr, line_ptr,
                                                               static_cast<const uint32_t*>(w_sell), nlines, nslices,
                                                               toff, static_cast<uint32_t*>(out));
  else
    panel_sell_w_kernel<uint16_t><<<blocks, 256, 0, stream>>>(slice_ptr, line_ptr,
                                                               static_cast<const uint16_t*>(w_sell), nlines, nslices,
                                                               toff, static_cast<uint16_t*>(out));
  return cudaGetLastError();
}

cudaError_t launch_ordered_weights(const uint32_t* row_ptr, const void* w, int esize, const uint32_t* order,
                                   uint64_t nrows, const uint64_t* toff, void* ow, cudaStream_t stream) {
  const uint64_t ntiles = (nrows + 31) / 32;
  if (ntiles == 0) return cudaSuccess;
  const uint32_t blocks = (uint32_t)std::min<uint64_t>(ntiles, 148ull * 8);
  if (esize == 4)
    ordered_w_kernel<uint32_t><<<blocks, 256, 0, stream>>>(row_ptr, static_cast<const uint32_t*>(w), order, nrows,
                                                            ntiles, toff, static_cast<uint32_t*>(ow));
  else
    ordered_w_kernel<uint16_t><<<blocks, 256, 0, stream>>>(row_ptr, static_cast<const uint16_t*>(w), order, nrows,
                                                            ntiles, toff, static_cast<uint16_t*>(ow));
  return cudaGetLastError();
}

cudaError_t launch_ordered_build(const uint32_t* row_ptr, const uint32_t* col, const void* w, int esize,
                                 const uint32_t* order, uint64_t nrows, const uint64_t* toff, uint32_t* ocol,
                                 void* ow, uint32_t* olen, cudaStream_t stream) {
  const uint64_t ntiles = (nrows + 31) / 32;
  if (ntiles == 0) return cudaSuccess;
  const uint32_t blocks = (uint32_t)std::min<uint64_t>(ntiles, 148ull * 8);
  ordered_col_kernel<<<blocks, 256, 0, stream>>>(row_ptr, col, order, nrows, ntiles, toff, ocol, olen);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_ordered_weights(row_ptr, w, esize, order, nrows, toff, ow, stream);
}

namespace {

template <int WK, int XM, int EPI>
cudaError_t ordered_go(const OrdLaunch& p, cudaStream_t stream) {
  const uint32_t work = p.nlong + (p.nrows - p.nlong + 31) / 32;  // long rows and tiles, a warp each
  if constexpr (XM == X_DENSE) {
    const uint32_t blocks = std::max<uint32_t>(1, (work + kOrdWarps - 1) / kOrdWarps);
    ordered_fold_kernel<WK, XM, EPI><<<blocks, kOrdWarps * 32, 0, stream>>>(p);
  } else {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = ((size_t)p.xbits_words * 4 + 15) & ~(size_t)15;
    e = cudaFuncSetAttribute(ordered_fold_kernel<WK, XM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    const uint32_t blocks = std::max<uint32_t>(
        1, std::min<uint32_t>((work + kOrdBitsWarps - 1) / kOrdBitsWarps, (uint32_t)std::max(panel_sms(dev), 1)));
    ordered_fold_kernel<WK, XM, EPI><<<blocks, kOrdBitsWarps * 32, smem, stream>>>(p);
  }
  return cudaGetLastError();
}

template <int XM, int EPI>
cudaError_t ordered_wk(int wkind, const OrdLaunch& p, cudaStream_t stream) {
  switch (wkind) {
    case W_F32: return ordered_go<W_F32, XM, EPI>(p, stream);
    case W_F16: return ordered_go<W_F16, XM, EPI>(p, stream);
    default: return ordered_go<W_BF16, XM, EPI>(p, stream);
  }
}

OrdLaunch ordered_launch(const OrderedOp& op) {
  OrdLaunch p{};
  p.col = reinterpret_cast<const uint4*>(op.col);
  p.w = reinterpret_cast<const uint4*>(op.w);
  p.len = op.len;
  p.toff = op.toff;
  p.order = op.order;
  p.rp = op.row_ptr;
  p.ccol = op.csr_col;
  p.cw = op.csr_w;
  p.nlong = op.nlong;
  p.nrows = op.nrows;
  return p;
}

}  // namespace

cudaError_t launch_ordered_spmv(const OrderedOp& op, const float* x, float* y, cudaStream_t stream) {
  return launch_ordered_fold(op, x, nullptr, 0, y, nullptr, nullptr, nullptr, 0.f, 0.f, 0.f, stream);
}

cudaError_t launch_ordered_fold(const OrderedOp& op, const float* x, const uint32_t* xbits, uint32_t xbits_words,
                                float* y, float* v, float* theta, uint8_t* spikes, float decay, float v_reset,
                                float dtheta, cudaStream_t stream, const LifHostState& hs) {
  if (!op.ok || (xbits && (uint64_t)xbits_words * 4 > kOrderedBitsMaxBytes)) return cudaErrorInvalidValue;
  if (op.nrows == 0) return cudaSuccess;
  OrdLaunch p = ordered_launch(op);
  p.x = x;
  p.xbits = xbits;
  p.xbits_words = xbits_words;
  p.y = y;
  p.v = v;
  p.theta = theta;
  p.spikes = spikes;
  p.hs = hs;
  p.decay = decay;
  p.v_reset = v_reset;
  p.dtheta = dtheta;
  const bool lif = v != nullptr;
  if (xbits)
    return lif ? ordered_wk<X_BITS_SMEM, EPI_LIF>(op.wkind, p, stream)
               : ordered_wk<X_BITS_SMEM, EPI_ACCUM>(op.wkind, p, stream);
  return lif ? ordered_wk<X_DENSE, EPI_LIF>(op.wkind, p, stream) : ordered_wk<X_DENSE, EPI_ACCUM>(op.wkind, p, stream);
}

cudaError_t launch_panel_spmv(const PanelOp& op, const float* x, float* y, cudaStream_t stream) {
  if (!op.ok || op.width == 0 || op.width > kPanelMaxFloats) return cudaErrorInvalidValue;
  if (op.nrows == 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int sms = panel_sms(dev);
  const uint32_t ntiles = (op.nrows + 31) / 32;
  const uint32_t grid = std::min<uint32_t>(ntiles, (uint32_t)std::max(sms, 1));
  const uint32_t nw = std::min<uint32_t>(kPanelMaxWarps, (ntiles + grid - 1) / grid);
  const PanelLaunch p{reinterpret_cast<const uint4*>(op.col16),
                      reinterpret_cast<const uint4*>(op.w),
                      op.split, op.toff, x, y, op.nrows, op.L, op.ncols, op.width, op.npanels, (op.L + 7) / 8};
  const size_t smem = (size_t)op.width * 4;
  switch (op.wkind) {
    case W_F32: return go<W_F32>(dev, p, grid, nw * 32, smem, stream);
    case W_F16: return go<W_F16>(dev, p, grid, nw * 32, smem, stream);
    default: return go<W_BF16>(dev, p, grid, nw * 32, smem, stream);
  }
}

}  // namespace sparsl
