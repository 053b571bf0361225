// Row-fold engine for operators whose rows all hold the same number of
// entries L (row_ptr[r] == r * L): fixed fan-in networks and fixed-degree
// matrices.  Their column and weight arrays are dense [nrows x L] matrices, so
// a warp's 32 rows x 32 entries are one 2-D TMA box.
//
// Per warp: a 4-stage pipeline of (column tile, weight tile) pairs loaded by
// cp.async.bulk.tensor into 128-byte-swizzled shared memory and signalled by
// one mbarrier per stage; lane 0 keeps three chunks in flight while all 32
// lanes fold the current one.  The swizzle makes the transposed reads (lane r
// reads row r, 16 bytes at a time) bank-conflict free.  The arithmetic is the
// row-fold engine's: one lane per row, strict left fold, separate
// round-to-nearest multiply and add (src/backend/mod.rs:2259-2267).
//
// No multicast, no clusters: every load reads this GPU's own memory.
#include <cuda.h>

#include "common.cuh"
#include "ell.cuh"

namespace sparsl {
namespace {

constexpr int kStages = 4;
constexpr int kTileBytes = 32 * 32 * 4;  // one 32 x 32 box of 4-byte elements

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// One bounded probe of the barrier's phase.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int WK>
struct WBox {
  // bytes of one weight box: 32 rows x 32 entries
  static constexpr int kBytes = WK == W_F32 ? 4096 : 2048;
};

template <int WK, int XM, int EPI, bool COMPACT>
__global__ void __launch_bounds__(kEllWarps * 32, 1) ell_fold_kernel(const __grid_constant__ CUtensorMap tm_idx,
                                                                 const __grid_constant__ CUtensorMap tm_w,
                                                                 const RowLaunch p, uint32_t L) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kEllWarps][kStages];
  __shared__ uint32_t s_tile, s_base, s_last;
  __shared__ uint32_t s_wc[kEllWarps];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  // 1024-byte alignment of the swizzled tiles is required by the hardware.
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const size_t bits_bytes = (XM == X_BITS_SMEM) ? (((size_t)p.xbits_words * 4 + 1023) & ~(size_t)1023) : 0;
  uint32_t* s_bits = reinterpret_cast<uint32_t*>(smem);
  constexpr int kWBytes = WBox<WK>::kBytes;
  constexpr int kStageBytes = kTileBytes + kWBytes;
  unsigned char* wbase = smem + bits_bytes + (size_t)wid * kStages * kStageBytes;

  uint32_t tile;
  if constexpr (COMPACT) {
    if (threadIdx.x == 0) s_tile = atomicAdd(p.tile_ticket, 1u);
    __syncthreads();
    tile = s_tile;
  } else {
    tile = blockIdx.x;
  }
  if constexpr (XM == X_BITS_SMEM) {
    const uint4* src = reinterpret_cast<const uint4*>(p.xbits);
    const uint32_t nvec = p.xbits_words >> 2;
    for (uint32_t i = threadIdx.x; i < nvec; i += blockDim.x) reinterpret_cast<uint4*>(s_bits)[i] = __ldg(src + i);
    for (uint32_t i = (nvec << 2) + threadIdx.x; i < p.xbits_words; i += blockDim.x) s_bits[i] = __ldg(p.xbits + i);
  }

  const uint32_t row0 = tile * kEllLines + wid * 32;
  const uint32_t line = row0 + lane;
  const bool valid = line < p.nlines;
  const bool warp_active = row0 < p.nlines;
  const uint32_t nchunks = (L + 31) / 32;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[wid][s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  auto issue = [&](uint32_t c) {
    const int s = c % kStages;
    unsigned char* st = wbase + s * kStageBytes;
    mbar_expect_tx(&bars[wid][s], kStageBytes);
    tma_load_2d(st, &tm_idx, (int)(c * 32), (int)row0, &bars[wid][s]);
    tma_load_2d(st + kTileBytes, &tm_w, (int)(c * 32), (int)row0, &bars[wid][s]);
  };

  float sum = 0.0f;
  bool ok = true;
  uint32_t issued = 0;
  if (warp_active && lane == 0)
    for (; issued < nchunks && issued < (uint32_t)kStages; ++issued) issue(issued);
  __syncthreads();  // the bitmask (if any) is staged before the first fold
  if (warp_active) {
    issued = __shfl_sync(0xffffffffu, issued, 0);
    uint32_t c = 0;
    for (; c < nchunks; ++c) {
      const int s = c % kStages;
      if (!mbar_wait(&bars[wid][s], (c / kStages) & 1u)) {
        ok = false;
        break;
      }
      const unsigned char* st = wbase + s * kStageBytes;
      const unsigned char* irow = st + lane * 128;
      const uint32_t cnt = min(32u, L - c * 32);
      const uint32_t sw = lane & 7;
#pragma unroll
      for (uint32_t g = 0; g < 4; ++g) {  // 8 entries per group
        if (g * 8 >= cnt) break;
        const uint4 ca = *reinterpret_cast<const uint4*>(irow + (((2 * g) ^ sw) << 4));
        const uint4 cb = *reinterpret_cast<const uint4*>(irow + (((2 * g + 1) ^ sw) << 4));
        float wv[8];
        if constexpr (WK == W_F32) {
          const unsigned char* wrow = st + kTileBytes + lane * 128;
          const float4 wa = *reinterpret_cast<const float4*>(wrow + (((2 * g) ^ sw) << 4));
          const float4 wb = *reinterpret_cast<const float4*>(wrow + (((2 * g + 1) ^ sw) << 4));
          wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
          wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
        } else {
          const unsigned char* wrow = st + kTileBytes + lane * 64;
          const uint4 h = *reinterpret_cast<const uint4*>(wrow + ((g ^ ((lane >> 1) & 3)) << 4));
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t lo = hw[k] & 0xffffu, hi = hw[k] >> 16;
            if constexpr (WK == W_F16) {
              wv[2 * k] = widen_f16(lo);
              wv[2 * k + 1] = widen_f16(hi);
            } else {
              wv[2 * k] = widen_bf16(lo);
              wv[2 * k + 1] = widen_bf16(hi);
            }
          }
        }
        const uint32_t cv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
        const uint32_t lim = min(8u, cnt - g * 8);
        // The eight gathers and products are independent: issue them all
        // before the dependent add chain.  Entries past the row end were
        // zero-filled by the TMA box (column 0, weight 0), so their gathers
        // stay in bounds; only their adds are skipped.
        float prod[8];
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) {
          const uint32_t col = cv[k];
          float xv;
          if constexpr (XM == X_DENSE) {
            xv = __ldg(p.x + col);
          } else if constexpr (XM == X_BITS_SMEM) {
            xv = (float)((s_bits[col >> 5] >> (col & 31)) & 1u);
          } else {
            xv = (float)((__ldg(p.xbits + (col >> 5)) >> (col & 31)) & 1u);
          }
          prod[k] = fmul(wv[k], xv);
        }
        if (lim == 8) {
#pragma unroll
          for (uint32_t k = 0; k < 8; ++k) sum = fadd(sum, prod[k]);
        } else {
          for (uint32_t k = 0; k < lim; ++k) sum = fadd(sum, prod[k]);
        }
      }
      __syncwarp();
      if (c + kStages < nchunks) {
        if (lane == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(c + kStages);
        }
        ++issued;
      }
    }
    if (!ok) {
      set_err(p.err, DEVERR_LOOKBACK_TIMEOUT);
      // Let every copy still in flight land before the shared memory is released.
      for (uint32_t cc = c; cc < issued; ++cc) mbar_wait(&bars[wid][cc % kStages], (cc / kStages) & 1u);
    }
  }

  if constexpr (EPI == EPI_ACCUM) {
    if (valid && ok) p.y[line] = fadd(p.y[line], sum);
  } else {
    bool spike = false;
    if (valid && ok) {
      float vv = p.v[line];
      float th = p.theta[line];
      const float vol = fadd(fmul(vv, p.decay), sum);
      if (vol >= th) {
        spike = true;
        vv = p.v_reset;
        th = fadd(th, p.dtheta);
      } else {
        vv = vol;
      }
      p.v[line] = vv;
      p.theta[line] = th;
      p.spikes[line] = spike ? 1 : 0;
    }
    const uint32_t ballot = __ballot_sync(0xffffffffu, spike);
    if (p.out_bits && lane == 0 && warp_active) p.out_bits[row0 >> 5] = ballot;
    if constexpr (COMPACT) {
      const uint32_t ntiles = (p.nlines + kEllLines - 1) / kEllLines;
      if (lane == 0) s_wc[wid] = __popc(ballot);
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t agg = 0;
        for (int w2 = 0; w2 < kEllWarps; ++w2) agg += s_wc[w2];
        const uint32_t excl = lookback_count(p.tile_flags, tile, agg, p.err);
        s_base = excl;
        if (tile == ntiles - 1) *p.idx_count = excl + agg;
      }
      __syncthreads();
      uint32_t wexcl = s_base;
      for (int w2 = 0; w2 < wid; ++w2) wexcl += s_wc[w2];
      if (spike) p.idx_list[wexcl + __popc(ballot & ((1u << lane) - 1u))] = p.idx_base + line;
      if (threadIdx.x == 0) {
        __threadfence();
        s_last = (atomicAdd(p.tile_ticket + 1, 1u) == ntiles - 1) ? 1u : 0u;
      }
      __syncthreads();
      if (s_last) {
        for (uint32_t i = threadIdx.x; i < ntiles; i += blockDim.x) p.tile_flags[i] = 0ull;
        if (threadIdx.x == 0) {
          p.tile_ticket[0] = 0;
          p.tile_ticket[1] = 0;
        }
      }
    }
  }
}

template <int WK, int XM, int EPI, bool COMPACT>
cudaError_t launch_t(const EllMaps& m, const RowLaunch& p, uint32_t L, cudaStream_t stream) {
  auto kern = ell_fold_kernel<WK, XM, EPI, COMPACT>;
  const size_t bits_bytes = (XM == X_BITS_SMEM) ? (((size_t)p.xbits_words * 4 + 1023) & ~(size_t)1023) : 0;
  const size_t smem = 1024 + bits_bytes + (size_t)kEllWarps * kStages * (kTileBytes + WBox<WK>::kBytes);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const uint32_t tiles = (p.nlines + kEllLines - 1) / kEllLines;
  kern<<<tiles, kEllWarps * 32, smem, stream>>>(*reinterpret_cast<const CUtensorMap*>(m.idx),
                                                *reinterpret_cast<const CUtensorMap*>(m.w), p, L);
  return cudaGetLastError();
}

template <int WK>
cudaError_t dispatch(const EllMaps& m, const RowLaunch& p, uint32_t L, cudaStream_t s) {
  const bool compact = p.idx_list != nullptr;
  if (p.epilogue == EPI_ACCUM) {
    switch (p.xmode) {
      case X_DENSE: return launch_t<WK, X_DENSE, EPI_ACCUM, false>(m, p, L, s);
      case X_BITS_SMEM: return launch_t<WK, X_BITS_SMEM, EPI_ACCUM, false>(m, p, L, s);
      default: return launch_t<WK, X_BITS_GLOBAL, EPI_ACCUM, false>(m, p, L, s);
    }
  }
  switch (p.xmode) {
    case X_DENSE: return launch_t<WK, X_DENSE, EPI_LIF, false>(m, p, L, s);
    case X_BITS_SMEM:
      return compact ? launch_t<WK, X_BITS_SMEM, EPI_LIF, true>(m, p, L, s)
                     : launch_t<WK, X_BITS_SMEM, EPI_LIF, false>(m, p, L, s);
    default:
      return compact ? launch_t<WK, X_BITS_GLOBAL, EPI_LIF, true>(m, p, L, s)
                     : launch_t<WK, X_BITS_GLOBAL, EPI_LIF, false>(m, p, L, s);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

bool ell_encode(EllMaps& m, const uint32_t* col, const void* w, int wkind, uint64_t nrows, uint32_t L) {
  m.ok = false;
  EncodeTiledFn enc = encode_fn();
  if (!enc || nrows == 0 || L == 0 || nrows > 0xffffffffull) return false;
  const uint32_t wbytes = wkind == W_F32 ? 4 : 2;
  if ((L * 4) % 16 || (L * wbytes) % 16) return false;  // row pitch must be a multiple of 16 bytes
  if ((reinterpret_cast<uintptr_t>(col) | reinterpret_cast<uintptr_t>(w)) & 15) return false;
  static_assert(sizeof(CUtensorMap) == sizeof(m.idx), "tensor map storage");
  cuuint64_t dims[2] = {L, nrows};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  cuuint64_t istride[1] = {(cuuint64_t)L * 4};
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(m.idx), CU_TENSOR_MAP_DATA_TYPE_UINT32, 2,
                   const_cast<uint32_t*>(col), dims, istride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  cuuint64_t wstride[1] = {(cuuint64_t)L * wbytes};
  r = enc(reinterpret_cast<CUtensorMap*>(m.w),
          wkind == W_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w),
          dims, wstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          wkind == W_F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  m.L = L;
  m.ok = true;
  return true;
}

cudaError_t launch_ell(const EllMaps& m, const RowLaunch& p, cudaStream_t stream) {
  if (p.nlines == 0) return cudaSuccess;
  switch (p.wkind) {
    case W_F16: return dispatch<W_F16>(m, p, m.L, stream);
    case W_BF16: return dispatch<W_BF16>(m, p, m.L, stream);
    default: return dispatch<W_F32>(m, p, m.L, stream);
  }
}

}  // namespace sparsl
