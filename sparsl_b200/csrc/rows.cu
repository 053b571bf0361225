// Row-fold engine: SpMV, spike SpMV, transpose SpMV and the fused LIF tick.
//
// Bit-exactness rule: each output line (CSR row or CSC column) is a strict
// left fold from 0.0 with separate round-to-nearest multiply and add, then
// combined with the old value exactly as the reference does:
//   y[r] = y[r] + (((0 + w0*x0) + w1*x1) + ...)     (src/backend/mod.rs:2259-2267)
// so one lane owns one line and a line is never split across lanes.
//
// Layout: a warp owns 32 lines -- 32 consecutive lines, or, for operators
// with skewed row lengths, 32 consecutive entries of the rows-by-descending-
// length order, so a warp's lanes fold rows of similar length and the
// longest rows start first.  Their CSR segments are staged
// chunk by chunk (kChunk entries per line) into a padded shared-memory tile by
// coalesced loads -- one 128-byte load per line per array -- and each lane
// then folds its own line out of shared memory.  The padding (stride kChunk+1)
// makes the transposed per-lane reads bank-conflict free.
#include "common.cuh"
#include "rows.cuh"

namespace sparsl {
namespace {

constexpr int kChunk = 32;
constexpr int kStride = kChunk + 1;

struct WarpStage {
  uint32_t idx[32][kStride];
  float w[32][kStride];
};

// f32 CSR launches stage chunks asynchronously into two buffers per warp.
#ifndef SPARSL_ROWS_ASYNC
#define SPARSL_ROWS_ASYNC 1
#endif
template <int WK, bool CSC>
constexpr bool kAsyncStage = SPARSL_ROWS_ASYNC && WK == W_F32 && !CSC;
#ifndef SPARSL_ROWS_STAGES
#define SPARSL_ROWS_STAGES 2
#endif
constexpr int kRowStages = SPARSL_ROWS_STAGES;  // stage buffers per warp on the asynchronous path
static_assert(kRowStages >= 2 && kRowStages <= 4, "2 to 4 stage buffers");

// 4-byte asynchronous global -> shared copy; a false `ok` zero-fills the
// destination and reads nothing.
template <typename T>
__device__ __forceinline__ void cp_async4(T* dst, const T* src, bool ok) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const uint32_t n = ok ? 4u : 0u;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

template <int WK, int XM, bool CSC, int EPI, bool COMPACT, bool ORDERED = false>
__global__ void __launch_bounds__(kRowWarps * 32) row_fold_kernel(const RowLaunch p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint32_t s_tile, s_base, s_last;
  __shared__ uint32_t s_wc[kRowWarps];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint32_t* s_bits = reinterpret_cast<uint32_t*>(smem);
  const size_t bits_bytes = (XM == X_BITS_SMEM) ? (((size_t)p.xbits_words * 4 + 15) & ~(size_t)15) : 0;
  // Stage buffers: [buffer][warp]; two buffers for asynchronous staging.
  WarpStage* st = reinterpret_cast<WarpStage*>(smem + bits_bytes) + wid;

  uint32_t tile;
  if constexpr (COMPACT) {
    // Tiles are numbered in start order so a tile only ever waits on tiles
    // that are already resident.
    if (threadIdx.x == 0) s_tile = atomicAdd(p.tile_ticket, 1u);
    __syncthreads();
    tile = s_tile;
  } else {
    tile = blockIdx.x;
  }

  if constexpr (XM == X_BITS_SMEM) {
    const uint4* src = reinterpret_cast<const uint4*>(p.xbits);
    const uint32_t nvec = p.xbits_words >> 2;
    for (uint32_t i = threadIdx.x; i < nvec; i += blockDim.x)
      reinterpret_cast<uint4*>(s_bits)[i] = __ldg(src + i);
    for (uint32_t i = (nvec << 2) + threadIdx.x; i < p.xbits_words; i += blockDim.x)
      s_bits[i] = __ldg(p.xbits + i);
    __syncthreads();
  }

  const uint32_t line0 = tile * kRowLines + wid * 32;
  uint32_t line = line0 + lane;
  const bool valid = line < p.nlines;
  if constexpr (ORDERED) {
    if (valid) line = __ldg(p.order + line);
  }
  uint32_t start = 0, len = 0;
  if (valid) {
    start = __ldg(p.ptr + line);
    len = __ldg(p.ptr + line + 1) - start;
  }
  const uint32_t maxlen = __reduce_max_sync(0xffffffffu, len);

  // The lane's operand value for entry column c (spikes are multiplied as
  // 0.0 / 1.0, never branched on).
  auto operand = [&](uint32_t c) -> float {
    if constexpr (XM == X_DENSE) {
      return __ldg(p.x + c);
    } else if constexpr (XM == X_BITS_SMEM) {
      return (float)((s_bits[c >> 5] >> (c & 31)) & 1u);
    } else {
      return (float)((__ldg(p.xbits + (c >> 5)) >> (c & 31)) & 1u);
    }
  };
  // Fold the lane's own entries of one staged chunk: every operand gather
  // first, then the dependent add chain in entry order.  Entries past the
  // line's end were staged as column 0 (in bounds: a line with entries
  // implies ncols >= 1), so all gathers are issued unconditionally; only
  // their adds are skipped.
  float sum = 0.0f;
  auto fold = [&](const WarpStage* sg, uint32_t k) {
    const uint32_t cnt = len > k ? min((uint32_t)kChunk, len - k) : 0u;
    float xv[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) xv[j] = operand(sg->idx[lane][j]);
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
      if ((uint32_t)j < cnt) sum = fadd(sum, fmul(sg->w[lane][j], xv[j]));
  };

  if constexpr (kAsyncStage<WK, CSC>) {
    // f32 CSR: chunks are staged by asynchronous 4-byte copies into two
    // buffers, so chunk k + 1 is in flight while chunk k is folded.  Lane l
    // copies entry k + l of each of the warp's 32 lines (coalesced per line);
    // entries past a line's end are zero-filled and never folded.
    auto stage = [&](WarpStage* sg, uint32_t k) {
      const uint32_t off = k + lane;
#pragma unroll 8
      for (int rr = 0; rr < 32; ++rr) {
        const uint32_t s_rr = __shfl_sync(0xffffffffu, start, rr);
        const uint32_t l_rr = __shfl_sync(0xffffffffu, len, rr);
        const bool ok = off < l_rr;
        const uint64_t e = ok ? (uint64_t)s_rr + off : 0;
        cp_async4(&sg->idx[rr][lane], p.idx + e, ok);
        cp_async4(&sg->w[rr][lane], reinterpret_cast<const float*>(p.w) + e, ok);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // kRowStages buffers: chunks k + 1 .. k + kRowStages - 1 are in flight
    // while chunk k folds.  Every iteration commits one group (empty past the
    // end), so "all but the newest kRowStages - 1 groups complete" is always
    // chunk k.
#pragma unroll
    for (int i = 0; i < kRowStages - 1; ++i) {
      if ((uint32_t)i * kChunk < maxlen) {
        stage(st + kRowWarps * i, (uint32_t)i * kChunk);
      } else {
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
    }
    int buf = 0;
    for (uint32_t k = 0; k < maxlen; k += kChunk) {
      const uint32_t ahead = k + (kRowStages - 1) * kChunk;
      const int abuf = (buf + kRowStages - 1) % kRowStages;
      if (ahead < maxlen) {
        stage(st + kRowWarps * abuf, ahead);
      } else {
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
      asm volatile("cp.async.wait_group %0;" ::"n"(kRowStages - 1) : "memory");
      __syncwarp();
      fold(st + kRowWarps * buf, k);
      __syncwarp();
      buf = (buf + 1 == kRowStages) ? 0 : buf + 1;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  } else {
    for (uint32_t k = 0; k < maxlen; k += kChunk) {
      const uint32_t off = k + lane;
      // Stage the chunk: lane l loads entry k + l of each of the warp's 32
      // lines (one coalesced access per line and array), all loads issued
      // into registers before any is stored so their latencies overlap.
      uint32_t ci[32];
      float cw[32];
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) {
        const uint32_t s_rr = __shfl_sync(0xffffffffu, start, rr);
        const uint32_t l_rr = __shfl_sync(0xffffffffu, len, rr);
        ci[rr] = 0u;
        cw[rr] = 0.0f;
        if (off < l_rr) {
          const uint32_t e = s_rr + off;
          ci[rr] = __ldg(p.idx + e);
          if constexpr (CSC) {
            cw[rr] = load_weight<WK>(p.w, __ldg(p.eidx + e));
          } else {
            cw[rr] = load_weight<WK>(p.w, e);
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) {
        st->idx[rr][lane] = ci[rr];
        st->w[rr][lane] = cw[rr];
      }
      __syncwarp();
      fold(st, k);
      __syncwarp();
    }
  }

  if constexpr (EPI == EPI_ACCUM) {
    if (valid) p.y[line] = fadd(p.y[line], sum);
  } else {
    // lif_step (src/backend/mod.rs:2461-2472): two roundings, then >= theta.
    bool spike = false;
    if (valid) {
      float vv = (p.v_src ? p.v_src : p.v)[line];
      float th = (p.theta_src ? p.theta_src : p.theta)[line];
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
      if (p.v_mirror) {
        p.v_mirror[line] = vv;
        p.theta_mirror[line] = th;
      }
    }
    // Lane i of the ballot is line 32w+i: exactly the LSB-first packing of
    // src/spikes.rs:237-262, with tail bits of a partial word left zero.
    // (Ordered launches leave packing to a pass over the spike bytes.)
    const uint32_t ballot = __ballot_sync(0xffffffffu, spike);
    if (!ORDERED && p.out_bits && lane == 0 && line0 < p.nlines) p.out_bits[line0 >> 5] = ballot;

    if constexpr (COMPACT) {
      const uint32_t ntiles = row_tiles(p.nlines);
      if (lane == 0) s_wc[wid] = __popc(ballot);
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t agg = 0;
        for (int w2 = 0; w2 < kRowWarps; ++w2) agg += s_wc[w2];
        const uint32_t excl = lookback_count(p.tile_flags, tile, agg, p.err);
        s_base = excl;
        if (tile == ntiles - 1) *p.idx_count = excl + agg;
      }
      __syncthreads();
      uint32_t wexcl = s_base;
      for (int w2 = 0; w2 < wid; ++w2) wexcl += s_wc[w2];
      if (spike) {
        const uint32_t lt = ballot & ((1u << lane) - 1u);
        p.idx_list[wexcl + __popc(lt)] = p.idx_base + line;
      }
      // The last tile to finish clears the look-back state for the next launch.
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

template <int WK, int XM, bool CSC, int EPI, bool COMPACT, bool ORDERED = false>
cudaError_t launch_t(const RowLaunch& p, cudaStream_t stream) {
  auto kern = row_fold_kernel<WK, XM, CSC, EPI, COMPACT, ORDERED>;
  const size_t bits_bytes = (XM == X_BITS_SMEM) ? (((size_t)p.xbits_words * 4 + 15) & ~(size_t)15) : 0;
  const size_t smem = bits_bytes + sizeof(WarpStage) * kRowWarps * (kAsyncStage<WK, CSC> ? kRowStages : 1);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const uint32_t tiles = row_tiles(p.nlines);
  kern<<<tiles, kRowWarps * 32, smem, stream>>>(p);
  return cudaGetLastError();
}

template <int WK>
cudaError_t dispatch_x(const RowLaunch& p, cudaStream_t s) {
  const bool csc = p.eidx != nullptr;
  const bool compact = p.idx_list != nullptr;
  if (p.order && !csc && !compact) {
    if (p.epilogue == EPI_ACCUM) {
      switch (p.xmode) {
        case X_DENSE: return launch_t<WK, X_DENSE, false, EPI_ACCUM, false, true>(p, s);
        case X_BITS_SMEM: return launch_t<WK, X_BITS_SMEM, false, EPI_ACCUM, false, true>(p, s);
        default: return launch_t<WK, X_BITS_GLOBAL, false, EPI_ACCUM, false, true>(p, s);
      }
    }
    switch (p.xmode) {
      case X_DENSE: return launch_t<WK, X_DENSE, false, EPI_LIF, false, true>(p, s);
      case X_BITS_SMEM: return launch_t<WK, X_BITS_SMEM, false, EPI_LIF, false, true>(p, s);
      default: return launch_t<WK, X_BITS_GLOBAL, false, EPI_LIF, false, true>(p, s);
    }
  }
  if (p.epilogue == EPI_ACCUM) {
    if (csc) return launch_t<WK, X_DENSE, true, EPI_ACCUM, false>(p, s);
    switch (p.xmode) {
      case X_DENSE: return launch_t<WK, X_DENSE, false, EPI_ACCUM, false>(p, s);
      case X_BITS_SMEM: return launch_t<WK, X_BITS_SMEM, false, EPI_ACCUM, false>(p, s);
      default: return launch_t<WK, X_BITS_GLOBAL, false, EPI_ACCUM, false>(p, s);
    }
  }
  switch (p.xmode) {
    case X_DENSE: return launch_t<WK, X_DENSE, false, EPI_LIF, false>(p, s);
    case X_BITS_SMEM:
      return compact ? launch_t<WK, X_BITS_SMEM, false, EPI_LIF, true>(p, s)
                     : launch_t<WK, X_BITS_SMEM, false, EPI_LIF, false>(p, s);
    default:
      return compact ? launch_t<WK, X_BITS_GLOBAL, false, EPI_LIF, true>(p, s)
                     : launch_t<WK, X_BITS_GLOBAL, false, EPI_LIF, false>(p, s);
  }
}

}  // namespace

cudaError_t launch_rows(const RowLaunch& p, cudaStream_t stream) {
  if (p.nlines == 0) return cudaSuccess;
  switch (p.wkind) {
    case W_F16: return dispatch_x<W_F16>(p, stream);
    case W_BF16: return dispatch_x<W_BF16>(p, stream);
    default: return dispatch_x<W_F32>(p, stream);
  }
}

}  // namespace sparsl
