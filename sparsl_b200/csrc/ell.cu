// Row-fold engine for operators whose rows all hold the same number of
// entries L (row_ptr[r] == r * L): fixed fan-in networks and fixed-degree
// matrices.  Their column and weight arrays are dense [nrows x L] matrices, so
// a warp's 32 rows x kChunk entries are one 2-D TMA box.
//
// Persistent and streaming: one CTA per SM, 12 to 16 warps, and every warp
// walks its own sequence of 32-row tiles.  Per warp a ring of
// (column box, weight box) pairs is filled by cp.async.bulk.tensor into
// swizzled shared memory and signalled by one mbarrier per stage; lane 0
// refills a stage as soon as the warp has folded it, running ahead across
// tile boundaries, so the pipeline never drains between tiles.  The swizzle
// makes the transposed reads (lane r reads row r, 16 bytes at a time) bank
// conflict free.  The arithmetic is the row-fold engine's: one lane per row,
// strict left fold from 0.0, separate round-to-nearest multiply and add
// (src/backend/mod.rs:2259-2267).
//
// Spike operands live in shared memory: the whole bitmask when it fits
// (X_BITS_SMEM), otherwise (X_BITS_GLOBAL) a summary with one bit per group of
// G columns ("some column of this group spiked") built once per CTA; a gather
// reads the global bitmask only when its group's summary bit is set.  The
// bitmask itself is exact, so the summary only decides which zero words need
// not be fetched.
//
// Streaming loads carry an L2 evict-first policy so the gathered operand (x,
// bitmask) stays resident in L2 while the matrix streams past it.  No
// multicast, no clusters: every load reads this GPU's own memory.
#include <cuda.h>

#include "common.cuh"
#include "ell.cuh"

namespace sparsl {
namespace {

// Compile-time shape: kChunk entries per row per stage (16 or 32).  The
// number of stages per warp is chosen at launch from the shared memory left
// after the spike operand (kMinStages..kMaxStages).
#ifndef SPARSL_ELL_CHUNK
#define SPARSL_ELL_CHUNK 16
#endif
constexpr int kChunk = SPARSL_ELL_CHUNK;
static_assert(kChunk == 16 || kChunk == 32, "chunk of 16 or 32 entries");
constexpr int kMinStages = 2, kMaxStages = 8;
// Dense x: gathers go through L1/L2, so fewer stages (and more CTAs per SM)
// can hide more gather latency than deeper streaming does.
#ifndef SPARSL_ELL_DENSE_STAGES
#define SPARSL_ELL_DENSE_STAGES 2
#endif
constexpr int kDenseStages = SPARSL_ELL_DENSE_STAGES;
constexpr int kIdxRow = kChunk * 4;            // bytes of one row of a column box
constexpr int kIdxBox = 32 * kIdxRow;          // column box: 32 rows x kChunk entries
constexpr uint32_t kSumMaxWords = 16384;       // 64 KiB summary
constexpr uint32_t kFifo = 16;                 // > kMaxStages: tiles a warp can run ahead
constexpr size_t kSmemBudget = 227 * 1024 - 4096;  // per-CTA limit less static use and alignment slack

// 16-byte piece p of row `row` of a box whose rows are RB bytes, under the
// matching TMA swizzle (RB = 32, 64 or 128 bytes: SWIZZLE_32B/64B/128B).
template <int RB>
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t p) {
  return ((p ^ (((row * RB) >> 7) & (RB / 16 - 1))) << 4);
}
template <int RB>
constexpr CUtensorMapSwizzle swizzle_mode() {
  return RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

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

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

template <int WK>
struct WBox {
  static constexpr int kRow = WK == W_F32 ? kChunk * 4 : kChunk * 2;  // bytes of one weight-box row
  static constexpr int kBytes = 32 * kRow;
  static constexpr int kStage = kIdxBox + kBytes;
};

// Summary bits of one bitmask word for groups of 2^gs columns, gs in [3, 5]:
// bit j is set when bits [j*G, (j+1)*G) of the word are not all zero.
__device__ __forceinline__ uint32_t word_groups(uint32_t w, uint32_t gs) {
  if (gs == 3) {
    const uint32_t t = (((w & 0x7f7f7f7fu) + 0x7f7f7f7fu) | w) & 0x80808080u;  // high bit per nonzero byte
    return ((t >> 7) & 1u) | ((t >> 14) & 2u) | ((t >> 21) & 4u) | ((t >> 28) & 8u);
  }
  if (gs == 4) return ((w & 0xffffu) ? 1u : 0u) | ((w >> 16) ? 2u : 0u);
  return w ? 1u : 0u;
}

// Builds the shared-memory summary: summary word s covers bitmask words
// [s*G, s*G + G) (G = 2^gs), i.e. 32 groups of G columns.
__device__ void build_summary(uint32_t* s_sum, const uint32_t* __restrict__ bits, uint32_t words, uint32_t gs,
                              uint32_t sum_words) {
  const uint32_t G = 1u << gs;
  for (uint32_t s = threadIdx.x; s < sum_words; s += blockDim.x) {
    const uint32_t w0 = s << gs;
    uint32_t out = 0;
    if (gs <= 5) {
      const uint32_t per = 32u >> gs;  // summary bits per bitmask word
      for (uint32_t k = 0; k < G; k += 8) {
        uint32_t v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = (w0 + k + u < words) ? __ldg(bits + w0 + k + u) : 0u;
#pragma unroll
        for (int u = 0; u < 8; ++u) out |= word_groups(v[u], gs) << ((k + u) * per);
      }
    } else {
      const uint32_t wpb = G >> 5;  // bitmask words per summary bit
      for (uint32_t b = 0; b < 32; ++b) {
        uint32_t acc = 0;
        for (uint32_t k = 0; k < wpb; ++k) {
          const uint32_t wi = w0 + b * wpb + k;
          acc |= (wi < words) ? __ldg(bits + wi) : 0u;
        }
        out |= (acc ? 1u : 0u) << b;
      }
    }
    s_sum[s] = out;
  }
}

// Warp-wide decoupled look-back over 32-row tile counts.  Flags are tagged
// with the launch's epoch, so no launch has to clear them for the next one:
// [63:34] epoch, [33:32] status (1 aggregate, 2 inclusive), [31:0] count.
// Each flag word carries everything it publishes, so relaxed accesses do.
__device__ uint32_t lookback_warp(unsigned long long* flags, uint32_t tile, uint32_t agg, uint32_t epoch,
                                  uint32_t* err, int lane) {
  const unsigned long long tag = (unsigned long long)epoch << 34;
  if (lane == 0) st_relaxed_u64(flags + tile, tag | (tile == 0 ? 2ull : 1ull) << 32 | agg);
  uint32_t excl = 0;
  int64_t base = tile;  // next window covers tiles [base-32, base)
  uint32_t spins = 0;
  bool timed_out = false;
  while (base > 0) {
    const int64_t j = base - 1 - lane;
    uint32_t st = 2, cnt = 0;
    if (j >= 0) {
      const unsigned long long f = ld_relaxed_u64(flags + j);
      st = ((f >> 34) == epoch) ? (uint32_t)(f >> 32) & 3u : 0u;
      cnt = (uint32_t)f;
    }
    const uint32_t incl = __ballot_sync(0xffffffffu, st == 2);
    const uint32_t ready = __ballot_sync(0xffffffffu, st != 0);
    const uint32_t upto = incl ? ((incl & (0u - incl)) << 1) - 1u : 0xffffffffu;  // lanes up to the first inclusive
    if ((ready & upto) == upto) {
      uint32_t c = (upto >> lane) & 1u ? cnt : 0u;
#pragma unroll
      for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
      excl += c;
      if (incl) break;
      base -= 32;
      continue;
    }
    if (++spins > kSpinLimit) {
      timed_out = true;
      break;
    }
    __nanosleep(32);
  }
  if (lane == 0) {
    if (timed_out) set_err(err, DEVERR_LOOKBACK_TIMEOUT);
    if (tile != 0) st_relaxed_u64(flags + tile, tag | 2ull << 32 | (excl + agg));
  }
  return excl;
}

// One spike bit of column `col` as 0.0f / 1.0f.
template <int XM>
__device__ __forceinline__ float spike_value(const uint32_t* s_x, const uint32_t* __restrict__ gbits, uint32_t col,
                                             uint32_t gs) {
  uint32_t bit;
  if constexpr (XM == X_BITS_SMEM) {
    const uint32_t w = s_x[col >> 5];
    bit = __funnelshift_r(w, w, col) & 1u;  // the shift count is taken mod 32
  } else {
    const uint32_t q = col >> gs;
    const uint32_t sw = s_x[q >> 5];
    bit = 0;
    if (__funnelshift_r(sw, sw, q) & 1u) {
      const uint32_t w = __ldg(gbits + (col >> 5));
      bit = __funnelshift_r(w, w, col) & 1u;
    }
  }
  return __uint_as_float(bit * 0x3f800000u);  // exactly 0.0f or 1.0f
}

template <int WK, int XM, int EPI, bool COMPACT, int NW>
__global__ void __launch_bounds__(NW * 32, 1)
    ell_stream_kernel(const __grid_constant__ CUtensorMap tm_idx, const __grid_constant__ CUtensorMap tm_w,
                      const RowLaunch p, uint32_t L, uint32_t gs, uint32_t sum_words, uint32_t nst) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[NW][kMaxStages];
  __shared__ uint32_t s_fifo[NW][kFifo];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  // 1024-byte alignment keeps every swizzled box on its swizzle period.
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStageBytes = WBox<WK>::kStage;
  unsigned char* ring = smem + (size_t)wid * nst * kStageBytes;
  uint32_t* s_x = reinterpret_cast<uint32_t*>(smem + (size_t)NW * nst * kStageBytes);

  const uint32_t ntiles = (p.nlines + 31) / 32;
  const uint32_t nch = (L + kChunk - 1) / kChunk;
  const uint32_t nwarps = gridDim.x * NW;
  const uint64_t pol = evict_first_policy();

  if (lane == 0) {
    for (uint32_t s = 0; s < nst; ++s) mbar_init(&bars[wid][s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // Tile sequence: dynamic tickets.  They balance the load when CTAs start
  // at different times (another kernel's tail still holds some SMs), and they
  // keep the compaction look-back safe: a ticket is only taken by a running
  // warp, so a tile only ever waits on tiles whose owners are running.
  auto grab = [&]() -> uint32_t {
    uint32_t t = 0;
    if (lane == 0) t = atomicAdd(p.tile_ticket, 1u);
    return __shfl_sync(0xffffffffu, t, 0);
  };

  // Issue state (warp-uniform): next tile / chunk, ring slot, chunks issued.
  uint32_t i_tile = grab(), i_ch = 0, i_slot = 0, issued = 0, fifo_w = 0, fifo_r = 0;
  bool i_more = i_tile < ntiles;
  if (i_more) s_fifo[wid][fifo_w++ % kFifo] = i_tile;
  auto issue_next = [&]() {
    if (!i_more) return;
    if (i_ch == nch) {
      i_tile = grab();
      i_ch = 0;
      if (i_tile >= ntiles) {
        i_more = false;
        return;
      }
      s_fifo[wid][fifo_w++ % kFifo] = i_tile;
    }
    if (lane == 0) {
      unsigned char* st = ring + i_slot * kStageBytes;
      mbar_expect_tx(&bars[wid][i_slot], kStageBytes);
      tma_load_2d(st, &tm_idx, (int)(i_ch * kChunk), (int)(i_tile * 32), &bars[wid][i_slot], pol);
      tma_load_2d(st + kIdxBox, &tm_w, (int)(i_ch * kChunk), (int)(i_tile * 32), &bars[wid][i_slot], pol);
    }
    i_slot = (i_slot + 1 == nst) ? 0 : i_slot + 1;
    ++issued;
    ++i_ch;
  };
  for (uint32_t s = 0; s < nst; ++s) issue_next();

  // Spike operand into shared memory while the first boxes are in flight.
  if constexpr (XM == X_BITS_SMEM) {
    const uint32_t nvec = p.xbits_words >> 2;
    const uint4* src = reinterpret_cast<const uint4*>(p.xbits);
    for (uint32_t i = threadIdx.x; i < nvec; i += blockDim.x) reinterpret_cast<uint4*>(s_x)[i] = __ldg(src + i);
    for (uint32_t i = (nvec << 2) + threadIdx.x; i < p.xbits_words; i += blockDim.x) s_x[i] = __ldg(p.xbits + i);
  } else if constexpr (XM == X_BITS_GLOBAL) {
    build_summary(s_x, p.xbits, p.xbits_words, gs, sum_words);
  }
  __syncthreads();

  bool ok = true;
  uint32_t c_slot = 0, c_phase = 0, consumed = 0;
  constexpr int kWRow = WBox<WK>::kRow;
  while (ok && fifo_r != fifo_w) {
    const uint32_t tile = s_fifo[wid][fifo_r++ % kFifo];
    float sum = 0.0f;
    // The tile's y (or LIF state) is loaded now and used after its last
    // chunk, so the load's latency (a PCIe round trip when it is in host
    // memory) hides under the tile's stream.
    float v_in = 0.f, th_in = 0.f;
    {
      const uint32_t l = tile * 32 + lane;
      if (l < p.nlines) {
        if constexpr (EPI == EPI_ACCUM) {
          v_in = p.y[l];
        } else {
          v_in = (p.v_src ? p.v_src : p.v)[l];
          th_in = (p.theta_src ? p.theta_src : p.theta)[l];
        }
      }
    }
    for (uint32_t c = 0; c < nch; ++c) {
      if (!mbar_wait(&bars[wid][c_slot], c_phase)) {
        ok = false;
        break;
      }
      const unsigned char* st = ring + c_slot * kStageBytes;
      const unsigned char* irow = st + lane * kIdxRow;
      const unsigned char* wrow = st + kIdxBox + lane * kWRow;
      const uint32_t cnt = min((uint32_t)kChunk, L - c * kChunk);
      // Gathers and products are independent of the add chain: issue them
      // first -- all kChunk of them for spike operands (shared-memory
      // lookups), 8 at a time for dense x (where the add chain then overlaps
      // the next group's L1 gathers; measured faster).  Entries past the row
      // end (and rows past the last line) were zero-filled by the TMA box
      // (column 0, weight 0), so their gathers stay in bounds; only their
      // adds are skipped.
#ifndef SPARSL_ELL_DENSE_GATHER_ALL
#define SPARSL_ELL_DENSE_GATHER_ALL 0
#endif
      constexpr bool kGatherAll = XM != X_DENSE || SPARSL_ELL_DENSE_GATHER_ALL;
      float prod[kChunk];
#pragma unroll
      for (uint32_t g = 0; g < kChunk / 8; ++g) {  // 8 entries per group
        const uint4 ca = *reinterpret_cast<const uint4*>(irow + swz<kIdxRow>(lane, 2 * g));
        const uint4 cb = *reinterpret_cast<const uint4*>(irow + swz<kIdxRow>(lane, 2 * g + 1));
        float wv[8];
        if constexpr (WK == W_F32) {
          const float4 wa = *reinterpret_cast<const float4*>(wrow + swz<kWRow>(lane, 2 * g));
          const float4 wb = *reinterpret_cast<const float4*>(wrow + swz<kWRow>(lane, 2 * g + 1));
          wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
          wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
        } else {
          const uint4 h = *reinterpret_cast<const uint4*>(wrow + swz<kWRow>(lane, g));
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
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) {
          float xv;
          if constexpr (XM == X_DENSE) {
            xv = __ldg(p.x + cv[k]);
          } else {
            xv = spike_value<XM>(s_x, p.xbits, cv[k], gs);
          }
          prod[8 * g + k] = fmul(wv[k], xv);
        }
        if constexpr (!kGatherAll) {
          if (cnt >= 8 * g + 8) {
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) sum = fadd(sum, prod[8 * g + k]);
          } else {
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
              if (8 * g + k < cnt) sum = fadd(sum, prod[8 * g + k]);
          }
        }
      }
      if constexpr (kGatherAll) {
        if (cnt == (uint32_t)kChunk) {
#pragma unroll
          for (uint32_t k = 0; k < (uint32_t)kChunk; ++k) sum = fadd(sum, prod[k]);
        } else {
#pragma unroll
          for (uint32_t k = 0; k < (uint32_t)kChunk; ++k)
            if (k < cnt) sum = fadd(sum, prod[k]);
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      c_slot = (c_slot + 1 == nst) ? 0 : c_slot + 1;
      c_phase ^= (c_slot == 0);
      ++consumed;
      issue_next();
    }
    if (!ok) break;

    // Epilogue of one 32-row tile.
    const uint32_t row0 = tile * 32;
    const uint32_t line = row0 + lane;
    const bool valid = line < p.nlines;
    if constexpr (EPI == EPI_ACCUM) {
      if (valid) p.y[line] = fadd(v_in, sum);
    } else {
      bool spike = false;
      if (valid) {
        float vv = v_in;
        float th = th_in;
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
      const uint32_t ballot = __ballot_sync(0xffffffffu, spike);
      if (p.out_bits && lane == 0) {
        p.out_bits[tile] = ballot;
        // The word goes straight to every peer GPU over NVLink while the
        // tick streams on; no separate collective moves the spike vector.
        if (p.peer_out) {
          for (uint32_t r = 0; r < p.npeers; ++r) {
            uint32_t* q = p.peer_out[r];
            if (q) q[tile] = ballot;
          }
        }
        if (p.tick_count && ballot) atomicAdd(p.tick_count, (uint32_t)__popc(ballot));
      }
      if constexpr (COMPACT) {
        const uint32_t agg = __popc(ballot);
        const uint32_t excl = lookback_warp(p.tile_flags, tile, agg, p.epoch, p.err, lane);
        if (spike) p.idx_list[excl + __popc(ballot & ((1u << lane) - 1u))] = p.idx_base + line;
        if (lane == 0 && tile == ntiles - 1) *p.idx_count = excl + agg;
      }
    }
  }

  if (!ok) {
    if (lane == 0) set_err(p.err, DEVERR_LOOKBACK_TIMEOUT);
    // Let every copy still in flight land before the shared memory is released.
    for (; consumed < issued; ++consumed) {
      mbar_wait(&bars[wid][c_slot], c_phase);
      c_slot = (c_slot + 1 == nst) ? 0 : c_slot + 1;
      c_phase ^= (c_slot == 0);
    }
  }
  // Peer stores become visible system-wide before the warp is done, so the
  // exchange that follows the tick can publish them with one flag per peer.
  if (p.peer_out && lane == 0) __threadfence_system();
  // The last warp out rewinds the ticket counters for the next launch; the
  // epoch-tagged flags need no clearing.
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(p.tile_ticket + 1, 1u) == nwarps - 1) {
      atomicExch(p.tile_ticket, 0u);
      atomicExch(p.tile_ticket + 1, 0u);
    }
  }
}

// Shared-memory bytes of the spike operand for a launch.
struct XPlan {
  size_t bytes = 0;
  uint32_t gs = 0, sum_words = 0;
};

XPlan plan_x(const RowLaunch& p) {
  XPlan x;
  if (p.xmode == X_BITS_SMEM) {
    x.bytes = (size_t)p.xbits_words * 4;
  } else if (p.xmode == X_BITS_GLOBAL) {
    uint32_t gs = 3;
    while (gs < 31 && (((uint64_t)p.xbits_words + (1ull << gs) - 1) >> gs) > kSumMaxWords) ++gs;
    x.gs = gs;
    x.sum_words = (uint32_t)(((uint64_t)p.xbits_words + (1ull << gs) - 1) >> gs);
    x.bytes = (size_t)x.sum_words * 4;
  }
  x.bytes = (x.bytes + 15) & ~size_t(15);
  return x;
}

int g_num_sms = 0;

template <int WK, int XM, int EPI, bool COMPACT, int NW>
cudaError_t launch_nw(const EllMaps& m, const RowLaunch& p, cudaStream_t stream) {
  auto kern = ell_stream_kernel<WK, XM, EPI, COMPACT, NW>;
  const XPlan xp = plan_x(p);
  constexpr size_t kStage = WBox<WK>::kStage;
  // As many stages per warp as the shared memory left by the spike operand holds.
  size_t nst = (kSmemBudget - xp.bytes) / ((size_t)NW * kStage);
  nst = std::min<size_t>(std::max<size_t>(nst, kMinStages), XM == X_DENSE ? kDenseStages : kMaxStages);
  const size_t smem = 1024 + (size_t)NW * nst * kStage + xp.bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NW * 32, smem)) != cudaSuccess)
    return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  if constexpr (XM == X_DENSE) {
    // Dense x is gathered through L1: one CTA per SM, and a shared-memory
    // carveout just large enough for it, so the rest of the SM's L1/shared
    // storage caches x (a second CTA would squeeze that L1 to almost nothing).
    per_sm = 1;
    const int pct = (int)std::min<size_t>(100, (smem + 4096) * 100 / (228 * 1024) + 1);
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct)) != cudaSuccess)
      return e;
  }
  const uint32_t tiles = (p.nlines + 31) / 32;
  const uint32_t want = (tiles + NW - 1) / NW;
  const uint32_t grid = std::max(1u, std::min(want, (uint32_t)(per_sm * g_num_sms)));
  kern<<<grid, NW * 32, smem, stream>>>(*reinterpret_cast<const CUtensorMap*>(m.idx),
                                        *reinterpret_cast<const CUtensorMap*>(m.w), p, m.L, xp.gs, xp.sum_words,
                                        (uint32_t)nst);
  return cudaGetLastError();
}

// Warps per CTA.  Every warp streams whole 32-row tiles, so a launch lasts
// about (the most tiles any warp takes) x (one tile's time), and one tile's
// time grows with the warps sharing an SM's bandwidth.  When the spike vector
// is read through the summary (the large networks), the launch takes
// whichever of 12, 14 and 16 warps gives the smallest ceil(tiles / warps) x
// warps: a multi-GPU shard of 16,384 tiles runs 10 tiles on some of 1,776
// warps (an 8 % tail) but at most 8 on 2,072.  Measured at 32,768 tiles:
// 1.260 ms with 14 warps against 1.296 ms with 12.  Shorter launches keep 12:
// config 3's 8,192 tiles measured 1.6 % slower with 14 warps, and dense x's
// gathers want the L1 that more warps' stages would take.
#ifndef SPARSL_ELL_NW_CHOICE
#define SPARSL_ELL_NW_CHOICE 1
#endif

template <int WK, int XM, int EPI, bool COMPACT>
cudaError_t launch_t(const EllMaps& m, const RowLaunch& p, cudaStream_t stream) {
  if (!p.tile_ticket) return cudaErrorInvalidValue;
  cudaError_t e;
  if (!g_num_sms) {
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  }
  if constexpr (XM == X_BITS_GLOBAL && SPARSL_ELL_NW_CHOICE) {
    const uint64_t tiles = (p.nlines + 31) / 32;
    auto cost = [&](uint64_t nw) {
      const uint64_t w = nw * (uint64_t)g_num_sms;
      return (tiles + w - 1) / w * nw;
    };
    const uint64_t c12 = cost(12), c14 = cost(14), c16 = cost(16);
    if (c14 < c12 && c14 <= c16) return launch_nw<WK, XM, EPI, COMPACT, 14>(m, p, stream);
    if (c16 < c12 && c16 < c14) return launch_nw<WK, XM, EPI, COMPACT, 16>(m, p, stream);
    return launch_nw<WK, XM, EPI, COMPACT, 12>(m, p, stream);
  }
  return launch_nw<WK, XM, EPI, COMPACT, kEllWarps>(m, p, stream);
}

template <int WK>
cudaError_t dispatch(const EllMaps& m, const RowLaunch& p, cudaStream_t s) {
  const bool compact = p.idx_list != nullptr;
  if (p.epilogue == EPI_ACCUM) {
    switch (p.xmode) {
      case X_DENSE: return launch_t<WK, X_DENSE, EPI_ACCUM, false>(m, p, s);
      case X_BITS_SMEM: return launch_t<WK, X_BITS_SMEM, EPI_ACCUM, false>(m, p, s);
      default: return launch_t<WK, X_BITS_GLOBAL, EPI_ACCUM, false>(m, p, s);
    }
  }
  switch (p.xmode) {
    case X_DENSE: return launch_t<WK, X_DENSE, EPI_LIF, false>(m, p, s);
    case X_BITS_SMEM:
      return compact ? launch_t<WK, X_BITS_SMEM, EPI_LIF, true>(m, p, s)
                     : launch_t<WK, X_BITS_SMEM, EPI_LIF, false>(m, p, s);
    default:
      return compact ? launch_t<WK, X_BITS_GLOBAL, EPI_LIF, true>(m, p, s)
                     : launch_t<WK, X_BITS_GLOBAL, EPI_LIF, false>(m, p, s);
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
  cuuint32_t box[2] = {(cuuint32_t)kChunk, 32};
  cuuint32_t estr[2] = {1, 1};
  cuuint64_t istride[1] = {(cuuint64_t)L * 4};
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(m.idx), CU_TENSOR_MAP_DATA_TYPE_UINT32, 2,
                   const_cast<uint32_t*>(col), dims, istride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_mode<kIdxRow>(), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  cuuint64_t wstride[1] = {(cuuint64_t)L * wbytes};
  r = enc(reinterpret_cast<CUtensorMap*>(m.w),
          wkind == W_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w),
          dims, wstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          wkind == W_F32 ? swizzle_mode<WBox<W_F32>::kRow>() : swizzle_mode<WBox<W_F16>::kRow>(),
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  m.L = L;
  m.ok = true;
  return true;
}

cudaError_t launch_ell(const EllMaps& m, const RowLaunch& p, cudaStream_t stream) {
  if (p.nlines == 0) return cudaSuccess;
  switch (p.wkind) {
    case W_F16: return dispatch<W_F16>(m, p, stream);
    case W_BF16: return dispatch<W_BF16>(m, p, stream);
    default: return dispatch<W_F32>(m, p, stream);
  }
}

}  // namespace sparsl
