// Exact inclusive scan over affine maps, bit-identical to the sequential fold.
//
// The reference's CPU arms are a strict left fold (src/scan.rs:298-313):
//   acc = x[0]; acc = (x.a * acc.a, x.a * acc.b + x.b) for every later x
// with two separate roundings.  That is a nonlinear recurrence in f32 and no
// reassociation reproduces it, so this kernel never reassociates the values it
// writes.  It parallelises the *search* for each sub-chunk's incoming state
// instead, and then proves every guess:
//
//  * Multiplier chain A (a' = x.a * a) -- made exact by construction.  Each
//    tile learns the exact A entering it (look-back, below) and one thread
//    walks its 256 sub-chunks: while A is a tiny denormal m * 2^-149 with
//    m <= 7 it jumps a whole sub-chunk through that sub-chunk's exact transfer
//    table (m -> m'), otherwise it multiplies element by element.  Tables are
//    what make long decaying chains cheap: on [0.9, 1] multipliers the f32
//    chain sticks at a denormal fixed point (m * 2^-149, m <= 5) that only an
//    exact replay can predict.
//  * Offset chain B (b' = x.a * b + x.b) -- speculated.  A tree composition of
//    the preceding maps (decoupled look-back across tiles, block scan inside a
//    tile) gives a guess a few ulps off; each thread then replays the exact
//    recurrence over the 128 elements before its own 16, which contracts the
//    guess onto the sequential trajectory bit for bit in practice.
//  * Verify: each thread's assumed incoming state is compared bitwise with the
//    final state its predecessor actually produced.  If every adjacent pair
//    agrees, the whole output equals the sequential fold by induction.
//  * Repair: a second kernel walks forward from the first disagreement with
//    the exact recurrence, overwriting until the recomputed state equals the
//    stored one (after which the stored trajectory is exact again), then jumps
//    to the next recorded disagreement.  The worst case is a serial fold --
//    slower, never different.
//
// The first element is copied, never combined (src/scan.rs:280-286), so
// (inf, -0.0) survives bit for bit.  Every spin is bounded (kSpinLimit).
#include "common.cuh"
#include "scan.cuh"

namespace sparsl {
namespace {

constexpr int kRowStride = kScanK + 1;                      // padded float2 stride
constexpr int kRows = kScanHaloSub + kScanThreads;          // halo + tile rows
constexpr uint32_t kTabId = 0x76543210u;                    // identity table
constexpr uint32_t kNone = 0xffffffffu;

struct Aff {
  float a, b;
};

// Apply p, then q: (q.a * p.a, q.a * p.b + q.b) -- scan.rs:127-132 with the
// reference's operand order and two roundings.
__device__ __forceinline__ Aff comb(Aff p, Aff q) {
  return Aff{fmul(q.a, p.a), fadd(fmul(q.a, p.b), q.b)};
}

__device__ __forceinline__ uint32_t tab_at(uint32_t tab, uint32_t m) { return (tab >> (4 * m)) & 0xfu; }

// Transfer tables: nibble m holds the multiplier leaving a run of maps when
// m * 2^-149 entered it, or 8 when that output left the domain {0..7} * 2^-149.
// Composition (t1 first, then t2) propagates the invalid marker.
__device__ __forceinline__ uint32_t tab_comb(uint32_t t1, uint32_t t2) {
  uint32_t r = 0;
#pragma unroll
  for (uint32_t m = 0; m < 8; ++m) {
    const uint32_t e = tab_at(t1, m);
    r |= ((e & 8u) ? 8u : tab_at(t2, e)) << (4 * m);
  }
  return r;
}

__device__ __forceinline__ bool in_domain(float a) { return __float_as_uint(a) <= 7u; }

__device__ __forceinline__ bool same_bits(Aff x, Aff y) {
  return __float_as_uint(x.a) == __float_as_uint(y.a) && __float_as_uint(x.b) == __float_as_uint(y.b);
}

__device__ __forceinline__ void stamp(const ScanScratch& s, uint32_t tile, int k) {
  if (s.timeline && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    s.timeline[(uint64_t)tile * 16 + k] = t;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_main(const float2* __restrict__ in,
                                                         float2* __restrict__ out, uint64_t n,
                                                         ScanScratch s, uint32_t* err) {
  extern __shared__ __align__(16) float2 sm[];  // kRows x kRowStride
  __shared__ float s_Ea[kScanThreads], s_Eb[kScanThreads];
  __shared__ uint32_t s_Et[kScanThreads], s_tab[kScanThreads];
  __shared__ float s_Ain[kScanThreads + 1];
  __shared__ float s_fa[kScanThreads], s_fb[kScanThreads];
  __shared__ float s_wa[8], s_wb[8];
  __shared__ uint32_t s_wt[8];
  __shared__ float s_P[4];        // P_full (a, b), P_head (a, b)
  __shared__ float s_AG[4];       // tile aggregate full, head
  __shared__ uint32_t s_TG[1];    // tile transfer table
  __shared__ float s_Atin;
  __shared__ uint32_t s_tile, s_last, s_incl;

  const int t = threadIdx.x;
  const int lane = t & 31;
  const int wid = t >> 5;
  const uint64_t ntiles = (n + kScanTile - 1) / kScanTile;

  if (t == 0) s_tile = atomicAdd(s.ticket, 1u);
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint64_t tile_start = (uint64_t)tile * kScanTile;
  stamp(s, tile, 0);

  // ---- 1. stage halo + tile into padded shared memory (identity past n) ----
  {
    // All loads first, then all shared stores, so every thread keeps its
    // whole share of the tile in flight at once.
    constexpr int kPer = (kScanHalo + kScanTile) / kScanThreads;
    static_assert((kScanHalo + kScanTile) % kScanThreads == 0, "tile staging");
    float2 v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int li = t + i * kScanThreads;
      const int64_t g = (int64_t)tile_start - kScanHalo + li;
      v[i] = make_float2(1.0f, 0.0f);
      if (g >= 0 && (uint64_t)g < n) v[i] = __ldg(in + g);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int li = t + i * kScanThreads;
      sm[(li / kScanK) * kRowStride + (li % kScanK)] = v[i];
    }
  }
  __syncthreads();
  stamp(s, tile, 1);

  const float2* row = sm + (t + kScanHaloSub) * kRowStride;

  // ---- 2. sub-chunk aggregate (tree guess input) and multiplier table ----
  Aff agg{row[0].x, row[0].y};
#pragma unroll
  for (int j = 1; j < kScanK; ++j) agg = comb(agg, Aff{row[j].x, row[j].y});
  uint32_t tab = 0;
#pragma unroll
  for (uint32_t m = 0; m < 8; ++m) {
    float v = __uint_as_float(m);
#pragma unroll
    for (int j = 0; j < kScanK; ++j) v = fmul(row[j].x, v);
    const uint32_t b = __float_as_uint(v);
    tab |= (b <= 7u ? b : 8u) << (4 * m);
  }
  s_tab[t] = tab;

  // ---- 3. block scan: exclusive in-tile prefix of maps and of tables ----
  Aff inc = agg;
  uint32_t tinc = tab;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const Aff o = Aff{__shfl_up_sync(0xffffffffu, inc.a, d), __shfl_up_sync(0xffffffffu, inc.b, d)};
    const uint32_t to = __shfl_up_sync(0xffffffffu, tinc, d);
    if (lane >= d) {
      inc = comb(o, inc);
      tinc = tab_comb(to, tinc);
    }
  }
  if (lane == 31) {
    s_wa[wid] = inc.a;
    s_wb[wid] = inc.b;
    s_wt[wid] = tinc;
  }
  __syncthreads();
  Aff wpre{1.0f, 0.0f};
  uint32_t wtab = kTabId;
  bool have_wpre = false;
  for (int w2 = 0; w2 < wid; ++w2) {
    const Aff o{s_wa[w2], s_wb[w2]};
    wpre = have_wpre ? comb(wpre, o) : o;
    have_wpre = true;
    wtab = tab_comb(wtab, s_wt[w2]);
  }
  if (have_wpre) {
    inc = comb(wpre, inc);
    tinc = tab_comb(wtab, tinc);
  }
  {
    Aff ex = Aff{__shfl_up_sync(0xffffffffu, inc.a, 1), __shfl_up_sync(0xffffffffu, inc.b, 1)};
    uint32_t tex = __shfl_up_sync(0xffffffffu, tinc, 1);
    if (lane == 0) {
      ex = wpre;  // identity (1, 0) for t == 0
      tex = wtab;
    }
    s_Ea[t] = ex.a;
    s_Eb[t] = ex.b;
    s_Et[t] = tex;
  }
  if (t == kScanThreads - 1) {
    s_AG[0] = inc.a;
    s_AG[1] = inc.b;
    s_TG[0] = tinc;
  }
  if (t == kScanThreads - 1 - kScanHaloSub) {
    s_AG[2] = inc.a;
    s_AG[3] = inc.b;
  }
  __syncthreads();

  stamp(s, tile, 2);
  // ---- 4. publish the aggregate, 5. look back across tiles ----
  ScanTileRecord* rec = s.rec;
  if (t == 0) {
    ScanTileRecord* r = rec + tile;
    r->agg[0] = s_AG[0];
    r->agg[1] = s_AG[1];
    r->agg[2] = s_AG[2];
    r->agg[3] = s_AG[3];
    r->tab = s_TG[0];
    __threadfence();
    st_release_u32(&r->status, 1u);
  }
  if (tile > 0 && wid == 0) {
    // Warp-parallel look-back: lane k inspects tile (base - k).
    Aff Sf{1.f, 0.f}, Sh{1.f, 0.f};
    uint32_t St = kTabId;
    bool have = false;
    int64_t base = (int64_t)tile - 1;
    uint32_t spins = 0;
    bool done = false;
    Aff Pf{1.f, 0.f}, Ph{1.f, 0.f};
    float atin = 0.f;
    bool atin_ok = false;
    uint32_t windows = 0, lastL = 0;
    while (!done) {
      const int64_t j = base - lane;
      uint32_t stt = 0;
      if (j >= 0) stt = ld_acquire_u32(&rec[j].status);
      const uint32_t incl_mask = __ballot_sync(0xffffffffu, stt == 2u);
      // Tile 0 has no predecessor, so the walk may only stop there, never
      // pass through it: it counts as ready once it is inclusive.
      const uint32_t ready_mask = __ballot_sync(0xffffffffu, stt == 2u || (stt == 1u && j > 0));
      const int L = incl_mask ? (__ffs(incl_mask) - 1) : 32;
      const uint32_t need = (L == 32) ? 0xffffffffu : ((1u << L) - 1u) | (1u << L);
      if ((ready_mask & need) != need) {
        if (++spins > kSpinLimit) {
          set_err(err, DEVERR_LOOKBACK_TIMEOUT);
          if (lane == 0 && atomicCAS(s.repair_stats + 2, 0u, 1u) == 0u) {
            s.repair_stats[3] = tile;
            s.repair_stats[4] = (uint32_t)base;
            s.repair_stats[5] = (uint32_t)L;
            s.repair_stats[6] = ready_mask;
            s.repair_stats[7] = incl_mask;
            s.repair_stats[8] = s.ticket[0];
            s.repair_stats[9] = s.ticket[1];
          }
          break;
        }
        __nanosleep(32);
        continue;
      }
      ++windows;
      lastL = (uint32_t)L;
      // Every lane <= L is published; fetch what the fold needs.
      float ga = 1.f, gb = 0.f, ha = 1.f, hb = 0.f, ia = 1.f, ib = 0.f, iha = 1.f, ihb = 0.f, av = 0.f;
      uint32_t tb = kTabId;
      if (lane <= L && j >= 0) {
        const ScanTileRecord* r = rec + j;
        ga = r->agg[0];
        gb = r->agg[1];
        ha = r->agg[2];
        hb = r->agg[3];
        tb = r->tab;
        if (lane == L) {
          ia = r->inc[0];
          ib = r->inc[1];
          iha = r->inc[2];
          ihb = r->inc[3];
          av = r->av;
        }
      }
      // Compose this window's aggregates (lanes 0..L-1, farther lanes first)
      // with a shuffle tree.  Lanes 1..L-1 are reduced together; lane 0 --
      // the nearest tile -- is applied last, with its head aggregate instead of
      // its full one on the head chain of the first window.
      {
        const bool mid = lane >= 1 && lane < L;
        Aff rf = mid ? Aff{ga, gb} : Aff{1.f, 0.f};
        uint32_t rt = mid ? tb : kTabId;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const Aff up{__shfl_down_sync(0xffffffffu, rf.a, d), __shfl_down_sync(0xffffffffu, rf.b, d)};
          const uint32_t ut = __shfl_down_sync(0xffffffffu, rt, d);
          if (lane + d < 32) {
            rf = comb(up, rf);
            rt = tab_comb(ut, rt);
          }
        }
        const Aff W1{__shfl_sync(0xffffffffu, rf.a, 0), __shfl_sync(0xffffffffu, rf.b, 0)};
        const uint32_t W1t = __shfl_sync(0xffffffffu, rt, 0);
        if (L > 0) {
          const Aff g0{__shfl_sync(0xffffffffu, ga, 0), __shfl_sync(0xffffffffu, gb, 0)};
          const Aff h0{__shfl_sync(0xffffffffu, ha, 0), __shfl_sync(0xffffffffu, hb, 0)};
          const uint32_t t0 = __shfl_sync(0xffffffffu, tb, 0);
          const Aff wf = comb(W1, g0);
          const uint32_t wt = tab_comb(W1t, t0);
          if (!have) {
            Sf = wf;
            Sh = comb(W1, h0);
            St = wt;
            have = true;
          } else {
            Sf = comb(wf, Sf);
            Sh = comb(wf, Sh);
            St = tab_comb(wt, St);
          }
        }
      }
      if (L < 32) {
        const Aff I{__shfl_sync(0xffffffffu, ia, L), __shfl_sync(0xffffffffu, ib, L)};
        const Aff IH{__shfl_sync(0xffffffffu, iha, L), __shfl_sync(0xffffffffu, ihb, L)};
        const float A = __shfl_sync(0xffffffffu, av, L);
        if (!have) {  // the nearest predecessor is inclusive
          Pf = I;
          Ph = IH;
          atin = A;
          atin_ok = true;
        } else {
          Pf = comb(I, Sf);
          Ph = comb(I, Sh);
          if (in_domain(A)) {
            const uint32_t e = tab_at(St, __float_as_uint(A));
            if (!(e & 8u)) {
              atin = __uint_as_float(e);
              atin_ok = true;
            }
          }
        }
        done = true;
      }
      base -= 32;
    }
    // The exact multiplier entering this tile: if the tables could not carry
    // it, take it straight from the nearest predecessor once it is inclusive.
    if (s.timeline && lane == 0) {
      s.timeline[(uint64_t)tile * 16 + 11] = windows;
      s.timeline[(uint64_t)tile * 16 + 12] = lastL;
      s.timeline[(uint64_t)tile * 16 + 13] = atin_ok ? 1 : 0;
      s.timeline[(uint64_t)tile * 16 + 14] = spins;
    }
    if (!atin_ok) {
      uint32_t sp = 0;
      if (lane == 0) {
        while (ld_acquire_u32(&rec[tile - 1].status) != 2u) {
          if (++sp > kSpinLimit) {
            set_err(err, DEVERR_LOOKBACK_TIMEOUT);
            if (atomicCAS(s.repair_stats + 2, 0u, 2u) == 0u) {
              s.repair_stats[3] = tile;
              s.repair_stats[8] = s.ticket[0];
              s.repair_stats[9] = s.ticket[1];
            }
            break;
          }
          __nanosleep(32);
        }
        atin = rec[tile - 1].av;
      }
      atin = __shfl_sync(0xffffffffu, atin, 0);
    }
    if (lane == 0) {
      s_P[0] = Pf.a;
      s_P[1] = Pf.b;
      s_P[2] = Ph.a;
      s_P[3] = Ph.b;
      s_Atin = atin;
      // When the tables carry the multiplier across this tile, its inclusive
      // record is known now: publish it before the rest of the block catches
      // up, so successors' look-backs stop here sooner.
      s_incl = 0;
      if (in_domain(atin)) {
        const uint32_t e = tab_at(s_TG[0], __float_as_uint(atin));
        if (!(e & 8u)) {
          ScanTileRecord* r = rec + tile;
          const Aff f = comb(Pf, Aff{s_AG[0], s_AG[1]});
          const Aff h = comb(Pf, Aff{s_AG[2], s_AG[3]});
          r->inc[0] = f.a;
          r->inc[1] = f.b;
          r->inc[2] = h.a;
          r->inc[3] = h.b;
          r->av = __uint_as_float(e);
          __threadfence();
          st_release_u32(&r->status, 2u);
          s_incl = 1;
        }
      }
    }
  }
  __syncthreads();

  stamp(s, tile, 3);
  // ---- 6. exact multiplier at every sub-chunk boundary ----
  // Fast path: the multiplier entering the tile is in the table domain and
  // the tile's table keeps it there -- every prefix table then does too, and
  // each thread reads its own boundary value.
  const bool fast = tile > 0 && in_domain(s_Atin) &&
                    !(tab_at(s_TG[0], __float_as_uint(s_Atin)) & 8u);
  if (fast) {
    s_Ain[t] = __uint_as_float(tab_at(s_Et[t], __float_as_uint(s_Atin)));
    if (t == kScanThreads - 1) s_Ain[kScanThreads] = __uint_as_float(tab_at(s_TG[0], __float_as_uint(s_Atin)));
  } else if (t == 0) {
    // Hybrid walk: jump a sub-chunk through its table while the multiplier is
    // in the domain and the entry is valid, multiply element by element
    // otherwise.  Either way the value is the sequential one.
    float A;
    int first;
    if (tile == 0) {
      A = sm[kScanHaloSub * kRowStride].x;  // x[0] is copied, not combined
      s_Ain[0] = A;                          // unused: element 0 is copied
      for (int j = 1; j < kScanK; ++j) A = fmul(sm[kScanHaloSub * kRowStride + j].x, A);
      s_Ain[1] = A;
      first = 1;
    } else {
      A = s_Atin;
      s_Ain[0] = A;
      first = 0;
    }
    for (int c = first; c < kScanThreads; ++c) {
      bool jumped = false;
      if (in_domain(A)) {
        const uint32_t e = tab_at(s_tab[c], __float_as_uint(A));
        if (!(e & 8u)) {
          A = __uint_as_float(e);
          jumped = true;
        }
      }
      if (!jumped) {
        const float2* rc = sm + (c + kScanHaloSub) * kRowStride;
        for (int j = 0; j < kScanK; ++j) A = fmul(rc[j].x, A);
      }
      s_Ain[c + 1] = A;
    }
  }
  __syncthreads();

  // ---- 7. publish the inclusive record (guesses for B, exact A) ----
  if (t == 0 && !(tile > 0 && s_incl)) {
    ScanTileRecord* r = rec + tile;
    Aff f{s_AG[0], s_AG[1]}, h{s_AG[2], s_AG[3]};
    if (tile > 0) {
      const Aff P{s_P[0], s_P[1]};
      f = comb(P, f);
      h = comb(P, h);
    }
    r->inc[0] = f.a;
    r->inc[1] = f.b;
    r->inc[2] = h.a;
    r->inc[3] = h.b;
    r->av = s_Ain[kScanThreads];
    __threadfence();
    st_release_u32(&r->status, 2u);
  }

  stamp(s, tile, 4);
  // ---- 8. warm-up: replay the elements before this sub-chunk ----
  // In-tile threads replay the 128 elements before their sub-chunk from the
  // block-scan guess; the first threads of a tile replay the 256-element halo
  // from the look-back guess, so a tile's entry state is very rarely wrong.
  const uint64_t start_t = tile_start + (uint64_t)t * kScanK;
  Aff st;
  int wrow0;  // first shared-memory row replayed
  int wcol0 = 0;
  if (tile == 0) {
    if (t <= kScanWarmSub) {
      st = Aff{sm[kScanHaloSub * kRowStride].x, sm[kScanHaloSub * kRowStride].y};  // exact start
      wrow0 = kScanHaloSub;
      wcol0 = 1;
    } else {
      st = Aff{s_Ea[t - kScanWarmSub], s_Eb[t - kScanWarmSub]};
      wrow0 = t - kScanWarmSub + kScanHaloSub;
    }
  } else if (t < kScanWarmSub) {
    st = Aff{s_P[2], s_P[3]};
    wrow0 = 0;
  } else {
    st = comb(Aff{s_P[0], s_P[1]}, Aff{s_Ea[t - kScanWarmSub], s_Eb[t - kScanWarmSub]});
    if (t == kScanWarmSub) st = Aff{s_P[0], s_P[1]};  // empty in-tile prefix
    wrow0 = t - kScanWarmSub + kScanHaloSub;
  }
  const bool copy_first = (tile == 0 && t == 0);
  if (!copy_first) {
    for (int r = wrow0; r < t + kScanHaloSub; ++r) {
      const float2* rr = sm + r * kRowStride;
      for (int j = (r == wrow0 ? wcol0 : 0); j < kScanK; ++j) st = comb(st, Aff{rr[j].x, rr[j].y});
    }
    st.a = s_Ain[t];  // the multiplier is exact by construction
  }
  const Aff assumed = st;
  __syncthreads();  // every warm-up read is done before rows are overwritten

  // ---- 9. own sub-chunk, written in place ----
  float2* wrow = sm + (t + kScanHaloSub) * kRowStride;
  int j0 = 0;
  if (copy_first) {
    st = Aff{wrow[0].x, wrow[0].y};
    j0 = 1;
  }
  for (int j = j0; j < kScanK; ++j) {
    st = comb(st, Aff{wrow[j].x, wrow[j].y});
    wrow[j] = make_float2(st.a, st.b);
  }
  s_fa[t] = st.a;
  s_fb[t] = st.b;
  __syncthreads();

  stamp(s, tile, 5);
  // ---- 9b. in-tile relaxation ----
  // A thread whose assumed entry state differs from its predecessor's final
  // state replays its sub-chunk from that final state (inputs re-read from
  // global memory; the tile's copy was overwritten).  Thread t is exact after
  // at most t rounds, so the loop ends; misses are rare, so it is usually one
  // round or none.  Only thread 0's entry state is left to the cross-tile check.
  Aff used = assumed;
  {
    bool stale = t > 0 && start_t < n && !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
    if (s.timeline) {
      const int cnt = __syncthreads_count(stale);
      // first stale thread, for the profiling timeline
      __shared__ int s_first;
      if (t == 0) s_first = 1 << 30;
      __syncthreads();
      if (stale) atomicMin(&s_first, t);
      __syncthreads();
      if (t == 0) {
        s.timeline[(uint64_t)tile * 16 + 8] = cnt;
        s.timeline[(uint64_t)tile * 16 + 10] = s_first;
      }
    }
    int rounds_done = 0;
    for (int round = 0; round < kScanThreads && __syncthreads_or(stale); ++round) {
      ++rounds_done;
      Aff fin{0.f, 0.f};
      if (stale) {
        used = Aff{s_fa[t - 1], s_fb[t - 1]};
        Aff r = used;
        for (int j = 0; j < kScanK; ++j) {
          if (start_t + j < n) {
            const float2 x = __ldg(in + start_t + j);
            r = comb(r, Aff{x.x, x.y});
          }
          wrow[j] = make_float2(r.a, r.b);
        }
        fin = r;
      }
      __syncthreads();
      if (stale) {
        s_fa[t] = fin.a;
        s_fb[t] = fin.b;
      }
      __syncthreads();
      stale = t > 0 && start_t < n && !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
    }
    if (s.timeline && t == 0) s.timeline[(uint64_t)tile * 16 + 9] = rounds_done;
  }

  stamp(s, tile, 6);
  // ---- 10. verify adjacent sub-chunks inside the tile ----
  bool mis = false;  // relaxation leaves none unless its round cap was hit
  if (t > 0 && start_t < n) mis = !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
  const uint32_t word = __ballot_sync(0xffffffffu, mis);
  if (lane == 0) {
    s.mis_bits[(uint64_t)tile * 8 + wid] = word;
    if (word) atomicOr(s.tile_bits + (tile >> 5), 1u << (tile & 31));
  }

  // ---- 11. coalesced store ----
  for (int li = t; li < kScanTile; li += kScanThreads) {
    const uint64_t g = tile_start + li;
    if (g < n) out[g] = sm[(kScanHaloSub + li / kScanK) * kRowStride + (li % kScanK)];
  }

  // ---- 12. tile-boundary check: whichever side arrives second compares ----
  if (t == 0) {
    if (tile > 0) {
      s.assumed[2 * (uint64_t)tile] = assumed.a;
      s.assumed[2 * (uint64_t)tile + 1] = assumed.b;
      __threadfence();
      if (atomicInc(s.arrive + tile, 1u) == 1u) {
        __threadfence();
        const Aff l{s.last[2 * (uint64_t)(tile - 1)], s.last[2 * (uint64_t)(tile - 1) + 1]};
        const bool bad = !same_bits(l, assumed);
        s.xmis[tile] = bad ? 1u : 0u;
        if (bad) atomicOr(s.tile_bits + (tile >> 5), 1u << (tile & 31));
      }
    }
    if ((uint64_t)tile + 1 < ntiles) {
      const Aff fin{s_fa[kScanThreads - 1], s_fb[kScanThreads - 1]};
      s.last[2 * (uint64_t)tile] = fin.a;
      s.last[2 * (uint64_t)tile + 1] = fin.b;
      __threadfence();
      if (atomicInc(s.arrive + tile + 1, 1u) == 1u) {
        __threadfence();
        const uint32_t nt = tile + 1;
        const Aff as{s.assumed[2 * (uint64_t)nt], s.assumed[2 * (uint64_t)nt + 1]};
        const bool bad = !same_bits(fin, as);
        s.xmis[nt] = bad ? 1u : 0u;
        if (bad) atomicOr(s.tile_bits + (nt >> 5), 1u << (nt & 31));
      }
    }
    __threadfence();
    s_last = (atomicAdd(s.ticket + 1, 1u) == ntiles - 1) ? 1u : 0u;
  }
  __syncthreads();
  stamp(s, tile, 7);
  // ---- 13. the last tile to finish clears the look-back state ----
  if (s_last) {
    for (uint64_t i = t; i < ntiles; i += kScanThreads) rec[i].status = 0u;
    if (t == 0) {
      s.ticket[0] = 0;
      s.ticket[1] = 0;
    }
  }
}

// Single-block repair: walk each recorded disagreement forward with the exact
// recurrence until the stored trajectory is met again.
__global__ void __launch_bounds__(256) scan_repair(const float2* __restrict__ in, float2* __restrict__ out,
                                                   uint64_t n, ScanScratch s, uint32_t* err) {
  __shared__ uint32_t s_min;
  __shared__ unsigned long long s_sub;
  const uint32_t ntiles = (uint32_t)((n + kScanTile - 1) / kScanTile);
  const uint32_t nwords = (ntiles + 31) / 32;
  const int t = threadIdx.x;
  const int lane = t & 31;
  uint64_t cursor = 1;  // sub-chunk 0 is the copied start, always exact
  uint64_t repaired = 0, segments = 0;
  const uint64_t nsub = (n + kScanK - 1) / kScanK;

  while (cursor < nsub) {
    // Next tile at or after the cursor's tile with any disagreement.
    uint32_t ctile = (uint32_t)(cursor / kScanThreads);
    if (t == 0) s_sub = ~0ull;
    __syncthreads();
    while (true) {
      if (t == 0) s_min = kNone;
      __syncthreads();
      for (uint32_t w = (ctile >> 5) + t; w < nwords; w += blockDim.x) {
        uint32_t b = s.tile_bits[w];
        if (w == (ctile >> 5)) b &= ~((1u << (ctile & 31)) - 1u);
        if (b) atomicMin(&s_min, w * 32 + (__ffs(b) - 1));
      }
      __syncthreads();
      const uint32_t T = s_min;
      if (T == kNone) break;
      if (t == 0) {
        // First flagged sub-chunk of tile T at or after the cursor.
        uint64_t best = ~0ull;
        const uint64_t base = (uint64_t)T * kScanThreads;
        if (T > 0 && s.xmis[T] && base >= cursor) best = base;
        if (best == ~0ull) {
          for (int w = 0; w < 8 && best == ~0ull; ++w) {
            uint32_t b = s.mis_bits[(uint64_t)T * 8 + w];
            while (b) {
              const int bit = __ffs(b) - 1;
              const uint64_t sc = base + w * 32 + bit;
              if (sc >= cursor) {
                best = sc;
                break;
              }
              b &= b - 1;
            }
          }
        }
        s_sub = best;
      }
      __syncthreads();
      if (s_sub != ~0ull) break;
      ctile = T + 1;
      __syncthreads();
    }
    __syncthreads();
    const uint64_t sc = s_sub;
    if (sc == ~0ull) break;

    // Warp 0 replays from the start of sub-chunk sc.  All lanes carry the same
    // state; lane j owns element i + j of each 32-element batch.
    if (t < 32) {
      uint64_t i = sc * kScanK;
      const float2 p = out[i - 1];
      Aff stt{p.x, p.y};
      bool conv = false;
      uint64_t steps = 0;
      while (i < n && !conv) {
        const uint64_t gi = i + lane;
        float2 xv = make_float2(1.f, 0.f), ov = make_float2(0.f, 0.f);
        if (gi < n) {
          xv = in[gi];
          ov = out[gi];
        }
        float2 mine = ov;
        int upto = 32;
        for (int j = 0; j < 32; ++j) {
          if (i + j >= n) {
            upto = j;
            break;
          }
          const Aff x{__shfl_sync(0xffffffffu, xv.x, j), __shfl_sync(0xffffffffu, xv.y, j)};
          const Aff o{__shfl_sync(0xffffffffu, ov.x, j), __shfl_sync(0xffffffffu, ov.y, j)};
          stt = comb(stt, x);
          if (same_bits(stt, o)) {
            conv = true;
            upto = j;
            break;
          }
          if (lane == j) mine = make_float2(stt.a, stt.b);
        }
        if (lane < upto) out[gi] = mine;
        steps += upto;
        i += conv ? upto : 32;
      }
      repaired += steps;
      if (t == 0) s_sub = conv ? i : ~0ull;  // element where the stored trajectory was met
    }
    ++segments;
    __syncthreads();
    if (s_sub == ~0ull) break;
    cursor = s_sub / kScanK + 1;
    __syncthreads();
  }
  __syncthreads();
  for (uint32_t w = t; w < nwords; w += blockDim.x) s.tile_bits[w] = 0u;
  if (t == 0) {
    s.repair_stats[0] = (uint32_t)min(repaired, (uint64_t)0xffffffffu);
    s.repair_stats[1] = (uint32_t)min(segments, (uint64_t)0xffffffffu);
  }
}

}  // namespace

size_t scan_scratch_bytes(uint64_t n) {
  const uint64_t nt = (n + kScanTile - 1) / kScanTile + 1;
  size_t b = 0;
  b += nt * sizeof(ScanTileRecord);
  b += 64;                         // ticket
  b += nt * 4;                     // arrive
  b += nt * 8;                     // assumed
  b += nt * 8;                     // last
  b += nt * 8 * 4;                 // mis_bits
  b += nt * 4;                     // xmis
  b += ((nt + 31) / 32 + 1) * 4;   // tile_bits
  b += 64;                         // stats
  return b + 16 * 256;             // alignment slack
}

ScanScratch scan_scratch_carve(void* base, uint64_t n) {
  const uint64_t nt = (n + kScanTile - 1) / kScanTile + 1;
  uintptr_t p = reinterpret_cast<uintptr_t>(base);
  auto take = [&](size_t bytes) {
    p = (p + 255) & ~(uintptr_t)255;
    void* r = reinterpret_cast<void*>(p);
    p += bytes;
    return r;
  };
  ScanScratch s;
  s.rec = static_cast<ScanTileRecord*>(take(nt * sizeof(ScanTileRecord)));
  s.ticket = static_cast<uint32_t*>(take(64));
  s.arrive = static_cast<uint32_t*>(take(nt * 4));
  s.assumed = static_cast<float*>(take(nt * 8));
  s.last = static_cast<float*>(take(nt * 8));
  s.mis_bits = static_cast<uint32_t*>(take(nt * 8 * 4));
  s.xmis = static_cast<uint32_t*>(take(nt * 4));
  s.tile_bits = static_cast<uint32_t*>(take(((nt + 31) / 32 + 1) * 4));
  s.repair_stats = static_cast<uint32_t*>(take(64));
  return s;
}

cudaError_t launch_scan(const float* in, float* out, uint64_t n, const ScanScratch& s, uint32_t* err,
                        cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const uint64_t ntiles = (n + kScanTile - 1) / kScanTile;
  if (ntiles > 0x7fffffffull) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float2) * kRows * kRowStride;
  cudaError_t e = cudaFuncSetAttribute(scan_main, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  scan_main<<<(unsigned)ntiles, kScanThreads, smem, stream>>>(reinterpret_cast<const float2*>(in),
                                                              reinterpret_cast<float2*>(out), n, s, err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  scan_repair<<<1, 256, 0, stream>>>(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), n,
                                     s, err);
  return cudaGetLastError();
}

}  // namespace sparsl
