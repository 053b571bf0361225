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
//    sub-chunk warp composes its 32 transfer tables; a ninth warp per tile
//    composes the 8 warp tables and runs a decoupled look-back over one
//    64-bit word per tile: first the tile's transfer table (aggregate),
//    later the exact multiplier leaving it (inclusive).  Tables of aggregate tiles compose
//    exactly onto the nearest inclusive value, which gives the exact A
//    entering the tile; each sub-chunk's A then comes from its in-tile table
//    prefix.  A table maps m to the multiplier leaving a run of maps when
//    m * 2^-149 (m <= 7) entered it: on [0.9, 1] multipliers the f32 chain
//    sticks at such a denormal fixed point, which only an exact replay can
//    predict.  Outside that domain one thread multiplies element by element.
//  * Offset chain B (b' = x.a * b + x.b) -- speculated, with no look-back.
//    The recurrence contracts: B's dependence on its value n elements earlier
//    is a product of n multipliers.  So each thread replays the elements
//    before its sub-chunk (kScanWarmSub sub-chunks, 160 elements;
//    kScanT0Sub for a tile's thread 0) from a tree-composed guess that
//    assumes B = 0 at the start of the tile, or 32 sub-chunks before it for
//    the first warp (a halo of kScanHaloSub sub-chunks staged with the tile,
//    and before it the rest, which the look-back warp composes from global
//    memory); that assumption is contracted over at least 1,024 elements,
//    and the replay removes the tree's rounding.  For contracting data this lands on the sequential trajectory
//    bit for bit; the look-back warp works meanwhile.
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
#include <algorithm>

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
  // Nibbles 8..15 of the widened t2 are the invalid marker, so an invalid
  // entry of t1 (8) selects it.
  const unsigned long long t2x = (unsigned long long)t2 | 0x8888888800000000ull;
  uint32_t r = 0;
#pragma unroll
  for (uint32_t m = 0; m < 8; ++m) {
    const uint32_t e = tab_at(t1, m);
    r |= (uint32_t)((t2x >> (4 * e)) & 0xfull) << (4 * m);
  }
  return r;
}

__device__ __forceinline__ bool in_domain(float a) { return __float_as_uint(a) <= 7u; }

__device__ __forceinline__ bool same_bits(Aff x, Aff y) {
  return __float_as_uint(x.a) == __float_as_uint(y.a) && __float_as_uint(x.b) == __float_as_uint(y.b);
}

// Thread numbering of scan_main: the look-back warp is hardware warp 0
// (threads 256..287 here), sub-chunk thread t is hardware thread t + 32.  So
// the look-back warp and sub-chunk warp 0, which carries the halo, run on
// different SM sub-partitions (warp id mod 4).
__device__ __forceinline__ int scan_tid() { return (threadIdx.x + kScanBlock - 32) % kScanBlock; }

__device__ __forceinline__ void stamp(const ScanScratch& s, uint32_t tile, int k) {
  if (s.timeline && scan_tid() == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    s.timeline[(uint64_t)tile * 16 + k] = t;
  }
}

constexpr unsigned long long kStAgg = 1ull << 32;   // payload: the tile's transfer table
constexpr unsigned long long kStIncl = 2ull << 32;  // payload: bits of the exact multiplier leaving the tile

__device__ __forceinline__ uint32_t fbits(float x) { return __float_as_uint(x); }

// 8-byte asynchronous global -> shared copy (cached in L1 on the way).
__device__ __forceinline__ void cp_async8(float2* dst, const float2* src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(src) : "memory");
}

// Two f32 lanes in one 64-bit register (lo = first), and their lane-wise
// product: mul.rn.f32x2 rounds each product to nearest and keeps subnormals,
// exactly as two separate fmul.rn.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ unsigned long long fmul2(unsigned long long x, unsigned long long y) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  return r;
}

// One thread walks the exact multiplier across a tile's 256 sub-chunks from
// A (the multiplier entering sub-chunk `first`): it jumps a sub-chunk through
// its transfer table while A is a tiny denormal the table carries, and
// multiplies element by element otherwise.  Either way the values are the
// sequential ones.  Writes s_Ain[first + 1 .. kScanThreads].
__device__ void walk_multiplier(float A, int first, const float2* sm, const uint32_t* s_tab, float* s_Ain) {
  for (int c = first; c < kScanThreads; ++c) {
    bool jumped = false;
    if (in_domain(A)) {
      const uint32_t e = tab_at(s_tab[c], fbits(A));
      if (!(e & 8u)) {
        A = __uint_as_float(e);
        jumped = true;
      }
    }
    if (!jumped) {
      const float2* rc = sm + (c + kScanHaloSub) * kRowStride;
#pragma unroll
      for (int j = 0; j < kScanK; ++j) A = fmul(rc[j].x, A);
    }
    s_Ain[c + 1] = A;
  }
}

// Three tiles per SM: a tile (16 sub-chunk rows of halo + 256 of tile, 32
// maps each, padded) takes 70 KB of dynamic shared memory, and 72 registers
// per thread.
#ifndef SPARSL_SCAN_MIN_BLOCKS
#define SPARSL_SCAN_MIN_BLOCKS 3
#endif
__global__ void __launch_bounds__(kScanBlock, SPARSL_SCAN_MIN_BLOCKS) scan_main(const float2* __restrict__ in, float2* __restrict__ out,
                                                       uint64_t n, ScanScratch s, uint32_t* err, int has_entry,
                                                       float2 entry, const float2* entry_dev) {
  extern __shared__ __align__(16) float2 sm[];  // kRows x kRowStride
  // s_Eb (phases 2-3) shares words with s_fa (phases 4-6); s_tab (phases
  // 2-3) with s_fb (phases 4-6): each pair is separated by the barrier that
  // ends phase 3.
  __shared__ float s_u1[kScanThreads];
  __shared__ uint32_t s_u2[kScanThreads];
  float* const s_Eb = s_u1;    // in-tile exclusive guess of B (from identity)
  uint32_t* const s_tab = s_u2;
  __shared__ uint32_t s_tabx[kScanThreads];  // in-warp exclusive prefix of the tables
  __shared__ uint32_t s_wtab[8];             // each warp's composed table
  __shared__ uint32_t s_Awarp[8];            // fast path: multiplier entering each warp (m of m * 2^-149)
  __shared__ int s_fast;
  __shared__ float s_outb;  // B after the outer sub-chunks (before the halo), from B = 0
  __shared__ float s_Ain[kScanThreads + 1];
  float* const s_fa = s_u1;
  float* const s_fb = reinterpret_cast<float*>(s_u2);
  __shared__ float s_wa[8], s_wb[8];
  __shared__ float s_wb0;  // thread 0's warmed-up entry B
  __shared__ uint32_t s_tile;

  const int t = scan_tid();
  const int lane = t & 31;
  const int wid = t >> 5;
  const bool lb_warp = wid == kScanThreads / 32;  // the look-back warp
  const uint64_t ntiles = (n + kScanTile - 1) / kScanTile;

  if (t == 0) s_tile = atomicAdd(s.ticket, 1u);
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint64_t tile_start = (uint64_t)tile * kScanTile;
  stamp(s, tile, 0);

  // ---- 1. stage halo + tile into padded shared memory (identity outside [0, n)) ----
  // Sub-chunks before the halo that the look-back warp composes from global
  // memory, so that warp 0's guesses assume B = 0 32 sub-chunks before the
  // tile, as far back as a full-length halo would.
  constexpr int kOuterSub = 32 - kScanHaloSub;
  float2 ov[kOuterSub > 0 ? kOuterSub : 1];
  {
    // The look-back warp issues its reads of the outer sub-chunks first
    // (lane k: kOuterSub consecutive maps).
    if (kOuterSub > 0 && lb_warp) {
#pragma unroll
      for (int i = 0; i < kOuterSub; ++i) {
        const int64_t g = (int64_t)tile_start - kScanHalo - kOuterSub * 32 + lane * kOuterSub + i;
        ov[i] = (g >= 0 && (uint64_t)g < n) ? __ldg(in + g) : make_float2(1.0f, 0.0f);
      }
    }
    // Asynchronous 8-byte copies straight into the padded rows: every load
    // of the tile is in flight at once and none holds a register.
    constexpr int kStage = kScanHalo + kScanTile;
    constexpr int kPer = (kStage + kScanBlock - 1) / kScanBlock;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int li = t + i * kScanBlock;
      if (kStage % kScanBlock == 0 || li < kStage) {
        const int64_t g = (int64_t)tile_start - kScanHalo + li;
        float2* dst = sm + (li / kScanK) * kRowStride + (li % kScanK);
        if (g >= 0 && (uint64_t)g < n)
          cp_async8(dst, in + g);
        else
          *dst = make_float2(1.0f, 0.0f);
      }
    }
    if (kOuterSub > 0 && lb_warp) {
      // The outer sub-chunks composed in order (lane k's maps, then a warp
      // scan); warp 0's guesses continue from their B.
      Aff o{ov[0].x, ov[0].y};
#pragma unroll
      for (int i = 1; i < kOuterSub; ++i) o = comb(o, Aff{ov[i].x, ov[i].y});
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const Aff u = Aff{__shfl_up_sync(0xffffffffu, o.a, d), __shfl_up_sync(0xffffffffu, o.b, d)};
        if (lane >= d) o = comb(u, o);
      }
      if (lane == 31) s_outb = o.b;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // A run that continues a longer sequence: its first map is the entry
    // state combined with x[0], exactly as the fold combines it; the
    // copy-first rule then emits it unchanged.  The thread that staged x[0]
    // patches it.
    if (has_entry && tile == 0 && t == kScanHalo % kScanBlock) {
      float2* f = sm + (kScanHalo / kScanK) * kRowStride + (kScanHalo % kScanK);
      const float2 en = entry_dev ? *entry_dev : entry;
      const Aff e = comb(Aff{en.x, en.y}, Aff{f->x, f->y});
      *f = make_float2(e.a, e.b);
    }
  }
  __syncthreads();
  stamp(s, tile, 1);

  // ---- 2. sub-chunk aggregates (guesses) and multiplier tables; block scan
  //         of the guesses (the look-back warp composes the tables) ----
  Aff inc{1.f, 0.f};
  float w0_guess = 0.f;  // warp 0: guessed B at the start of its warm-up
  if (!lb_warp) {
    const float2* row = sm + (t + kScanHaloSub) * kRowStride;
    // The sub-chunk's transfer table first: the look-back warp waits for it.
    // Entries m and m + 1 ride in one packed multiply (two separate f32
    // products, rounded to nearest, subnormals kept).
    uint32_t tab = 0;
    {
      unsigned long long v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = pack2(__uint_as_float(2 * i), __uint_as_float(2 * i + 1));
#pragma unroll
      for (int j = 0; j < kScanK; ++j) {
        const unsigned long long xx = pack2(row[j].x, row[j].x);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = fmul2(xx, v[i]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t b0 = (uint32_t)v[i], b1 = (uint32_t)(v[i] >> 32);
        tab |= (b0 <= 7u ? b0 : 8u) << (8 * i);
        tab |= (b1 <= 7u ? b1 : 8u) << (8 * i + 4);
      }
    }
    s_tab[t] = tab;
    // Compose the warp's 32 tables now, so that the look-back warp only
    // composes 8 and publishes the tile's table early.
    uint32_t itab = tab;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, itab, d);
      if (lane >= d) itab = tab_comb(o, itab);
    }
    const uint32_t xtab = __shfl_up_sync(0xffffffffu, itab, 1);
    s_tabx[t] = lane == 0 ? kTabId : xtab;
    if (lane == 31) s_wtab[wid] = itab;
    asm volatile("bar.arrive 3, %0;" ::"n"(kScanBlock) : "memory");
    Aff agg{row[0].x, row[0].y};
#pragma unroll
    for (int j = 1; j < kScanK; ++j) agg = comb(agg, Aff{row[j].x, row[j].y});
    inc = agg;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const Aff o = Aff{__shfl_up_sync(0xffffffffu, inc.a, d), __shfl_up_sync(0xffffffffu, inc.b, d)};
      if (lane >= d) inc = comb(o, inc);
    }
    if (lane == 31) {
      s_wa[wid] = inc.a;
      s_wb[wid] = inc.b;
    }
    if (wid == 0) {  // warp 0's exclusive guesses need no other warp
      Aff ex{__shfl_up_sync(0xffffffffu, inc.a, 1), __shfl_up_sync(0xffffffffu, inc.b, 1)};
      if (lane == 0) ex = Aff{1.f, 0.f};
      s_Eb[t] = ex.b;
      // Warp 0's warm-up guesses reach into the halo: lane t < H composes
      // halo sub-chunk t, a warp scan chains them (from the look-back warp's
      // B before the halo), and the halo total continues into the in-tile
      // prefix.
      Aff h{1.f, 0.f};
      if (lane < kScanHaloSub) {
        const float2* hrow = sm + lane * kRowStride;
        h = Aff{hrow[0].x, hrow[0].y};
#pragma unroll
        for (int j = 1; j < kScanK; ++j) h = comb(h, Aff{hrow[j].x, hrow[j].y});
      }
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const Aff o = Aff{__shfl_up_sync(0xffffffffu, h.a, d), __shfl_up_sync(0xffffffffu, h.b, d)};
        if (lane >= d) h = comb(o, h);
      }
      const float ob = kOuterSub > 0 ? s_outb : 0.f;  // B entering the halo, from B = 0 at the outer start
      h.b = fadd(fmul(h.a, ob), h.b);
      const Aff htot{__shfl_sync(0xffffffffu, h.a, 31), __shfl_sync(0xffffffffu, h.b, 31)};
      // Lane t's warm-up starts at row t + H - W (H = kScanHaloSub, W =
      // kScanWarmSub); lane 0 starts at halo row H - kScanT0Sub.  Lanes
      // 1 .. W-1 start in the halo: the prefix through halo row t + H - 1 - W.
      // The others start in the tile: the halo total, then lane t - W's
      // in-tile exclusive prefix.
      constexpr int W = kScanWarmSub;
      constexpr int H = kScanHaloSub;
      static_assert(W >= 1 && W <= H, "warp 0 warm-up guesses");
      const float hb = __shfl_sync(0xffffffffu, h.b, lane == 0 ? H - kScanT0Sub - 1 : (lane + H - 1 - W) & 31);
      const Aff exw{__shfl_sync(0xffffffffu, ex.a, (lane + 32 - W) & 31),
                    __shfl_sync(0xffffffffu, ex.b, (lane + 32 - W) & 31)};
      w0_guess = lane < W ? hb : comb(htot, exw).b;
    }
  }
  // Warp 0's warm-up needs nothing from the block scan: it only signals the
  // barrier and starts at once, and so does the look-back warp, which waits
  // for the warps' tables instead.  The other warps finish the block scan.
  if (wid == 0 || lb_warp) {
    asm volatile("bar.arrive 1, %0;" ::"n"(kScanBlock) : "memory");
    if (lb_warp) asm volatile("bar.sync 3, %0;" ::"n"(kScanBlock) : "memory");
  } else {
    asm volatile("bar.sync 1, %0;" ::"n"(kScanBlock) : "memory");
    Aff wpre{s_wa[0], s_wb[0]};
    for (int w2 = 1; w2 < wid; ++w2) wpre = comb(wpre, Aff{s_wa[w2], s_wb[w2]});
    inc = comb(wpre, inc);
    float exb = __shfl_up_sync(0xffffffffu, inc.b, 1);
    if (lane == 0) exb = wpre.b;
    s_Eb[t] = exb;
    asm volatile("bar.sync 2, %0;" ::"n"(kScanThreads - 32) : "memory");
  }
  stamp(s, tile, 2);

  // ---- 3. at the same time: the look-back warp finds the exact multiplier
  //         entering every sub-chunk, and the sub-chunk threads warm up B ----
  const bool copy_first = (tile == 0 && t == 0);
  float wb = 0.f;  // the warmed-up B entering this thread's sub-chunk
  if (lb_warp) {
    if (tile == 0) {
      // The chain starts at x[0], which is copied, not combined.
      if (lane == 0) {
        const float2* r0 = sm + kScanHaloSub * kRowStride;
        float A = r0[0].x;
        s_Ain[0] = A;  // unused: element 0 is copied
        for (int j = 1; j < kScanK; ++j) A = fmul(r0[j].x, A);
        s_Ain[1] = A;
        walk_multiplier(A, 1, sm, s_tab, s_Ain);
        st_relaxed_u64(s.flags, kStIncl | fbits(s_Ain[kScanThreads]));
        s_fast = 0;
      }
    } else {
      // Lane w < 8 holds warp w's composed table; a scan over the 8 lanes
      // gives each its entry table (ext) and lane 7 the tile's table.
      uint32_t it = lane < 8 ? s_wtab[lane] : kTabId;
#pragma unroll
      for (int d = 1; d < 8; d <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, it, d);
        if (lane >= d) it = tab_comb(o, it);
      }
      const uint32_t TG = __shfl_sync(0xffffffffu, it, 7);
      uint32_t ext = __shfl_up_sync(0xffffffffu, it, 1);
      if (lane == 0) ext = kTabId;
      if (lane == 0) st_relaxed_u64(s.flags + tile, kStAgg | TG);
      // Warp-parallel look-back: lane k inspects tile base - 1 - k.  Tables of
      // aggregate tiles compose (farther tiles first) until an inclusive word
      // gives the exact multiplier leaving some earlier tile.
      uint32_t C = kTabId;
      uint32_t pay = 0, windows = 0, spins = 0;
      bool direct = false, timed_out = false;
      int64_t base = tile;
      while (true) {
        const int64_t j = base - 1 - lane;
        uint32_t st = 0, py = 0;
        if (j >= 0) {
          const unsigned long long f = ld_relaxed_u64(s.flags + j);
          st = (uint32_t)(f >> 32) & 3u;
          py = (uint32_t)f;
        }
        const uint32_t incl = __ballot_sync(0xffffffffu, st == 2u);
        const uint32_t ready = __ballot_sync(0xffffffffu, st != 0u);
        const uint32_t upto = incl ? (((incl & (0u - incl)) << 1) - 1u) : 0xffffffffu;
        if ((ready & upto) != upto) {
          if (++spins > kSpinLimit) {
            timed_out = true;
            break;
          }
          __nanosleep(32);
          continue;
        }
        const int L = incl ? (__ffs(incl) - 1) : 32;
        uint32_t rt = lane < L ? py : kTabId;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const uint32_t ut = __shfl_down_sync(0xffffffffu, rt, d);
          if (lane + d < 32) rt = tab_comb(ut, rt);
        }
        C = tab_comb(__shfl_sync(0xffffffffu, rt, 0), C);
        ++windows;
        if (L < 32) {
          pay = __shfl_sync(0xffffffffu, py, L);
          direct = windows == 1 && L == 0;
          break;
        }
        base -= 32;
      }
      // The exact multiplier entering the tile.
      float Aent = 0.f;
      bool ok = !timed_out;
      if (ok) {
        if (direct) {
          Aent = __uint_as_float(pay);
        } else if (pay <= 7u && !(tab_at(C, pay) & 8u)) {
          Aent = __uint_as_float(tab_at(C, pay));
        } else {
          // The tables cannot carry it: wait for the nearest predecessor's
          // inclusive word.
          uint32_t sp = 0, v = 0;
          bool got = false;
          if (lane == 0) {
            while (true) {
              const unsigned long long f = ld_relaxed_u64(s.flags + tile - 1);
              if (((f >> 32) & 3u) == 2u) {
                v = (uint32_t)f;
                got = true;
                break;
              }
              if (++sp > kSpinLimit) break;
              __nanosleep(32);
            }
          }
          ok = __shfl_sync(0xffffffffu, got, 0);
          Aent = __uint_as_float(__shfl_sync(0xffffffffu, v, 0));
        }
      }
      if (!ok && lane == 0) set_err(err, DEVERR_LOOKBACK_TIMEOUT);
      const bool fast = ok && in_domain(Aent) && !(tab_at(TG, fbits(Aent)) & 8u);
      if (fast) {
        const uint32_t m = fbits(Aent);
        if (lane == 0) {
          st_relaxed_u64(s.flags + tile, kStIncl | tab_at(TG, m));  // successors stop here
          s_Ain[0] = Aent;
          s_Ain[kScanThreads] = __uint_as_float(tab_at(TG, m));
          s_fast = 1;
        }
        // Sub-chunk c of warp w enters with s_tabx[c] applied to s_Awarp[w].
        if (lane < 8) s_Awarp[lane] = tab_at(ext, m);
      } else if (lane == 0) {
        s_Ain[0] = Aent;
        walk_multiplier(Aent, 0, sm, s_tab, s_Ain);
        st_relaxed_u64(s.flags + tile, kStIncl | fbits(s_Ain[kScanThreads]));
        s_fast = 0;
      }
      if (s.timeline && lane == 0) {
        s.timeline[(uint64_t)tile * 16 + 11] = windows;
        s.timeline[(uint64_t)tile * 16 + 13] = fast ? 1 : 0;
        s.timeline[(uint64_t)tile * 16 + 14] = spins;
      }
    }
  } else if (!copy_first) {
    // Each thread replays the elements before its sub-chunk from a tree
    // guess that assumes B = 0 at the start of the tile (warps 1-7) or 32
    // sub-chunks before it (warp 0); by contraction over the replay and the
    // sub-chunks before it that no longer shows, and the replay removes the
    // tree's rounding.  Replays are kScanWarmSub sub-chunks, except thread
    // 0's, which only the cross-tile check (and a serial repair) would catch:
    // it replays kScanT0Sub.  In tile 0 the first element is copied, so warp
    // 0 starts there exactly.
    int r0;
    float b;
    if (wid == 0 && tile == 0) {
      const float2* rr = sm + kScanHaloSub * kRowStride;
      b = rr[0].y;
      for (int j = 1; j < kScanK; ++j) b = fadd(fmul(rr[j].x, b), rr[j].y);
      r0 = kScanHaloSub + 1;
    } else if (wid == 0) {
      b = w0_guess;
      r0 = t == 0 ? kScanHaloSub - kScanT0Sub : t + kScanHaloSub - kScanWarmSub;
    } else {
      b = s_Eb[t - kScanWarmSub];
      r0 = t - kScanWarmSub + kScanHaloSub;
    }
    for (int r = r0; r < t + kScanHaloSub; ++r) {
      const float2* rr = sm + r * kRowStride;
      float2 x[kScanK];
#pragma unroll
      for (int j = 0; j < kScanK; ++j) x[j] = rr[j];
#pragma unroll
      for (int j = 0; j < kScanK; ++j) b = fadd(fmul(x[j].x, b), x[j].y);
    }
    wb = b;
    if (t == 0) s_wb0 = b;
  }
  __syncthreads();  // every warm-up read is done before rows are overwritten
  stamp(s, tile, 3);

  // ---- 4. own sub-chunk, written in place ----
  const uint64_t start_t = tile_start + (uint64_t)t * kScanK;
  float2* wrow = sm + (t + kScanHaloSub) * kRowStride;
  Aff assumed{0.f, 0.f};
  if (!lb_warp) {
    float a, b;
    int j0 = 0;
    if (copy_first) {
      a = wrow[0].x;
      b = wrow[0].y;
      j0 = 1;
    } else {
      a = s_fast ? __uint_as_float(tab_at(s_tabx[t], s_Awarp[wid])) : s_Ain[t];  // exact by construction
      b = wb;
    }
    assumed = Aff{a, b};
    float2 x[kScanK];
#pragma unroll
    for (int j = 0; j < kScanK; ++j) x[j] = wrow[j];
#pragma unroll
    for (int j = 0; j < kScanK; ++j) {
      if (j < j0) continue;
      a = fmul(x[j].x, a);
      b = fadd(fmul(x[j].x, b), x[j].y);
      wrow[j] = make_float2(a, b);
    }
    s_fa[t] = a;
    s_fb[t] = b;
  } else if (lane == 0 && tile > 0) {
    // Cross-tile check, entry side: thread 0's assumed entry state (it is
    // never relaxed).  scan_check compares it with the predecessor's exit.
    s.assumed[2 * (uint64_t)tile] = s_Ain[0];
    s.assumed[2 * (uint64_t)tile + 1] = s_wb0;
  }
  __syncthreads();
  stamp(s, tile, 4);

  // ---- 5. in-tile relaxation ----
  // A thread whose assumed entry state differs from its predecessor's final
  // state replays its sub-chunk from that final state (inputs re-read from
  // global memory; the tile's copy was overwritten).  Thread t is exact after
  // at most t rounds, so the loop ends; misses are rare, so it is usually no
  // round at all.  Only thread 0's entry state is left to the cross-tile check.
  Aff used = assumed;
  {
    bool stale = !lb_warp && t > 0 && start_t < n && !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
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
      stale = !lb_warp && t > 0 && start_t < n && !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
    }
    if (s.timeline && t == 0) s.timeline[(uint64_t)tile * 16 + 9] = rounds_done;
  }
  stamp(s, tile, 5);

  // ---- 6. verify adjacent sub-chunks inside the tile; the look-back warp
  //         records the tile's exit state for the cross-tile check ----
  if (!lb_warp) {
    bool mis = false;  // relaxation leaves none unless its round cap was hit
    if (t > 0 && start_t < n) mis = !same_bits(used, Aff{s_fa[t - 1], s_fb[t - 1]});
    const uint32_t word = __ballot_sync(0xffffffffu, mis);
    if (lane == 0) {
      s.mis_bits[(uint64_t)tile * 8 + wid] = word;
      if (word) atomicOr(s.tile_bits + (tile >> 5), 1u << (tile & 31));
    }
  } else if (lane == 0 && (uint64_t)tile + 1 < ntiles) {
    s.last[2 * (uint64_t)tile] = s_fa[kScanThreads - 1];
    s.last[2 * (uint64_t)tile + 1] = s_fb[kScanThreads - 1];
  }

  // ---- 7. coalesced store ----
  for (int li = t; li < kScanTile; li += kScanBlock) {
    const uint64_t g = tile_start + li;
    if (g < n) out[g] = sm[(kScanHaloSub + li / kScanK) * kRowStride + (li % kScanK)];
  }
  stamp(s, tile, 7);
}

// Cross-tile check: every tile's assumed entry state against the exit state
// its predecessor produced, bit for bit.  It runs after every tile is done,
// so it also returns the look-back words and the ticket to zero for the next
// call.
__global__ void __launch_bounds__(256) scan_check(ScanScratch s, uint32_t ntiles) {
  for (uint32_t T = blockIdx.x * blockDim.x + threadIdx.x; T < ntiles; T += gridDim.x * blockDim.x)
    s.flags[T] = 0ull;
  if (blockIdx.x == 0 && threadIdx.x == 0) s.ticket[0] = 0;
  for (uint32_t T = blockIdx.x * blockDim.x + threadIdx.x + 1; T < ntiles; T += gridDim.x * blockDim.x) {
    const Aff l{s.last[2 * (uint64_t)(T - 1)], s.last[2 * (uint64_t)(T - 1) + 1]};
    const Aff a{s.assumed[2 * (uint64_t)T], s.assumed[2 * (uint64_t)T + 1]};
    const bool bad = !same_bits(l, a);
    s.xmis[T] = bad ? 1u : 0u;
    if (bad) atomicOr(s.tile_bits + (T >> 5), 1u << (T & 31));
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
  b += nt * 8;                     // look-back words
  b += 64;                         // ticket
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
  s.flags = static_cast<unsigned long long*>(take(nt * 8));
  s.ticket = static_cast<uint32_t*>(take(64));
  s.assumed = static_cast<float*>(take(nt * 8));
  s.last = static_cast<float*>(take(nt * 8));
  s.mis_bits = static_cast<uint32_t*>(take(nt * 8 * 4));
  s.xmis = static_cast<uint32_t*>(take(nt * 4));
  s.tile_bits = static_cast<uint32_t*>(take(((nt + 31) / 32 + 1) * 4));
  s.repair_stats = static_cast<uint32_t*>(take(64));
  return s;
}

cudaError_t launch_scan(const float* in, float* out, uint64_t n, const ScanScratch& s, uint32_t* err,
                        cudaStream_t stream, const float* entry, const float* entry_dev) {
  if (n == 0) return cudaSuccess;
  const uint64_t ntiles = (n + kScanTile - 1) / kScanTile;
  if (ntiles > 0x7fffffffull) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float2) * kRows * kRowStride;
  cudaError_t e = cudaFuncSetAttribute(scan_main, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // All of the unified L1/shared storage as shared memory: three tiles per SM.
  e = cudaFuncSetAttribute(scan_main, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  const float2 ent = entry ? make_float2(entry[0], entry[1]) : make_float2(1.0f, 0.0f);
  scan_main<<<(unsigned)ntiles, kScanBlock, smem, stream>>>(reinterpret_cast<const float2*>(in),
                                                              reinterpret_cast<float2*>(out), n, s, err,
                                                              (entry || entry_dev) ? 1 : 0, ent,
                                                              reinterpret_cast<const float2*>(entry_dev));
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  {
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((ntiles + 255) / 256, 592);
    scan_check<<<blocks, 256, 0, stream>>>(s, (uint32_t)ntiles);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  scan_repair<<<1, 256, 0, stream>>>(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), n,
                                     s, err);
  return cudaGetLastError();
}

// Serial walks over a run, one block: the block stages batches of maps (and,
// when repairing, of stored outputs) in shared memory with coalesced loads,
// and thread 0 walks each batch from there, so the serial chain never waits
// on a global load.
//  FOLD (mode 0): the state after folding in[0..n) (the first map combined
//    with *entry when given, else copied), into state[0..1].
//  REJOIN (mode 1): walks the exact fold from *entry, overwriting out[i]
//    until the recomputed state equals the stored one bit for bit (from there
//    on the stored run is the exact trajectory); stats[0] = rewritten maps,
//    state = the run's final state.
//  SETTLE (mode 2): the multiplier chain from a copy of in[0] until it is one
//    of {0..7} * 2^-149 (or the run ends); state[0] = that multiplier,
//    stats[0] = maps folded (the table of in[stats[0]..n) continues it).
constexpr int kWalkThreads = 256;
constexpr int kWalkBatch = 2048;

__global__ void __launch_bounds__(kWalkThreads) scan_walk_kernel(const float2* __restrict__ in,
                                                                 float2* __restrict__ out, uint64_t n,
                                                                 int has_entry, float2 entry, int mode,
                                                                 float* state, unsigned long long* stats) {
  __shared__ float2 s_in[kWalkBatch];
  __shared__ float2 s_out[kWalkBatch];
  __shared__ int s_stop;
  __shared__ uint32_t s_upto;  // entries of the batch thread 0 rewrote
  if (blockIdx.x != 0 || n == 0) return;
  Aff acc{1.f, 0.f};
  float am = 1.f;
  uint64_t rewritten = 0, folded = 0;
  for (uint64_t base = 0; base < n; base += kWalkBatch) {
    const uint32_t cnt = (uint32_t)(n - base < (uint64_t)kWalkBatch ? n - base : (uint64_t)kWalkBatch);
    for (uint32_t j = threadIdx.x; j < cnt; j += kWalkThreads) {
      s_in[j] = in[base + j];
      if (mode == 1) s_out[j] = out[base + j];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int stop = 0;
      uint32_t upto = 0;
      for (uint32_t j = 0; j < cnt; ++j) {
        const uint64_t i = base + j;
        const float2 x = s_in[j];
        if (mode == 2) {
          if (i == 0) {
            am = x.x;
          } else {
            am = fmul(x.x, am);
          }
          folded = i + 1;
          if (fbits(am) <= 7u) {
            stop = 1;
            break;
          }
          continue;
        }
        if (i == 0)
          acc = has_entry ? comb(Aff{entry.x, entry.y}, Aff{x.x, x.y}) : Aff{x.x, x.y};
        else
          acc = comb(acc, Aff{x.x, x.y});
        if (mode == 1) {
          const float2 o = s_out[j];
          if (__float_as_uint(o.x) == __float_as_uint(acc.a) && __float_as_uint(o.y) == __float_as_uint(acc.b)) {
            stop = 1;
            break;
          }
          s_out[j] = make_float2(acc.a, acc.b);
          upto = j + 1;
          ++rewritten;
        }
      }
      s_stop = stop;
      s_upto = upto;
    }
    __syncthreads();
    if (mode == 1)
      for (uint32_t j = threadIdx.x; j < s_upto; j += kWalkThreads) out[base + j] = s_out[j];
    const int stop = s_stop;
    __syncthreads();
    if (stop) break;
  }
  if (threadIdx.x != 0) return;
  if (mode == 2) {
    state[0] = am;
    state[1] = 0.f;
    if (stats) stats[0] = folded;
    return;
  }
  if (mode == 1) {
    __threadfence_block();
    const float2 last = out[n - 1];
    acc = Aff{last.x, last.y};
  }
  state[0] = acc.a;
  state[1] = acc.b;
  if (stats) stats[0] = rewritten;
}

// Transfer table of a whole run for the multiplier chain: nibble m is the
// multiplier leaving in[0..n) when m * 2^-149 entered it (or 8 when that
// value is not one of {0..7} * 2^-149).  Each thread folds the eight chains
// over a contiguous stretch with the actual products; stretches compose in
// order (tab_comb) within the block, then across blocks in a second pass.
constexpr int kTabThreads = 256;

// The eight chains over in[lo..hi) with the actual products.
__device__ uint32_t chains_table_smem(const float2* s, int stride, int cnt) {
  float v[8];
#pragma unroll
  for (uint32_t m = 0; m < 8; ++m) v[m] = __uint_as_float(m);
  for (int j = 0; j < cnt; ++j) {
    const float a = s[j * stride].x;
#pragma unroll
    for (uint32_t m = 0; m < 8; ++m) v[m] = fmul(a, v[m]);
  }
  uint32_t tab = 0;
#pragma unroll
  for (uint32_t m = 0; m < 8; ++m) {
    const uint32_t b = fbits(v[m]);
    tab |= (b <= 7u ? b : 8u) << (4 * m);
  }
  return tab;
}

__device__ uint32_t block_compose(uint32_t* s_t, uint32_t mine) {
  s_t[threadIdx.x] = mine;
  __syncthreads();
  for (int d = 1; d < kTabThreads; d <<= 1) {
    uint32_t r = 0;
    const bool act = (threadIdx.x % (2 * d)) == 0 && threadIdx.x + d < kTabThreads;
    if (act) r = tab_comb(s_t[threadIdx.x], s_t[threadIdx.x + d]);
    __syncthreads();
    if (act) s_t[threadIdx.x] = r;
    __syncthreads();
  }
  const uint32_t t = s_t[0];
  __syncthreads();
  return t;
}

// Each warp owns a contiguous stretch of the run (blocks own consecutive
// stretches, warps consecutive parts of them) and walks it in batches of
// 32 x kTabK maps: the lanes load the next batch into registers (coalesced)
// while they fold the current one from the warp's padded shared-memory slice
// (lane l folds maps l*kTabK .. l*kTabK + kTabK - 1), and the 32 lane tables
// compose in order with shuffles.  No block barrier inside the loop; the
// warps' tables compose in warp order at the end, the blocks' in a second
// pass.
constexpr int kTabK = 16;
constexpr int kTabStride = kTabK + 1;  // float2 row pitch: no bank conflicts across lanes
constexpr int kTabWarps = kTabThreads / 32;
constexpr uint32_t kTabBatch = 32u * kTabK;

__device__ __forceinline__ uint32_t warp_compose(uint32_t t, uint32_t lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t o = __shfl_down_sync(0xffffffffu, t, d);
    if ((lane & (2 * d - 1)) == 0) t = tab_comb(t, o);  // lane covers [lane, lane + 2d) in order
  }
  return __shfl_sync(0xffffffffu, t, 0);
}

__global__ void __launch_bounds__(kTabThreads) scan_table_kernel(const float2* __restrict__ in, uint64_t n,
                                                                 const unsigned long long* start,
                                                                 uint32_t* __restrict__ blk_tab) {
  __shared__ float2 s_x[kTabWarps][32 * kTabStride];
  __shared__ uint32_t s_w[kTabWarps];
  if (start) {  // the run begins at a device-side offset (the same for every thread)
    const uint64_t lo = *start < n ? *start : n;
    in += lo;
    n -= lo;
  }
  const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint64_t nb = (n + kTabBatch - 1) / kTabBatch;  // batches in the run
  const uint64_t per_blk = (nb + gridDim.x - 1) / gridDim.x;
  const uint64_t per_w = (per_blk + kTabWarps - 1) / kTabWarps;
  const uint64_t b0 = min((uint64_t)blockIdx.x * per_blk + wid * per_w, nb);
  const uint64_t b1 = min(min(b0 + per_w, (uint64_t)(blockIdx.x + 1) * per_blk), nb);
  float2* sx = s_x[wid];
  float2 nxt[kTabK];
  auto load = [&](uint64_t q) {
    const uint64_t base = q * kTabBatch;
#pragma unroll
    for (int j = 0; j < kTabK; ++j) {
      const uint64_t i = base + (uint64_t)j * 32 + lane;
      nxt[j] = i < n ? __ldg(in + i) : make_float2(1.0f, 0.0f);  // identity maps past the end
    }
  };
  uint32_t acc = kTabId;
  if (b0 < b1) load(b0);
  for (uint64_t q = b0; q < b1; ++q) {
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kTabK; ++j) {
      const uint32_t e = (uint32_t)j * 32 + lane;  // map e of the batch
      sx[(e / kTabK) * kTabStride + (e % kTabK)] = nxt[j];
    }
    __syncwarp();
    if (q + 1 < b1) load(q + 1);
    acc = tab_comb(acc, warp_compose(chains_table_smem(sx + lane * kTabStride, 1, kTabK), lane));
  }
  if (lane == 0) s_w[wid] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = kTabId;
    for (int w = 0; w < kTabWarps; ++w) t = tab_comb(t, s_w[w]);
    blk_tab[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(kTabThreads) scan_table_reduce_kernel(const uint32_t* __restrict__ blk_tab,
                                                                        uint32_t nblk, uint32_t* __restrict__ out) {
  __shared__ uint32_t s_t[kTabThreads];
  uint32_t acc = kTabId;
  for (uint32_t base = 0; base < nblk; base += kTabThreads) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t t = block_compose(s_t, i < nblk ? blk_tab[i] : kTabId);
    acc = tab_comb(acc, t);
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = acc;
}

cudaError_t launch_scan_table(const float* in, uint64_t n, uint32_t* blk_scratch, uint32_t nblk_max, uint32_t* out,
                              cudaStream_t stream, const unsigned long long* start) {
  const float2* x = reinterpret_cast<const float2*>(in);
  // One wave of resident blocks, each with >= 8 batches.
  static int resident = 0;
  if (!resident) {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_table_kernel, kTabThreads, 0) != cudaSuccess)
      return cudaGetLastError();
    resident = std::max(1, sms * per_sm);
  }
  const uint64_t want = (n + 8ull * kTabBatch - 1) / (8ull * kTabBatch);
  const uint32_t nblk =
      (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(std::min<uint64_t>(want, nblk_max), (uint64_t)resident));
  scan_table_kernel<<<nblk, kTabThreads, 0, stream>>>(x, n, start, blk_scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  scan_table_reduce_kernel<<<1, kTabThreads, 0, stream>>>(blk_scratch, nblk, out);
  return cudaGetLastError();
}

// SETTLE on one warp: the multiplier chain from a copy of in[0] up to its
// first value in {0..7} * 2^-149.  The warp loads 32 multipliers at a time
// (the next 32 while it walks the current ones); every lane runs the same
// serial chain from shuffled values, so the walk is one multiply per map
// with the domain test off the dependency chain.
__global__ void __launch_bounds__(32) scan_settle_kernel(const float2* __restrict__ in, uint64_t n, float* state,
                                                         unsigned long long* stats) {
  const uint32_t lane = threadIdx.x;
  float am = 0.f, hit_a = 0.f;
  uint64_t hit = n;  // maps folded when the chain settled (n: it never did)
  float nxt = lane < n ? __ldg(&in[lane].x) : 1.0f;
  for (uint64_t base = 0; base < n && hit == n; base += 32) {
    const float cur = nxt;
    if (base + 32 + lane < n) nxt = __ldg(&in[base + 32 + lane].x);
    const uint32_t cnt = (uint32_t)(n - base < 32 ? n - base : 32);
#pragma unroll
    for (uint32_t j = 0; j < 32; ++j) {
      const float a = __shfl_sync(0xffffffffu, cur, j);
      if (j < cnt && hit == n) {
        am = (base + j == 0) ? a : fmul(a, am);
        if (fbits(am) <= 7u) {
          hit = base + j + 1;
          hit_a = am;
        }
      }
    }
  }
  if (lane == 0) {
    state[0] = hit < n ? hit_a : am;
    state[1] = 0.f;
    if (stats) stats[0] = hit;
  }
}

cudaError_t launch_scan_walk(const float* in, float* out, uint64_t n, const float* entry, int repair, float* state,
                             unsigned long long* stats, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const float2 ent = entry ? make_float2(entry[0], entry[1]) : make_float2(1.0f, 0.0f);
  if (repair == 2) {
    scan_settle_kernel<<<1, 32, 0, stream>>>(reinterpret_cast<const float2*>(in), n, state, stats);
    return cudaGetLastError();
  }
  scan_walk_kernel<<<1, kWalkThreads, 0, stream>>>(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), n,
                                         entry ? 1 : 0, ent, repair, state, stats);
  return cudaGetLastError();
}

// ---- a run's part of a split scan, entirely on the device ----------------

// blob[0 .. 2*halo): the run's last min(n, halo) maps, identity maps in front.
__global__ void scan_tail_kernel(const float2* __restrict__ in, uint64_t n, uint32_t halo, float2* __restrict__ blob) {
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < halo; j += gridDim.x * blockDim.x) {
    const int64_t src = (int64_t)n - (int64_t)halo + (int64_t)j;
    blob[j] = src >= 0 ? in[src] : make_float2(1.0f, 0.0f);
  }
}

// meta = {maps in the tail, the run's multiplier table (runs after the
// first), the first run's exit multiplier bits (8 = not in {0..7} * 2^-149), 0}.
__global__ void scan_publish_meta_kernel(const float* __restrict__ settle, const unsigned long long* __restrict__ settle_k,
                                         const uint32_t* __restrict__ table, uint64_t n, int first, uint32_t len,
                                         uint32_t* __restrict__ meta) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  meta[0] = len;
  if (first) {
    const uint32_t b = fbits(settle[0]);
    uint32_t ax = 8u;
    if (b <= 7u) ax = *settle_k < n ? tab_at(*table, b) : b;
    meta[1] = 0xffffffffu;
    meta[2] = ax;
  } else {
    meta[1] = *table;
    meta[2] = 8u;
  }
  meta[3] = 0u;
}

constexpr int kEntryMaxHalo = 4096;

// A run's guessed entry state from every run's published blob (stride
// 2*halo + 4 floats): the offset from a fold of the maps just before the run
// (nearest last, at most `halo`) starting from a copy of the first of them;
// the multiplier exactly, when the first run's exit multiplier and the tables
// of the runs in between keep it in {0..7} * 2^-149.
__global__ void __launch_bounds__(256) scan_entry_kernel(const float* __restrict__ gathered, uint32_t world,
                                                         uint32_t rank, uint32_t halo, float* __restrict__ entry) {
  __shared__ float2 s_h[kEntryMaxHalo];
  __shared__ uint32_t s_take[64], s_from[64], s_nr, s_total;
  const uint64_t stride = 2ull * halo + 4;
  if (threadIdx.x == 0) {
    uint32_t need = halo, k = 0, total = 0;
    for (int r = (int)rank - 1; r >= 0 && need > 0 && k < 64; --r, ++k) {
      const uint32_t len = __float_as_uint(gathered[(uint64_t)r * stride + 2ull * halo]);
      const uint32_t take = len < need ? len : need;
      s_take[k] = take;
      s_from[k] = (uint32_t)r;
      need -= take;
      total += take;
    }
    s_nr = k;
    s_total = total;
  }
  __syncthreads();
  // Oldest first: the last entry of the list is the earliest run.
  uint32_t dst = 0;
  for (int k = (int)s_nr - 1; k >= 0; --k) {
    const float2* tail = reinterpret_cast<const float2*>(gathered + (uint64_t)s_from[k] * stride);
    const uint32_t take = s_take[k];
    for (uint32_t j = threadIdx.x; j < take; j += blockDim.x) s_h[dst + j] = tail[halo - take + j];
    dst += take;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  Aff acc{1.0f, 0.0f};
  if (s_total) {
    acc = Aff{s_h[0].x, s_h[0].y};
    for (uint32_t j = 1; j < s_total; ++j) acc = comb(acc, Aff{s_h[j].x, s_h[j].y});
  }
  uint32_t m = __float_as_uint(gathered[2ull * halo + 2]);  // run 0's exit multiplier
  for (uint32_t r = 1; r < rank && m <= 7u; ++r) m = tab_at(__float_as_uint(gathered[r * stride + 2ull * halo + 1]), m);
  entry[0] = m <= 7u ? __uint_as_float(m) : acc.a;
  entry[1] = acc.b;
}

cudaError_t launch_scan_publish(const float* in, uint64_t n, int first, uint32_t halo, float* blob,
                                uint32_t* tab_scratch, uint32_t nblk_max, float* walk_state,
                                unsigned long long* walk_stats, cudaStream_t stream) {
  if (n == 0 || halo == 0) return cudaErrorInvalidValue;
  const float2* x = reinterpret_cast<const float2*>(in);
  scan_tail_kernel<<<(halo + 255) / 256, 256, 0, stream>>>(x, n, halo, reinterpret_cast<float2*>(blob));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  uint32_t* table = tab_scratch + nblk_max;
  if (first) {
    if ((e = launch_scan_walk(in, nullptr, n, nullptr, 2, walk_state, walk_stats, stream)) != cudaSuccess) return e;
    if ((e = launch_scan_table(in, n, tab_scratch, nblk_max, table, stream, walk_stats)) != cudaSuccess) return e;
  } else {
    if ((e = launch_scan_table(in, n, tab_scratch, nblk_max, table, stream)) != cudaSuccess) return e;
  }
  const uint32_t len = (uint32_t)(n < halo ? n : halo);
  scan_publish_meta_kernel<<<1, 32, 0, stream>>>(walk_state, walk_stats, table, n, first, len,
                                                 reinterpret_cast<uint32_t*>(blob + 2ull * halo));
  return cudaGetLastError();
}

cudaError_t launch_scan_entry(const float* gathered, uint32_t world, uint32_t rank, uint32_t halo, float* entry,
                              cudaStream_t stream) {
  if (halo == 0 || halo > (uint32_t)kEntryMaxHalo || rank == 0 || rank >= world) return cudaErrorInvalidValue;
  scan_entry_kernel<<<1, 256, 0, stream>>>(gathered, world, rank, halo, entry);
  return cudaGetLastError();
}

}  // namespace sparsl
