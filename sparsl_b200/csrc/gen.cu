// Seeded synthetic workloads generated on the GPU (include/sparsl_workload.h).
//
// ChaCha12 keyed by rand_core's seed_from_u64 PCG32 expansion, consumed in
// BlockRng order (src/rng.rs:21-71), with one stream per row.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "../../include/sparsl_workload.h"

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kWeightSalt = 0x5EED5EED5EED5EEDull;

__device__ __forceinline__ uint32_t rotl(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

struct Key {
  uint32_t k[8];
};

// rand_core 0.6 seed_from_u64: PCG32 output words fill the 32-byte seed.
__device__ Key seed_key(uint64_t state) {
  Key key;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    state = state * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27);
    const uint32_t rot = (uint32_t)(state >> 59);
    key.k[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  return key;
}

#define QR(a, b, c, d)     \
  a += b;                  \
  d = rotl(d ^ a, 16);     \
  c += d;                  \
  b = rotl(b ^ c, 12);     \
  a += b;                  \
  d = rotl(d ^ a, 8);      \
  c += d;                  \
  b = rotl(b ^ c, 7);

// ChaCha12 block `counter` of the stream (64-bit counter, zero stream id).
__device__ void chacha12(const Key& key, uint64_t counter, uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key.k[0], key.k[1], key.k[2], key.k[3],
                    key.k[4],    key.k[5],    key.k[6],    key.k[7],    (uint32_t)counter,
                    (uint32_t)(counter >> 32), 0u, 0u};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = s[i];
#pragma unroll
  for (int r = 0; r < 6; ++r) {
    QR(x[0], x[4], x[8], x[12]);
    QR(x[1], x[5], x[9], x[13]);
    QR(x[2], x[6], x[10], x[14]);
    QR(x[3], x[7], x[11], x[15]);
    QR(x[0], x[5], x[10], x[15]);
    QR(x[1], x[6], x[11], x[12]);
    QR(x[2], x[7], x[8], x[13]);
    QR(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

// Box-Muller without libm: ln and cos come from fixed sequences of IEEE
// double operations, so the host definition of this workload draws the same
// weights bit for bit (this file is built with -fmad=false, so no step is
// contracted into an FMA).
//   ln x = e ln2 + 2 s (1 + s^2/3 + ... + s^24/25), x = m 2^e with
//          m in (1/sqrt2, sqrt2], s = (m - 1)/(m + 1)  (atanh series);
//   cos(2 pi u): 4u = q + r exactly, then sin / cos Taylor series through
//          t^17 / t^18 at t = r pi/2 or (1 - r) pi/2 in [0, pi/4].
// The series coefficients are IEEE quotients 1/(2k+1) and (-1)^k/n!, computed
// on the host and passed in by value.
struct GenCoeffs {
  double inv_odd[13];
  double sin_c[9];
  double cos_c[10];
};

GenCoeffs make_coeffs() {
  GenCoeffs c;
  double fact[19];
  fact[0] = 1.0;
  for (int n = 1; n <= 18; ++n) fact[n] = fact[n - 1] * (double)n;  // exact below 2^53
  for (int k = 0; k <= 12; ++k) c.inv_odd[k] = 1.0 / (double)(2 * k + 1);
  for (int k = 0; k <= 8; ++k) c.sin_c[k] = (k & 1 ? -1.0 : 1.0) / fact[2 * k + 1];
  for (int k = 0; k <= 9; ++k) c.cos_c[k] = (k & 1 ? -1.0 : 1.0) / fact[2 * k];
  return c;
}

// ln x for normal x in (0, 1].
__device__ double gen_log(const GenCoeffs& c, double x) {
  unsigned long long b = (unsigned long long)__double_as_longlong(x);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  b = (b & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
  double m = __longlong_as_double((long long)b);
  if (m > 1.4142135623730951) {
    m = m * 0.5;
    e += 1;
  }
  const double s = (m - 1.0) / (m + 1.0);
  const double s2 = s * s;
  double p = c.inv_odd[12];
#pragma unroll
  for (int k = 11; k >= 1; --k) p = c.inv_odd[k] + s2 * p;
  const double poly = 1.0 + s2 * p;
  return (double)e * 0.6931471805599453 + 2.0 * s * poly;
}

__device__ double gen_sin_t(const GenCoeffs& c, double t) {
  const double t2 = t * t;
  double p = c.sin_c[8];
#pragma unroll
  for (int k = 7; k >= 0; --k) p = c.sin_c[k] + t2 * p;
  return t * p;
}

__device__ double gen_cos_t(const GenCoeffs& c, double t) {
  const double t2 = t * t;
  double p = c.cos_c[9];
#pragma unroll
  for (int k = 8; k >= 0; --k) p = c.cos_c[k] + t2 * p;
  return p;
}

// cos(2 pi u) for u in [0, 1): +cos, -sin, -cos, +sin of pi r/2 for q = 0..3.
__device__ double gen_cos2pi(const GenCoeffs& c, double u) {
  const double half_pi = 1.5707963267948966;
  const double t4 = 4.0 * u;
  const int q = (int)t4;
  const double r = t4 - (double)q;
  double v;
  if ((q & 1) == 0) {
    v = r <= 0.5 ? gen_cos_t(c, r * half_pi) : gen_sin_t(c, (1.0 - r) * half_pi);
    return q == 0 ? v : -v;
  }
  v = r <= 0.5 ? gen_sin_t(c, r * half_pi) : gen_cos_t(c, (1.0 - r) * half_pi);
  return q == 1 ? -v : v;
}

constexpr int kGenWarps = 4;
constexpr uint32_t kMaxFanIn = 4096;

// One warp per row: draw, bitonic-sort, write; then the weights.
__global__ void __launch_bounds__(kGenWarps * 32) fixed_fanin_kernel(uint64_t seed, uint64_t row0, uint64_t nrows,
                                                                    uint64_t ncols, uint32_t fan_in, uint32_t pow2,
                                                                    float sigma, GenCoeffs coeffs,
                                                                    uint32_t* __restrict__ col,
                                                                    float* __restrict__ weights) {
  extern __shared__ uint32_t sm[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint32_t* buf = sm + wid * pow2;
  for (uint64_t lr = blockIdx.x * (uint64_t)kGenWarps + wid; lr < nrows; lr += (uint64_t)gridDim.x * kGenWarps) {
    const uint64_t r = row0 + lr;
    const Key key = seed_key(seed ^ (r * kGolden));
    const uint32_t nblocks = (fan_in + 7) / 8;
    for (uint32_t b = lane; b < nblocks; b += 32) {
      uint32_t w[16];
      chacha12(key, b, w);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t i = b * 8 + k;
        if (i < fan_in) {
          const uint64_t u = ((uint64_t)w[2 * k + 1] << 32) | w[2 * k];
          buf[i] = (uint32_t)(u % ncols);  // Rng::gen_index
        }
      }
    }
    for (uint32_t i = fan_in + lane; i < pow2; i += 32) buf[i] = 0xffffffffu;
    __syncwarp();
    for (uint32_t k = 2; k <= pow2; k <<= 1) {
      for (uint32_t j = k >> 1; j > 0; j >>= 1) {
        for (uint32_t t = lane; t < pow2; t += 32) {
          const uint32_t p = t ^ j;
          if (p > t) {
            const uint32_t a = buf[t], c = buf[p];
            const bool up = (t & k) == 0;
            if ((a > c) == up) {
              buf[t] = c;
              buf[p] = a;
            }
          }
        }
        __syncwarp();
      }
    }
    uint32_t* out = col + lr * fan_in;
    for (uint32_t i = lane; i < fan_in; i += 32) out[i] = buf[i];
    __syncwarp();
    // Weights: two next_f64 draws per synapse, Box-Muller in f64.
    const Key wkey = seed_key((seed ^ kWeightSalt) ^ (r * kGolden));
    const uint32_t wblocks = (fan_in + 3) / 4;
    float* wo = weights + lr * fan_in;
    for (uint32_t b = lane; b < wblocks; b += 32) {
      uint32_t w[16];
      chacha12(wkey, b, w);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t i = b * 4 + k;
        if (i < fan_in) {
          const uint64_t d0 = ((uint64_t)w[4 * k + 1] << 32) | w[4 * k];
          const uint64_t d1 = ((uint64_t)w[4 * k + 3] << 32) | w[4 * k + 2];
          const double u1 = (double)(d0 >> 11) * (1.0 / 9007199254740992.0);
          const double u2 = (double)(d1 >> 11) * (1.0 / 9007199254740992.0);
          const double z = sqrt(-2.0 * gen_log(coeffs, 1.0 - u1)) * gen_cos2pi(coeffs, u2);
          wo[i] = (float)((double)sigma * z);
        }
      }
    }
  }
}

__global__ void row_ptr_kernel(uint64_t nrows, uint32_t fan_in, uint32_t* rp) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i <= nrows; i += (uint64_t)gridDim.x * blockDim.x)
    rp[i] = (uint32_t)(i * fan_in);
}

__global__ void lif_state_kernel(uint64_t seed, uint64_t cell0, uint64_t n, float v_lo, float v_hi, float theta0,
                                 float density, float* v, float* theta, uint32_t* packed) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t nround = (n + 31) / 32 * 32;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nround; i += stride) {
    bool spike = false;
    if (i < n) {
      const uint64_t c = cell0 + i;
      uint32_t w[16];
      chacha12(seed_key(seed ^ (c * kGolden)), 0, w);
      const float f0 = (float)(w[0] >> 8) * (1.0f / 16777216.0f);  // Rng::next_f32
      const float f1 = (float)(w[1] >> 8) * (1.0f / 16777216.0f);
      v[i] = v_lo + (v_hi - v_lo) * f0;
      if (theta) theta[i] = theta0;
      spike = f1 < density;
    }
    const uint32_t ballot = __ballot_sync(0xffffffffu, spike);
    if (packed && (threadIdx.x & 31) == 0 && i < n) packed[i >> 5] = ballot;
  }
}

unsigned grid_for(uint64_t n, unsigned block) {
  uint64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > 148ull * 32) g = 148ull * 32;
  return (unsigned)g;
}

}  // namespace

extern "C" int sparsl_workload_fixed_fanin(uint64_t seed, uint64_t row0, uint64_t nrows, uint64_t ncols,
                                           uint32_t fan_in, float sigma, uint32_t* col, float* weights,
                                           void* stream) {
  if (fan_in == 0 || nrows == 0) return 0;
  if (fan_in > kMaxFanIn || ncols == 0) return 4;
  uint32_t pow2 = 32;
  while (pow2 < fan_in) pow2 <<= 1;
  const size_t smem = (size_t)kGenWarps * pow2 * 4;
  cudaFuncSetAttribute(fixed_fanin_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const uint64_t blocks = (nrows + kGenWarps - 1) / kGenWarps;
  fixed_fanin_kernel<<<(unsigned)(blocks > 148ull * 64 ? 148ull * 64 : blocks), kGenWarps * 32, smem,
                       static_cast<cudaStream_t>(stream)>>>(seed, row0, nrows, ncols, fan_in, pow2, sigma,
                                                            make_coeffs(), col, weights);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

extern "C" int sparsl_workload_uniform_row_ptr(uint64_t nrows, uint32_t fan_in, uint32_t* row_ptr, void* stream) {
  row_ptr_kernel<<<grid_for(nrows + 1, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(nrows, fan_in, row_ptr);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

extern "C" int sparsl_workload_lif_state(uint64_t seed, uint64_t cell0, uint64_t n, float v_lo, float v_hi,
                                         float theta0, float density, float* v, float* theta, uint32_t* packed,
                                         void* stream) {
  if (n == 0) return 0;
  if (packed && (cell0 % 32)) return 4;
  lif_state_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(seed, cell0, n, v_lo, v_hi,
                                                                                   theta0, density, v, theta,
                                                                                   packed);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
