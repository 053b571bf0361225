// Host-side pieces of the library: the CSR gate and the narrow-weight
// encoders.  Plain C++; no CUDA calls.
#include "host.hpp"

#include "codec.cuh"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <thread>
#include <vector>

namespace sparsl {

namespace {

inline uint32_t fbits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
inline float bitsf(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

unsigned worker_count(uint64_t work) {
  unsigned hw = std::thread::hardware_concurrency();
  if (hw == 0) hw = 1;
  const uint64_t by_work = work / (1u << 22) + 1;  // ~4M items per worker at least
  return (unsigned)std::min<uint64_t>(hw, by_work);
}

// Runs fn(begin, end) over [0, n) on a few threads.
template <class F>
void parallel_ranges(uint64_t n, F fn) {
  const unsigned k = worker_count(n);
  if (k <= 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  const uint64_t step = (n + k - 1) / k;
  for (unsigned i = 0; i < k; ++i) {
    const uint64_t b = i * step, e = std::min<uint64_t>(n, b + step);
    if (b >= e) break;
    th.emplace_back([=] { fn(b, e); });
  }
  for (auto& t : th) t.join();
}

void atomic_min(std::atomic<uint64_t>& a, uint64_t v) {
  uint64_t cur = a.load();
  while (v < cur && !a.compare_exchange_weak(cur, v)) {
  }
}

}  // namespace

uint16_t f32_to_f16(float value) { return encode_f16(value); }

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  if (e == 0x1fu) return bitsf(sign | 0x7f800000u | (m << 13));
  if (e != 0) return bitsf(sign | ((e + 112u) << 23) | (m << 13));
  // Subnormal: m * 2^-24 exactly (m < 2^10 is exact in f32).
  const float mag = (float)m * 5.9604644775390625e-08f;
  return (h & 0x8000u) ? -mag : mag;
}

uint16_t f32_to_bf16(float value) { return encode_bf16(value); }

float bf16_to_f32(uint16_t h) { return bitsf((uint32_t)h << 16); }

void encode_narrow(int precision, const float* in, uint16_t* out, uint64_t n) {
  parallel_ranges(n, [&](uint64_t b, uint64_t e) {
    if (precision == 1)
      for (uint64_t i = b; i < e; ++i) out[i] = f32_to_f16(in[i]);
    else
      for (uint64_t i = b; i < e; ++i) out[i] = f32_to_bf16(in[i]);
  });
}

void quantise(int precision, const float* in, float* out, uint64_t n) {
  parallel_ranges(n, [&](uint64_t b, uint64_t e) {
    for (uint64_t i = b; i < e; ++i) {
      if (precision == 1)
        out[i] = f16_to_f32(f32_to_f16(in[i]));
      else if (precision == 2)
        out[i] = bf16_to_f32(f32_to_bf16(in[i]));
      else
        out[i] = in[i];
    }
  });
}

// validate_csr (src/backend/mod.rs:2116-2182).  The checks run in the
// reference's order and each reports its first failing index, so the error a
// caller sees is the one the reference would report.
PlanResult validate_csr(const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* col, uint64_t col_len,
                        uint64_t csr_ncols, uint64_t ncols) {
  PlanResult r{};
  if (row_ptr_len == 0) {
    r.code = PLAN_EMPTY_ROW_PTR;
    return r;
  }
  if (row_ptr[0] != 0) {
    r.code = PLAN_NONZERO_START;
    r.a = row_ptr[0];
    return r;
  }
  {
    std::atomic<uint64_t> first{UINT64_MAX};
    parallel_ranges(row_ptr_len - 1, [&](uint64_t b, uint64_t e) {
      for (uint64_t i = b + 1; i <= e; ++i)
        if (row_ptr[i] < row_ptr[i - 1]) {
          atomic_min(first, i);
          return;
        }
    });
    if (first.load() != UINT64_MAX) {
      r.code = PLAN_NOT_MONOTONIC;
      r.a = first.load();
      return r;
    }
  }
  const uint32_t end = row_ptr[row_ptr_len - 1];
  if ((uint64_t)end != col_len) {
    r.code = PLAN_NNZ_MISMATCH;
    r.a = end;
    r.b = col_len;
    return r;
  }
  if (csr_ncols != ncols) {
    r.code = PLAN_NCOLS_MISMATCH;
    r.a = csr_ncols;
    r.b = ncols;
    return r;
  }
  {
    std::atomic<uint64_t> first{UINT64_MAX};
    parallel_ranges(col_len, [&](uint64_t b, uint64_t e) {
      for (uint64_t i = b; i < e; ++i)
        if ((uint64_t)col[i] >= ncols) {
          atomic_min(first, i);
          return;
        }
    });
    if (first.load() != UINT64_MAX) {
      r.code = PLAN_COLUMN_OUT_OF_RANGE;
      r.a = first.load();
      r.b = col[r.a];
      r.c = ncols;
      return r;
    }
  }
  const uint64_t nrows = row_ptr_len - 1;
  {
    // First unsorted row, and within it the first unsorted edge.
    std::atomic<uint64_t> first{UINT64_MAX};
    parallel_ranges(nrows, [&](uint64_t b, uint64_t e) {
      for (uint64_t row = b; row < e; ++row) {
        for (uint64_t k = (uint64_t)row_ptr[row] + 1; k < row_ptr[row + 1]; ++k)
          if (col[k] < col[k - 1]) {
            atomic_min(first, row);
            return;
          }
      }
    });
    if (first.load() != UINT64_MAX) {
      const uint64_t row = first.load();
      r.code = PLAN_ROW_UNSORTED;
      r.a = row;
      for (uint64_t k = (uint64_t)row_ptr[row] + 1; k < row_ptr[row + 1]; ++k)
        if (col[k] < col[k - 1]) {
          r.b = k;
          break;
        }
      return r;
    }
  }
  uint64_t mx = 0;
  for (uint64_t row = 0; row < nrows; ++row) mx = std::max<uint64_t>(mx, row_ptr[row + 1] - row_ptr[row]);
  const uint64_t vals[3] = {nrows, ncols, col_len};
  for (int k = 0; k < 3; ++k)
    if (vals[k] > 0xffffffffull) {
      r.code = PLAN_TOO_LARGE;
      r.a = (uint64_t)k;
      r.b = vals[k];
      return r;
    }
  r.code = PLAN_OK;
  r.nrows = nrows;
  r.ncols = ncols;
  r.nnz = col_len;
  r.max_row_nnz = mx;
  return r;
}

}  // namespace sparsl
