// Host-side gate, codecs and reverse index (host.cpp).
#pragma once

#include <stdint.h>

namespace sparsl {

enum PlanCode : int {
  PLAN_OK = 0,
  PLAN_EMPTY_ROW_PTR = 1,
  PLAN_NONZERO_START = 2,
  PLAN_NOT_MONOTONIC = 3,
  PLAN_NNZ_MISMATCH = 4,
  PLAN_NCOLS_MISMATCH = 5,
  PLAN_COLUMN_OUT_OF_RANGE = 6,
  PLAN_ROW_UNSORTED = 7,
  PLAN_TOO_LARGE = 8,
  PLAN_WEIGHTS_LEN = 9
};

struct PlanResult {
  int code;
  uint64_t a, b, c;
  uint64_t nrows, ncols, nnz, max_row_nnz;
};

uint16_t f32_to_f16(float v);
float f16_to_f32(uint16_t h);
uint16_t f32_to_bf16(float v);
float bf16_to_f32(uint16_t h);
void encode_narrow(int precision, const float* in, uint16_t* out, uint64_t n);
void quantise(int precision, const float* in, float* out, uint64_t n);

PlanResult validate_csr(const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* col, uint64_t col_len,
                        uint64_t csr_ncols, uint64_t ncols);
}  // namespace sparsl
