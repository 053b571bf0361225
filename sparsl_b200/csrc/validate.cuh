// Device-side CSR gate and narrow-weight encoding (validate.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "host.hpp"

namespace sparsl {

// validate_csr (src/backend/mod.rs:2116-2182) for a CSR whose column array is
// in device memory: the row_ptr checks run on the host copy `row_ptr` (O(rows)),
// the O(nnz) column checks on the GPU, in the reference's order, each reporting
// its first failing index -- the same PlanResult the host gate returns.
// `d_col` must hold col_len entries; `scratch` is 4 u64 words of device memory.
// Returns a CUDA error if a launch or copy failed (the result is then unset).
cudaError_t validate_csr_device(const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* d_row_ptr,
                                const uint32_t* d_col, uint64_t col_len, uint64_t csr_ncols, uint64_t ncols,
                                unsigned long long* scratch, cudaStream_t s, PlanResult* out);

// out[i] = binary16 (precision 1) or bfloat16 (precision 2) bits of in[i],
// the same encoders as the host's (codec.cuh).
cudaError_t launch_encode_narrow(int precision, const float* in, uint16_t* out, uint64_t n, cudaStream_t s);

}  // namespace sparsl
