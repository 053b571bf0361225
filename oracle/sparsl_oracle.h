/*
 * sparsl CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the CPU sequential and CPU parallel arms of the
 * reference crate (bharathvbcr/sparsl 0.3.0).  It is the checker the CUDA
 * library is compared against and the timed CPU baseline; nothing in the
 * product library links, loads or calls it.  Only tests/, the smoke entry
 * point and bench.py's CPU-baseline leg may use it.
 *
 * Parity is pinned against the reference's own golden vectors:
 *   - ChaCha12 stream:   src/rng.rs:104-117 (GOLDEN_SEED -> GOLDEN_U64)
 *   - CPU fingerprint:   tests/golden.rs:30-77 (0x2D29_6707_56DF_C8D6)
 *   - half codecs:       src/half.rs:231-348 (exhaustive 65536 round trips)
 *   - scan:              tests/scan_backend.rs:322-419, src/scan.rs:410-433
 *
 * Build flags matter: -O2 -ffp-contract=off, no -ffast-math, SSE float math
 * (x86-64 default), so `a * b + c` rounds twice exactly as Rust does.
 */
#ifndef SPARSL_ORACLE_H
#define SPARSL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ChaCha12 stream (src/rng.rs:21-71; rand_chacha 0.3.1 + rand_core 0.6.4) ---- */
typedef struct {
    uint32_t key[8];
    uint64_t counter;   /* next block counter */
    uint32_t results[64];
    uint32_t index;
} or_rng;

size_t   or_rng_size(void);
void     or_rng_init(or_rng *r, uint64_t seed);
uint32_t or_rng_next_u32(or_rng *r);
uint64_t or_rng_next_u64(or_rng *r);
float    or_rng_next_f32(or_rng *r);
double   or_rng_next_f64(or_rng *r);
uint64_t or_rng_gen_index(or_rng *r, uint64_t max);

/* ---- half.rs codecs (src/half.rs:49-219) ---- */
float    or_f16_bits_to_f32(uint16_t bits);
uint16_t or_f32_to_f16_bits(float v);
float    or_bf16_bits_to_f32(uint16_t bits);
uint16_t or_f32_to_bf16_bits(float v);
/* precision: 0 = f32 (copy), 1 = f16, 2 = bf16 -- WeightPrecision::quantise (mod.rs:624-641) */
void     or_quantise(int precision, const float *in, float *out, size_t n);
void     or_narrow_bits(int precision, const float *in, uint16_t *out, size_t n);

/* ---- CSR / CSC (src/sparse.rs, src/backend/mod.rs:2116-2182) ---- */
/* Validation error codes, in the reference's check order. */
enum {
    OR_OK = 0,
    OR_EMPTY_ROW_PTR = 1,
    OR_NONZERO_START = 2,
    OR_NOT_MONOTONIC = 3,
    OR_NNZ_MISMATCH = 4,
    OR_NCOLS_MISMATCH = 5,
    OR_COLUMN_OUT_OF_RANGE = 6,
    OR_ROW_UNSORTED = 7,
    OR_TOO_LARGE = 8
};
typedef struct {
    uint64_t a, b, c; /* error payload (index/edge/col/...) */
    uint64_t nrows, ncols, nnz, max_row_nnz;
} or_shape;
int or_validate_csr(const uint32_t *row_ptr, size_t row_ptr_len, const uint32_t *col,
                    size_t col_len, size_t csr_ncols, size_t ncols, or_shape *out);
/* Stable reverse index (sparse.rs:361-427).  Returns 0 or a CsrError-ish code. */
int or_csc_from_csr(const uint32_t *row_ptr, size_t nrows, const uint32_t *col, size_t nnz,
                    size_t ncols, uint32_t *col_ptr, uint32_t *row, uint32_t *edge_idx);
/* tests/common/mod.rs:11-30 random_csr; returns nnz.  col must hold nrows*max_deg. */
size_t or_random_csr(or_rng *r, size_t nrows, size_t ncols, size_t max_deg, uint32_t *row_ptr,
                     uint32_t *col);
/* tests/common/mod.rs:33-37 random_vec */
void or_random_vec(or_rng *r, float *out, size_t n, float scale);

/* ---- CPU kernels (src/backend/mod.rs:2188-2614).  par=0 sequential, par=1 parallel ---- */
size_t or_nnz_balanced_partitions(const uint32_t *ptr, size_t n, size_t parts, uint64_t *out_pairs);
int  or_num_threads(void);
void or_set_num_threads(int n);
void or_spmv(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w, size_t nrows,
             const float *x, float *y);
void or_spmv_spikes(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w,
                    size_t nrows, const uint32_t *spikes, float *y);
void or_spmv_t(int par, const uint32_t *col_ptr, const uint32_t *row, const uint32_t *edge_idx,
               const float *w, size_t ncols, const float *x, float *y);
void or_spmm(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w, size_t nrows,
             const float *x, size_t n_vec, float *y);
void or_lif_integrate(int par, float *v, float *theta, const float *cur, uint8_t *spikes, size_t n,
                      float decay, float v_reset, float dtheta);
void or_fused_lif(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w,
                  size_t nrows, const float *x, float *v, float *theta, uint8_t *spikes,
                  float decay, float v_reset, float dtheta);
void or_fused_spikes_lif(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w,
                         size_t nrows, const uint32_t *spikes_in, float *v, float *theta,
                         uint8_t *spikes_out, float decay, float v_reset, float dtheta);
/* Recurrent ticks (mod.rs:1889-1932): fused spikes LIF then pack into x_spikes.
 * trace (nullable) receives the number of spikes emitted at each tick. */
void or_recurrent_steps(int par, const uint32_t *row_ptr, const uint32_t *col, const float *w,
                        size_t n, uint32_t *x_spikes, float *v, float *theta, uint8_t *spikes,
                        float decay, float v_reset, float dtheta, size_t steps, uint32_t *trace);

/* ---- spikes.rs ---- */
size_t or_packed_len(size_t n);
void   or_pack_spikes_into(const uint8_t *spikes, size_t n, uint32_t *out, size_t out_len);
void   or_unpack_spikes(const uint32_t *words, size_t n, uint8_t *out);

/* ---- scan.rs ---- */
void  or_scan_sequential(const float *xs, size_t n, float *out);           /* pairs [a,b] */
void  or_scan_chunked(const float *xs, size_t n, size_t chunk, float *out); /* parallel phase 2 */
float or_scan_magnitude_envelope(const float *xs, size_t n);

/* ---- tolerances (mod.rs:533-769) ---- */
float or_tolerance_for_elementwise(float max_abs_operand);
float or_tolerance_for_spmv(uint64_t max_row_nnz, float max_abs_term, float max_abs_result);
float or_tolerance_for_spmv_narrow(int precision, uint64_t max_row_nnz, float max_abs_term,
                                   float max_abs_result);
float or_tolerance_for_scan(uint64_t prefix_len, float magnitude_envelope);

/* ---- benchmark workloads (no reference counterpart; see sparsl_oracle.c) ---- */
double or_wl_log(double x);
double or_wl_cos2pi(double u);
void or_wl_fixed_fanin(uint64_t seed, uint64_t row0, size_t nrows, uint64_t ncols, uint32_t fan_in,
                       float sigma, uint32_t *col, float *w);
void or_wl_lif_state(uint64_t seed, uint64_t cell0, size_t n, float v_lo, float v_hi, float theta0,
                     float density, float *v, float *theta, uint8_t *spikes);
void or_net_ticks(size_t nblocks, const uint32_t *const *row_ptr, const uint32_t *const *col,
                  const float *const *w, const size_t *block_rows, size_t n_total, uint32_t *x_spikes,
                  float *v, float *theta, uint8_t *spikes, float decay, float v_reset, float dtheta,
                  size_t steps, uint32_t *trace);

/* ---- tests/golden.rs:30-77 ---- */
uint64_t or_golden_fingerprint(void);

#ifdef __cplusplus
}
#endif
#endif
