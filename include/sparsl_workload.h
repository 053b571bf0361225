/*
 * sparsl_workload.h -- seeded synthetic workloads generated on the GPU.
 *
 * Benchmark support with no counterpart in the reference crate: the
 * reference generates its inputs on the host with `Rng` (src/rng.rs), which
 * at 4.3e9 synapses takes minutes.  These kernels draw from the same kind of
 * stream -- ChaCha12 keyed by rand_core's `seed_from_u64` (src/rng.rs:29-31),
 * consumed as `next_u64` / `gen_index` / `next_f32` (src/rng.rs:42-70) --
 * with one independent stream per row so rows generate in parallel:
 *   row r of a connectivity draw uses stream seed  (seed ^ (r * 0x9E3779B97F4A7C15)).
 * All pointers are device pointers; the work is enqueued on `stream`
 * (cudaStream_t, NULL = legacy default stream).
 */
#ifndef SPARSL_WORKLOAD_H
#define SPARSL_WORKLOAD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Fixed fan-in connectivity for rows [row0, row0 + nrows): row r receives
 * `fan_in` presynaptic indices gen_index(ncols) from its stream, sorted
 * ascending (duplicates kept, as multi-edges), written to col[(r-row0)*fan_in..];
 * weights N(0, sigma^2) by Box-Muller in f64 from two next_f64 draws (u1, u2)
 * of the row's weight stream (seed ^ 0x5EED5EED5EED5EED) ^ (r * 0x9E37...),
 * w = (float)(sigma * sqrt(-2 ln(1 - u1)) * cos(2 pi u2)), where ln and cos are
 * fixed series of IEEE double operations (no libm), so a host restatement
 * draws the same arrays bit for bit.  fan_in <= 4096. */
int sparsl_workload_fixed_fanin(uint64_t seed, uint64_t row0, uint64_t nrows, uint64_t ncols,
                                uint32_t fan_in, float sigma, uint32_t *col, float *weights,
                                void *stream);

/* row_ptr[i] = (i) * fan_in for i in [0, nrows]. */
int sparsl_workload_uniform_row_ptr(uint64_t nrows, uint32_t fan_in, uint32_t *row_ptr, void *stream);

/* Per-cell initial state for cells [cell0, cell0 + n): v U[v_lo, v_hi) from
 * next_f32, theta = theta0, spike = (next_f32 < density). spikes may be NULL;
 * packed (nullable) receives the LSB-first words of the spikes for the cells
 * (cell0 must then be a multiple of 32). */
int sparsl_workload_lif_state(uint64_t seed, uint64_t cell0, uint64_t n, float v_lo, float v_hi,
                              float theta0, float density, float *v, float *theta, uint32_t *packed,
                              void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARSL_WORKLOAD_H */
