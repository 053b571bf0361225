/*
 * sparsl CPU oracle -- TEST INFRASTRUCTURE ONLY (see sparsl_oracle.h).
 *
 * Plain-C restatement of the reference crate's CPU arms.  Each function cites
 * the reference file:line it follows (paths inside bharathvbcr/sparsl).  The
 * ChaCha12 generator is restated from the published ChaCha specification plus
 * rand_core 0.6.4's documented seed_from_u64 (PCG32 key expansion) and
 * rand_core's BlockRng buffering, because rand_chacha 0.3.1 / rand_core 0.6.4
 * (Cargo.lock) are not vendored in the reference tree.  The reference's golden
 * stream (src/rng.rs:104-117) pins it.
 */
#include "sparsl_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* ChaCha12 (src/rng.rs:21-71)                                               */
/* ------------------------------------------------------------------------ */

static inline uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

#define QR(a, b, c, d)                                                                        \
    do {                                                                                      \
        a += b; d ^= a; d = rotl32(d, 16);                                                   \
        c += d; b ^= c; b = rotl32(b, 12);                                                   \
        a += b; d ^= a; d = rotl32(d, 8);                                                    \
        c += d; b ^= c; b = rotl32(b, 7);                                                    \
    } while (0)

/* One 64-byte ChaCha block with 12 rounds, 64-bit block counter in words
 * 12-13 and a zero 64-bit stream id in words 14-15. */
static void chacha12_block(const uint32_t key[8], uint64_t counter, uint32_t out[16]) {
    uint32_t s[16];
    s[0] = 0x61707865u; s[1] = 0x3320646eu; s[2] = 0x79622d32u; s[3] = 0x6b206574u;
    for (int i = 0; i < 8; i++) s[4 + i] = key[i];
    s[12] = (uint32_t)counter;
    s[13] = (uint32_t)(counter >> 32);
    s[14] = 0;
    s[15] = 0;
    uint32_t x[16];
    memcpy(x, s, sizeof x);
    for (int r = 0; r < 6; r++) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; i++) out[i] = x[i] + s[i];
}

/* rand_chacha buffers four consecutive blocks (64 words) per refill. */
static void or_rng_refill(or_rng *r) {
    for (int b = 0; b < 4; b++) chacha12_block(r->key, r->counter + (uint64_t)b, r->results + 16 * b);
    r->counter += 4;
}

size_t or_rng_size(void) { return sizeof(or_rng); }

/* rand_core 0.6.4 SeedableRng::seed_from_u64: PCG32 fills the 32-byte key. */
void or_rng_init(or_rng *r, uint64_t seed) {
    const uint64_t MUL = 6364136223846793005ull;
    const uint64_t INC = 11634580027462260723ull;
    uint64_t state = seed;
    for (int i = 0; i < 8; i++) {
        state = state * MUL + INC;
        uint32_t xorshifted = (uint32_t)(((state >> 18) ^ state) >> 27);
        uint32_t rot = (uint32_t)(state >> 59);
        uint32_t x = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
        r->key[i] = x; /* little-endian bytes of x == key word i */
    }
    r->counter = 0;
    r->index = 64;
}

uint32_t or_rng_next_u32(or_rng *r) {
    if (r->index >= 64) {
        or_rng_refill(r);
        r->index = 0;
    }
    return r->results[r->index++];
}

/* BlockRng::next_u64, including the split read across a refill. */
uint64_t or_rng_next_u64(or_rng *r) {
    uint32_t idx = r->index;
    if (idx < 63) {
        r->index += 2;
        return ((uint64_t)r->results[idx + 1] << 32) | r->results[idx];
    } else if (idx >= 64) {
        or_rng_refill(r);
        r->index = 2;
        return ((uint64_t)r->results[1] << 32) | r->results[0];
    } else {
        uint64_t lo = r->results[63];
        or_rng_refill(r);
        r->index = 1;
        return ((uint64_t)r->results[0] << 32) | lo;
    }
}

/* rng.rs:53-57 */
float or_rng_next_f32(or_rng *r) {
    return (float)(or_rng_next_u32(r) >> 8) * (1.0f / (float)(1u << 24));
}

/* rng.rs:60-63 */
double or_rng_next_f64(or_rng *r) {
    return (double)(or_rng_next_u64(r) >> 11) * (1.0 / (double)(1ull << 53));
}

/* rng.rs:66-70 */
uint64_t or_rng_gen_index(or_rng *r, uint64_t max) { return or_rng_next_u64(r) % max; }

/* ------------------------------------------------------------------------ */
/* half.rs                                                                   */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* half.rs:49-90 */
float or_f16_bits_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exp = (bits >> 10) & 0x1fu;
    uint32_t man = bits & 0x03ffu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else {
            uint32_t shift = (uint32_t)__builtin_clz(man) - 21; /* leading_zeros of u32 - 21 */
            uint32_t exp32 = 127 - 14 - shift;
            uint32_t man32 = (man << shift) & 0x03ffu;
            out = sign | (exp32 << 23) | (man32 << 13);
        }
    } else if (exp == 0x1f) {
        out = sign | 0x7f800000u | (man << 13);
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    return u2f(out);
}

/* half.rs:101-161 */
uint16_t or_f32_to_f16_bits(float value) {
    uint32_t bits = f2u(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exp = (int32_t)((bits >> 23) & 0xffu);
    uint32_t mantissa = bits & 0x007fffffu;
    if (exp == 0xff) {
        uint16_t man16 = (uint16_t)(mantissa >> 13);
        if (mantissa != 0 && man16 == 0) man16 = 1;
        return (uint16_t)(sign | 0x7c00u | man16);
    }
    int32_t unbiased = exp - 127;
    if (unbiased >= 16) return (uint16_t)(sign | 0x7c00u);
    if (unbiased < -24) return sign;
    if (unbiased < -14) {
        uint32_t significand = mantissa | 0x00800000u;
        uint32_t shift = (uint32_t)(-14 - unbiased) + 13;
        uint32_t round_bit = 1u << (shift - 1);
        uint32_t sticky = significand & (round_bit - 1);
        uint32_t out = significand >> shift;
        if ((significand & round_bit) && (sticky != 0 || (out & 1u))) out += 1;
        return (uint16_t)(sign | (uint16_t)out);
    }
    uint32_t significand = mantissa & 0x007fffffu;
    uint32_t shift = 13;
    uint32_t round_bit = 1u << (shift - 1);
    uint32_t sticky = significand & (round_bit - 1);
    uint32_t man16 = significand >> shift;
    uint32_t exp16 = (uint32_t)(unbiased + 15);
    if ((significand & round_bit) && (sticky != 0 || (man16 & 1u))) {
        man16 += 1;
        if (man16 == 0x400u) {
            man16 = 0;
            exp16 += 1;
            if (exp16 >= 0x1fu) return (uint16_t)(sign | 0x7c00u);
        }
    }
    return (uint16_t)(sign | (uint16_t)(exp16 << 10) | (uint16_t)man16);
}

/* half.rs:187-189 */
float or_bf16_bits_to_f32(uint16_t bits) { return u2f((uint32_t)bits << 16); }

/* half.rs:203-214 */
uint16_t or_f32_to_bf16_bits(float value) {
    uint32_t bits = f2u(value);
    if (value != value) return (uint16_t)((bits >> 16) | 0x0040u);
    uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + bias) >> 16);
}

/* mod.rs:624-641 */
void or_quantise(int precision, const float *in, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        if (precision == 1) out[i] = or_f16_bits_to_f32(or_f32_to_f16_bits(in[i]));
        else if (precision == 2) out[i] = or_bf16_bits_to_f32(or_f32_to_bf16_bits(in[i]));
        else out[i] = in[i];
    }
}

/* mod.rs:645-651 */
void or_narrow_bits(int precision, const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++)
        out[i] = precision == 1 ? or_f32_to_f16_bits(in[i]) : or_f32_to_bf16_bits(in[i]);
}

/* ------------------------------------------------------------------------ */
/* CSR validation (mod.rs:2116-2182) and CSC (sparse.rs:361-427)             */
/* ------------------------------------------------------------------------ */

int or_validate_csr(const uint32_t *row_ptr, size_t row_ptr_len, const uint32_t *col,
                    size_t col_len, size_t csr_ncols, size_t ncols, or_shape *o) {
    memset(o, 0, sizeof *o);
    if (row_ptr_len == 0) return OR_EMPTY_ROW_PTR;
    if (row_ptr[0] != 0) { o->a = row_ptr[0]; return OR_NONZERO_START; }
    for (size_t i = 1; i < row_ptr_len; i++)
        if (row_ptr[i] < row_ptr[i - 1]) { o->a = i; return OR_NOT_MONOTONIC; }
    uint32_t end = row_ptr[row_ptr_len - 1];
    if ((size_t)end != col_len) { o->a = end; o->b = col_len; return OR_NNZ_MISMATCH; }
    if (csr_ncols != ncols) { o->a = csr_ncols; o->b = ncols; return OR_NCOLS_MISMATCH; }
    for (size_t e = 0; e < col_len; e++)
        if ((size_t)col[e] >= ncols) { o->a = e; o->b = col[e]; o->c = ncols; return OR_COLUMN_OUT_OF_RANGE; }
    for (size_t r = 0; r + 1 < row_ptr_len; r++) {
        size_t s = row_ptr[r], t = row_ptr[r + 1];
        for (size_t e = s + 1; e < t; e++)
            if (col[e] < col[e - 1]) { o->a = r; o->b = e; return OR_ROW_UNSORTED; }
    }
    size_t nrows = row_ptr_len - 1, mx = 0;
    for (size_t r = 0; r < nrows; r++) {
        size_t d = row_ptr[r + 1] - row_ptr[r];
        if (d > mx) mx = d;
    }
    size_t vals[3] = {nrows, ncols, col_len};
    for (int k = 0; k < 3; k++)
        if (vals[k] > 0xffffffffull) { o->a = (uint64_t)k; o->b = vals[k]; return OR_TOO_LARGE; }
    o->nrows = nrows; o->ncols = ncols; o->nnz = col_len; o->max_row_nnz = mx;
    return OR_OK;
}

int or_csc_from_csr(const uint32_t *row_ptr, size_t nrows, const uint32_t *col, size_t nnz,
                    size_t ncols, uint32_t *col_ptr, uint32_t *row, uint32_t *edge_idx) {
    col_ptr[0] = 0;
    if (ncols == 0) return nnz == 0 ? 0 : OR_COLUMN_OUT_OF_RANGE;
    uint32_t *next = (uint32_t *)calloc(ncols, sizeof(uint32_t));
    for (size_t e = 0; e < nnz; e++) {
        if (col[e] >= ncols) { free(next); return OR_COLUMN_OUT_OF_RANGE; }
        next[col[e]]++;
    }
    uint32_t acc = 0;
    for (size_t c = 0; c < ncols; c++) {
        acc += next[c];
        col_ptr[c + 1] = acc;
    }
    for (size_t c = 0; c < ncols; c++) next[c] = col_ptr[c];
    for (size_t r = 0; r < nrows; r++) {
        for (size_t e = row_ptr[r]; e < row_ptr[r + 1]; e++) {
            uint32_t slot = next[col[e]]++;
            row[slot] = (uint32_t)r;
            edge_idx[slot] = (uint32_t)e;
        }
    }
    free(next);
    return 0;
}

static int cmp_u32(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return (x > y) - (x < y);
}

/* tests/common/mod.rs:11-30 and sparse.rs:135-172 (a sort of plain integers
 * is stable by value, so qsort gives the same array as Rust's stable sort). */
size_t or_random_csr(or_rng *r, size_t nrows, size_t ncols, size_t max_deg, uint32_t *row_ptr,
                     uint32_t *col) {
    size_t nnz = 0;
    row_ptr[0] = 0;
    for (size_t i = 0; i < nrows; i++) {
        size_t deg = max_deg == 0 ? 0 : (size_t)or_rng_gen_index(r, max_deg + 1);
        size_t start = nnz;
        for (size_t k = 0; k < deg; k++)
            if (ncols > 0) col[nnz++] = (uint32_t)or_rng_gen_index(r, ncols);
        qsort(col + start, nnz - start, sizeof(uint32_t), cmp_u32);
        row_ptr[i + 1] = (uint32_t)nnz;
    }
    return nnz;
}

void or_random_vec(or_rng *r, float *out, size_t n, float scale) {
    for (size_t i = 0; i < n; i++) out[i] = (or_rng_next_f32(r) * 2.0f - 1.0f) * scale;
}

/* ------------------------------------------------------------------------ */
/* Partitions (mod.rs:2195-2246)                                             */
/* ------------------------------------------------------------------------ */

size_t or_nnz_balanced_partitions(const uint32_t *ptr, size_t n, size_t parts, uint64_t *out) {
    if (n == 0) return 0;
    if (parts < 1) parts = 1;
    if (parts > n) parts = n;
    size_t cnt = 0, start = 0;
    for (size_t p = 0; p < parts; p++) {
        if (start >= n) break;
        size_t left = parts - p;
        if (left == 1) {
            out[2 * cnt] = start; out[2 * cnt + 1] = n; cnt++;
            break;
        }
        size_t nnz_left = ptr[n] - ptr[start];
        size_t target = (nnz_left + left - 1) / left;
        size_t end = start + 1;
        while (end < n && (size_t)(ptr[end] - ptr[start]) < target) end++;
        out[2 * cnt] = start; out[2 * cnt + 1] = end; cnt++;
        start = end;
    }
    return cnt;
}

static int g_threads = 0;
int or_num_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
void or_set_num_threads(int n) { g_threads = n; }

/* Work-stealing parallel loop: every worker claims the next item from a shared
 * counter, which mirrors rayon's stealing over the 16-parts-per-worker plan. */
typedef struct {
    void (*fn)(void *ctx, size_t item);
    void *ctx;
    size_t n;
    atomic_size_t next;
} par_job;

static void *par_worker(void *arg) {
    par_job *j = (par_job *)arg;
    for (;;) {
        size_t i = atomic_fetch_add(&j->next, 1);
        if (i >= j->n) break;
        j->fn(j->ctx, i);
    }
    return NULL;
}

static void par_for(size_t n, void (*fn)(void *, size_t), void *ctx) {
    int t = or_num_threads();
    if ((size_t)t > n) t = (int)n;
    par_job j = {fn, ctx, n, 0};
    if (t <= 1) {
        par_worker(&j);
        return;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)t);
    for (int k = 1; k < t; k++) pthread_create(&th[k], NULL, par_worker, &j);
    par_worker(&j);
    for (int k = 1; k < t; k++) pthread_join(th[k], NULL);
    free(th);
}

/* PARALLEL_PARTS_PER_WORKER = 16 (mod.rs:2234) */
static size_t line_partitions(const uint32_t *ptr, size_t lines, uint64_t **out) {
    size_t workers = (size_t)or_num_threads();
    size_t parts = workers * 16;
    if (parts < 1) parts = 1;
    if (parts > (lines ? lines : 1)) parts = lines ? lines : 1;
    *out = (uint64_t *)malloc(sizeof(uint64_t) * 2 * (parts + 1));
    return or_nnz_balanced_partitions(ptr, lines, parts, *out);
}

/* ------------------------------------------------------------------------ */
/* Kernels                                                                    */
/* ------------------------------------------------------------------------ */

/* mod.rs:2259-2267 row_dot: strict left fold from 0.0, separate mul and add. */
static inline float row_dot(const uint32_t *rp, const uint32_t *col, const float *w, const float *x,
                            size_t r) {
    float sum = 0.0f;
    for (size_t i = rp[r]; i < rp[r + 1]; i++) sum += w[i] * x[col[i]];
    return sum;
}

/* mod.rs:2408-2421 row_dot_spikes: multiply by the decoded bit, never branch. */
static inline float row_dot_spikes(const uint32_t *rp, const uint32_t *col, const float *w,
                                   const uint32_t *s, size_t r) {
    float sum = 0.0f;
    for (size_t i = rp[r]; i < rp[r + 1]; i++) {
        uint32_t c = col[i];
        uint32_t bit = (s[c >> 5] >> (c & 31)) & 1u;
        sum += w[i] * (float)bit;
    }
    return sum;
}

/* mod.rs:2277-2288 col_dot */
static inline float col_dot(const uint32_t *cp, const uint32_t *row, const uint32_t *eidx,
                            const float *w, const float *x, size_t c) {
    float sum = 0.0f;
    for (size_t k = cp[c]; k < cp[c + 1]; k++) sum += w[eidx[k]] * x[row[k]];
    return sum;
}

/* mod.rs:2461-2472 lif_step */
static inline void lif_step(float *v, float *theta, float current, uint8_t *spike, float decay,
                            float v_reset, float dtheta) {
    float voltage = *v * decay + current;
    if (voltage >= *theta) {
        *spike = 1;
        *v = v_reset;
        *theta += dtheta;
    } else {
        *spike = 0;
        *v = voltage;
    }
}

/* One parallel line walk: the reference's rayon arm over nnz-balanced parts
 * (mod.rs:2237-2246).  Each part is a contiguous run of lines owned by one
 * worker, so every output element is written by exactly one thread. */
enum { K_SPMV, K_SPIKES, K_T, K_SPMM, K_FUSED, K_FUSED_SPIKES };
typedef struct {
    int kind;
    const uint64_t *parts;
    const uint32_t *ptr, *idx, *eidx;
    const float *w, *x;
    const uint32_t *s;
    float *y, *v, *theta;
    uint8_t *spk;
    size_t n_vec;
    float decay, v_reset, dtheta;
} lines_job;

static void row_dot_batched(const uint32_t *rp, const uint32_t *col, const float *w,
                            const float *x, size_t n_vec, size_t r, float *out);

static void lines_item(void *ctx, size_t p) {
    const lines_job *j = (const lines_job *)ctx;
    for (size_t l = j->parts[2 * p]; l < j->parts[2 * p + 1]; l++) {
        switch (j->kind) {
        case K_SPMV: j->y[l] += row_dot(j->ptr, j->idx, j->w, j->x, l); break;
        case K_SPIKES: j->y[l] += row_dot_spikes(j->ptr, j->idx, j->w, j->s, l); break;
        case K_T: j->y[l] += col_dot(j->ptr, j->idx, j->eidx, j->w, j->x, l); break;
        case K_SPMM: row_dot_batched(j->ptr, j->idx, j->w, j->x, j->n_vec, l, j->y + l * j->n_vec); break;
        case K_FUSED:
            lif_step(&j->v[l], &j->theta[l], row_dot(j->ptr, j->idx, j->w, j->x, l), &j->spk[l],
                     j->decay, j->v_reset, j->dtheta);
            break;
        default:
            lif_step(&j->v[l], &j->theta[l], row_dot_spikes(j->ptr, j->idx, j->w, j->s, l), &j->spk[l],
                     j->decay, j->v_reset, j->dtheta);
            break;
        }
    }
}

static void run_lines(lines_job *j, size_t lines) {
    uint64_t *parts;
    size_t np = line_partitions(j->ptr, lines, &parts);
    j->parts = parts;
    par_for(np, lines_item, j);
    free(parts);
}

/* mod.rs:2442-2459 */
void or_spmv(int par, const uint32_t *rp, const uint32_t *col, const float *w, size_t nrows,
             const float *x, float *y) {
    if (!par) {
        for (size_t r = 0; r < nrows; r++) y[r] += row_dot(rp, col, w, x, r);
    } else {
        lines_job j = {.kind = K_SPMV, .ptr = rp, .idx = col, .w = w, .x = x, .y = y};
        run_lines(&j, nrows);
    }
}

/* mod.rs:2423-2440 */
void or_spmv_spikes(int par, const uint32_t *rp, const uint32_t *col, const float *w, size_t nrows,
                    const uint32_t *s, float *y) {
    if (!par) {
        for (size_t r = 0; r < nrows; r++) y[r] += row_dot_spikes(rp, col, w, s, r);
    } else {
        lines_job j = {.kind = K_SPIKES, .ptr = rp, .idx = col, .w = w, .s = s, .y = y};
        run_lines(&j, nrows);
    }
}

/* mod.rs:2290-2304 */
void or_spmv_t(int par, const uint32_t *cp, const uint32_t *row, const uint32_t *eidx,
               const float *w, size_t ncols, const float *x, float *y) {
    if (!par) {
        for (size_t c = 0; c < ncols; c++) y[c] += col_dot(cp, row, eidx, w, x, c);
    } else {
        lines_job j = {.kind = K_T, .ptr = cp, .idx = row, .eidx = eidx, .w = w, .x = x, .y = y};
        run_lines(&j, ncols);
    }
}

/* mod.rs:2331-2398 row_dot_batched with BATCH_TILE = 16: per vector, a fold
 * from 0 in edge order, then y += acc.  n_vec == 1 delegates to SpMV. */
static void row_dot_batched(const uint32_t *rp, const uint32_t *col, const float *w,
                            const float *x, size_t n_vec, size_t r, float *out) {
    size_t v0 = 0;
    while (v0 < n_vec) {
        size_t width = n_vec - v0 < 16 ? n_vec - v0 : 16;
        float acc[16] = {0};
        for (size_t i = rp[r]; i < rp[r + 1]; i++) {
            float wi = w[i];
            const float *xb = x + (size_t)col[i] * n_vec + v0;
            for (size_t k = 0; k < width; k++) acc[k] += wi * xb[k];
        }
        for (size_t k = 0; k < width; k++) out[v0 + k] += acc[k];
        v0 += width;
    }
}

void or_spmm(int par, const uint32_t *rp, const uint32_t *col, const float *w, size_t nrows,
             const float *x, size_t n_vec, float *y) {
    if (n_vec == 1) {
        or_spmv(par, rp, col, w, nrows, x, y);
        return;
    }
    if (!par) {
        for (size_t r = 0; r < nrows; r++) row_dot_batched(rp, col, w, x, n_vec, r, y + r * n_vec);
    } else {
        lines_job j = {.kind = K_SPMM, .ptr = rp, .idx = col, .w = w, .x = x, .y = y, .n_vec = n_vec};
        run_lines(&j, nrows);
    }
}

typedef struct {
    float *v, *theta;
    const float *cur;
    uint8_t *spk;
    size_t n, block;
    float decay, v_reset, dtheta;
} lif_job;

static void lif_item(void *ctx, size_t b) {
    const lif_job *j = (const lif_job *)ctx;
    size_t s = b * j->block, e = s + j->block < j->n ? s + j->block : j->n;
    for (size_t i = s; i < e; i++)
        lif_step(&j->v[i], &j->theta[i], j->cur[i], &j->spk[i], j->decay, j->v_reset, j->dtheta);
}

/* mod.rs:2474-2501 */
void or_lif_integrate(int par, float *v, float *theta, const float *cur, uint8_t *spikes, size_t n,
                      float decay, float v_reset, float dtheta) {
    if (!par) {
        for (size_t i = 0; i < n; i++) lif_step(&v[i], &theta[i], cur[i], &spikes[i], decay, v_reset, dtheta);
    } else {
        lif_job j = {v, theta, cur, spikes, n, 65536, decay, v_reset, dtheta};
        par_for((n + j.block - 1) / j.block, lif_item, &j);
    }
}

/* mod.rs:2503-2545 */
void or_fused_lif(int par, const uint32_t *rp, const uint32_t *col, const float *w, size_t nrows,
                  const float *x, float *v, float *theta, uint8_t *spikes, float decay,
                  float v_reset, float dtheta) {
    if (!par) {
        for (size_t r = 0; r < nrows; r++)
            lif_step(&v[r], &theta[r], row_dot(rp, col, w, x, r), &spikes[r], decay, v_reset, dtheta);
    } else {
        lines_job j = {.kind = K_FUSED, .ptr = rp, .idx = col, .w = w, .x = x, .v = v, .theta = theta,
                       .spk = spikes, .decay = decay, .v_reset = v_reset, .dtheta = dtheta};
        run_lines(&j, nrows);
    }
}

/* mod.rs:2572-2614 */
void or_fused_spikes_lif(int par, const uint32_t *rp, const uint32_t *col, const float *w,
                         size_t nrows, const uint32_t *s, float *v, float *theta, uint8_t *out,
                         float decay, float v_reset, float dtheta) {
    if (!par) {
        for (size_t r = 0; r < nrows; r++)
            lif_step(&v[r], &theta[r], row_dot_spikes(rp, col, w, s, r), &out[r], decay, v_reset, dtheta);
    } else {
        lines_job j = {.kind = K_FUSED_SPIKES, .ptr = rp, .idx = col, .w = w, .s = s, .v = v,
                       .theta = theta, .spk = out, .decay = decay, .v_reset = v_reset, .dtheta = dtheta};
        run_lines(&j, nrows);
    }
}

/* ------------------------------------------------------------------------ */
/* spikes.rs                                                                  */
/* ------------------------------------------------------------------------ */

size_t or_packed_len(size_t n) { return (n + 31) / 32; }

/* spikes.rs:237-262 pack_spikes_into: LSB first, stale tail words zeroed. */
void or_pack_spikes_into(const uint8_t *spikes, size_t n, uint32_t *out, size_t out_len) {
    size_t need = or_packed_len(n);
    for (size_t wi = 0; wi < need; wi++) {
        uint32_t word = 0;
        for (size_t b = 0; b < 32 && wi * 32 + b < n; b++) word |= (uint32_t)(spikes[wi * 32 + b] != 0) << b;
        out[wi] = word;
    }
    for (size_t wi = need; wi < out_len; wi++) out[wi] = 0;
}

/* spikes.rs unpack_spikes */
void or_unpack_spikes(const uint32_t *words, size_t n, uint8_t *out) {
    for (size_t i = 0; i < n; i++) out[i] = (uint8_t)((words[i >> 5] >> (i & 31)) & 1u);
}

/* mod.rs:1889-1932: fused spikes LIF, then pack_spikes_into x_spikes. */
void or_recurrent_steps(int par, const uint32_t *rp, const uint32_t *col, const float *w, size_t n,
                        uint32_t *x_spikes, float *v, float *theta, uint8_t *spikes, float decay,
                        float v_reset, float dtheta, size_t steps, uint32_t *trace) {
    size_t words = or_packed_len(n);
    for (size_t t = 0; t < steps; t++) {
        or_fused_spikes_lif(par, rp, col, w, n, x_spikes, v, theta, spikes, decay, v_reset, dtheta);
        or_pack_spikes_into(spikes, n, x_spikes, words);
        if (trace) {
            uint32_t cnt = 0;
            for (size_t i = 0; i < n; i++) cnt += spikes[i] != 0;
            trace[t] = cnt;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* scan.rs                                                                    */
/* ------------------------------------------------------------------------ */

/* scan.rs:127-132 combine: a' = next.a * self.a ; b' = next.a * self.b + next.b */
static inline void combine(float *acc_a, float *acc_b, float na, float nb) {
    float a = na * *acc_a;
    float b = na * *acc_b + nb;
    *acc_a = a;
    *acc_b = b;
}

/* scan.rs:298-313 */
void or_scan_sequential(const float *xs, size_t n, float *out) {
    if (n == 0) return;
    float a = xs[0], b = xs[1];
    out[0] = a;
    out[1] = b;
    for (size_t i = 1; i < n; i++) {
        combine(&a, &b, xs[2 * i], xs[2 * i + 1]);
        out[2 * i] = a;
        out[2 * i + 1] = b;
    }
}

typedef struct {
    const float *xs, *off;
    float *out;
    size_t n, chunk;
} scan_job;

/* Phase 2 of scan.rs:272-292: re-fold one chunk from its exact offset. */
static void scan_item(void *ctx, size_t c) {
    const scan_job *j = (const scan_job *)ctx;
    const float *xs = j->xs;
    float *out = j->out;
    size_t start = c * j->chunk, end = start + j->chunk < j->n ? start + j->chunk : j->n;
    float ca, cb;
    size_t begin;
    if (c == 0) {
        ca = xs[0];
        cb = xs[1];
        out[0] = ca;
        out[1] = cb;
        begin = 1;
    } else {
        ca = j->off[2 * c];
        cb = j->off[2 * c + 1];
        begin = 0;
    }
    for (size_t i = start + begin; i < end; i++) {
        combine(&ca, &cb, xs[2 * i], xs[2 * i + 1]);
        out[2 * i] = ca;
        out[2 * i + 1] = cb;
    }
}

/* scan.rs:218-295 */
void or_scan_chunked(const float *xs, size_t n, size_t chunk, float *out) {
    if (n == 0) return;
    if (n <= chunk) {
        or_scan_sequential(xs, n, out);
        return;
    }
    size_t n_chunks = (n + chunk - 1) / chunk;
    float *off = (float *)malloc(sizeof(float) * 2 * n_chunks);
    off[0] = 1.0f;
    off[1] = 0.0f;
    float a = xs[0], b = xs[1];
    size_t since = 1, ci = 0;
    for (size_t i = 1; i < n; i++) {
        if (since == chunk) {
            ci++;
            off[2 * ci] = a;
            off[2 * ci + 1] = b;
            since = 0;
        }
        combine(&a, &b, xs[2 * i], xs[2 * i + 1]);
        since++;
    }
    scan_job j = {xs, off, out, n, chunk};
    par_for(n_chunks, scan_item, &j);
    free(off);
}

/* scan.rs:160-188 */
float or_scan_magnitude_envelope(const float *xs, size_t n) {
    double suffix_a = 1.0, prefix_b = 0.0, env = 1.0;
    for (size_t i = 0; i < n; i++) {
        double a = fabs((double)xs[2 * i]), b = fabs((double)xs[2 * i + 1]);
        if (!isfinite(a) || !isfinite(b)) return INFINITY;
        suffix_a = a * (suffix_a > 1.0 ? suffix_a : 1.0);
        prefix_b = a * prefix_b + b;
        if (!isfinite(suffix_a) || !isfinite(prefix_b)) return INFINITY;
        if (suffix_a > env) env = suffix_a;
        if (prefix_b > env) env = prefix_b;
    }
    float rounded = (float)env;
    if (!isfinite(rounded) || (double)rounded >= env) return rounded;
    return u2f(f2u(rounded) + 1);
}

/* ------------------------------------------------------------------------ */
/* Tolerances (mod.rs:533-769)                                               */
/* ------------------------------------------------------------------------ */

#define F32_EPS 1.1920929e-07f
#define F32_MINPOS 1.17549435e-38f

float or_tolerance_for_elementwise(float m) {
    float mag = fabsf(m);
    if (!(mag >= F32_MINPOS)) mag = F32_MINPOS;
    return 2.0f * F32_EPS * mag;
}

float or_tolerance_for_spmv(uint64_t max_row_nnz, float term, float result) {
    float n = (float)(max_row_nnz > 1 ? max_row_nnz : 1);
    float t = fabsf(term), r = fabsf(result);
    if (!(t >= F32_MINPOS)) t = F32_MINPOS;
    if (!(r >= F32_MINPOS)) r = F32_MINPOS;
    return 8.0f * F32_EPS * fmaf(n, t, r); /* n.mul_add(term, result) */
}

float or_tolerance_for_spmv_narrow(int precision, uint64_t max_row_nnz, float term, float result) {
    float n = (float)(max_row_nnz > 1 ? max_row_nnz : 1);
    float t = fabsf(term);
    if (!(t >= F32_MINPOS)) t = F32_MINPOS;
    float acc = or_tolerance_for_spmv(max_row_nnz, term, result);
    if (precision == 0) return acc;
    float eps = precision == 1 ? 9.765625e-4f : 7.8125e-3f;
    return 8.0f * n * eps * t + acc;
}

float or_tolerance_for_scan(uint64_t prefix_len, float env) {
    if (!isfinite(env)) return fabsf(env);
    float n = (float)(prefix_len > 1 ? prefix_len : 1);
    float m = fabsf(env);
    if (!(m >= 1.0f)) m = 1.0f;
    return 8.0f * F32_EPS * n * m;
}

/* ------------------------------------------------------------------------ */
/* tests/golden.rs:30-77                                                     */
/* ------------------------------------------------------------------------ */

static const size_t GOLDEN_SHAPES[][3] = {
    {0, 0, 0}, {0, 8, 4}, {1, 1, 0}, {1, 1, 1}, {1, 64, 64}, {7, 7, 3},
    {31, 31, 5}, {32, 32, 5}, {33, 33, 5}, {63, 64, 8}, {64, 64, 8}, {65, 64, 8},
    {255, 128, 16}, {256, 128, 16}, {257, 128, 16}, {512, 512, 1}, {1000, 1000, 64},
    {2048, 512, 3},
};

static inline void fnv1a(uint64_t *h, uint32_t bits) {
    *h ^= (uint64_t)bits;
    *h *= 0x100000001b3ull;
}

uint64_t or_golden_fingerprint(void) {
    uint64_t hash = 0xcbf29ce484222325ull;
    or_rng rng;
    or_rng_init(&rng, 0x00601DE1ull);
    for (size_t s = 0; s < sizeof GOLDEN_SHAPES / sizeof GOLDEN_SHAPES[0]; s++) {
        size_t nrows = GOLDEN_SHAPES[s][0], ncols = GOLDEN_SHAPES[s][1], deg = GOLDEN_SHAPES[s][2];
        uint32_t *rp = (uint32_t *)malloc(sizeof(uint32_t) * (nrows + 1));
        uint32_t *col = (uint32_t *)malloc(sizeof(uint32_t) * (nrows * deg + 1));
        size_t nnz = or_random_csr(&rng, nrows, ncols, deg, rp, col);
        float *w = (float *)malloc(sizeof(float) * (nnz + 1));
        float *x = (float *)malloc(sizeof(float) * (ncols + 1));
        float *y = (float *)malloc(sizeof(float) * (nrows + 1));
        float *v = (float *)malloc(sizeof(float) * (nrows + 1));
        float *th = (float *)malloc(sizeof(float) * (nrows + 1));
        uint8_t *sp = (uint8_t *)calloc(nrows + 1, 1);
        or_random_vec(&rng, w, nnz, 1.0f);
        or_random_vec(&rng, x, ncols, 1.0f);
        or_random_vec(&rng, y, nrows, 1.0f);
        if (nrows) or_spmv(0, rp, col, w, nrows, x, y);
        for (size_t i = 0; i < nrows; i++) fnv1a(&hash, f2u(y[i]));
        or_random_vec(&rng, v, nrows, 0.5f);
        or_random_vec(&rng, th, nrows, 0.5f);
        for (size_t i = 0; i < nrows; i++) th[i] = fabsf(th[i]);
        if (nrows) or_fused_lif(0, rp, col, w, nrows, x, v, th, sp, 0.9f, 0.0f, 0.1f);
        for (size_t i = 0; i < nrows; i++) {
            fnv1a(&hash, f2u(v[i]));
            fnv1a(&hash, f2u(th[i]));
        }
        for (size_t i = 0; i < nrows; i++) fnv1a(&hash, sp[i]);
        free(rp); free(col); free(w); free(x); free(y); free(v); free(th); free(sp);
    }
    return hash;
}

/* ------------------------------------------------------------------------ */
/* Benchmark workloads (no reference counterpart)                            */
/* ------------------------------------------------------------------------ */
/*
 * The definition of the seeded synthetic networks the benchmark runs, so the
 * host can draw exactly the arrays the GPU generator (libsparsl_cuda's
 * sparsl_workload_* entry points) draws.  Streams are the reference's Rng
 * (ChaCha12 keyed by seed_from_u64, src/rng.rs:21-71), one per row:
 *   row r's columns: gen_index(ncols) x fan_in from seed ^ (r * 0x9E3779B97F4A7C15),
 *                    sorted ascending (duplicates kept);
 *   row r's weights: stream (seed ^ 0x5EED5EED5EED5EED) ^ (r * 0x9E3779B97F4A7C15),
 *                    two next_f64 draws (u1, u2) per synapse,
 *                    w = (float)(sigma * sqrt(-2 ln(1 - u1)) * cos(2 pi u2))  (Box-Muller).
 * ln and cos are evaluated by fixed sequences of IEEE double operations (no
 * libm), so the host and the GPU agree bit for bit:
 *   ln x  = e ln2 + 2 s (1 + s^2/3 + ... + s^24/25),  x = m 2^e, m in (1/sqrt2, sqrt2],
 *           s = (m - 1)/(m + 1)  (the atanh series);
 *   cos 2 pi u by quadrant: 4u = q + r exactly, then the Taylor series of
 *           sin / cos at t = r pi/2 or (1 - r) pi/2, t in [0, pi/4], through t^17 / t^18.
 * Series coefficients are 1/(2k+1) and (-1)^k / n! computed as IEEE quotients.
 */

#define WL_GOLDEN 0x9E3779B97F4A7C15ull
#define WL_WEIGHT_SALT 0x5EED5EED5EED5EEDull

typedef struct {
    double inv_odd[13];  /* 1/(2k+1), k = 0..12 */
    double sin_c[9];     /* (-1)^k / (2k+1)!, k = 0..8 */
    double cos_c[10];    /* (-1)^k / (2k)!, k = 0..9 */
} wl_coeffs;

static void wl_coeffs_init(wl_coeffs *c) {
    double fact[19];
    fact[0] = 1.0;
    for (int n = 1; n <= 18; n++) fact[n] = fact[n - 1] * (double)n; /* exact below 2^53 */
    for (int k = 0; k <= 12; k++) c->inv_odd[k] = 1.0 / (double)(2 * k + 1);
    for (int k = 0; k <= 8; k++) c->sin_c[k] = (k & 1 ? -1.0 : 1.0) / fact[2 * k + 1];
    for (int k = 0; k <= 9; k++) c->cos_c[k] = (k & 1 ? -1.0 : 1.0) / fact[2 * k];
}

/* ln x for normal x in (0, 1]. */
static double wl_log(const wl_coeffs *c, double x) {
    uint64_t b;
    memcpy(&b, &x, 8);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m;
    memcpy(&m, &b, 8);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        e += 1;
    }
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double p = c->inv_odd[12];
    for (int k = 11; k >= 1; k--) p = c->inv_odd[k] + s2 * p;
    double poly = 1.0 + s2 * p;
    return (double)e * 0.6931471805599453 + 2.0 * s * poly;
}

static double wl_sin_t(const wl_coeffs *c, double t) {
    double t2 = t * t;
    double p = c->sin_c[8];
    for (int k = 7; k >= 0; k--) p = c->sin_c[k] + t2 * p;
    return t * p;
}

static double wl_cos_t(const wl_coeffs *c, double t) {
    double t2 = t * t;
    double p = c->cos_c[9];
    for (int k = 8; k >= 0; k--) p = c->cos_c[k] + t2 * p;
    return p;
}

/* cos(2 pi u) for u in [0, 1).  With 4u = q + r (q = 0..3, r in [0, 1)):
 * cos(2 pi u) = +cos(pi r/2), -sin(pi r/2), -cos(pi r/2), +sin(pi r/2) for
 * q = 0..3, and cos(pi r/2) = sin(pi (1-r)/2), so the series only ever see
 * t in [0, pi/4]. */
static double wl_cos2pi(const wl_coeffs *c, double u) {
    const double half_pi = 1.5707963267948966;
    double t4 = 4.0 * u;
    int q = (int)t4;
    double r = t4 - (double)q;
    double v;
    if ((q & 1) == 0) { /* cos(pi r / 2) */
        v = r <= 0.5 ? wl_cos_t(c, r * half_pi) : wl_sin_t(c, (1.0 - r) * half_pi);
        return q == 0 ? v : -v;
    }
    /* sin(pi r / 2): negated for q = 1 */
    v = r <= 0.5 ? wl_sin_t(c, r * half_pi) : wl_cos_t(c, (1.0 - r) * half_pi);
    return q == 1 ? -v : v;
}

double or_wl_log(double x) {
    wl_coeffs c;
    wl_coeffs_init(&c);
    return wl_log(&c, x);
}

double or_wl_cos2pi(double u) {
    wl_coeffs c;
    wl_coeffs_init(&c);
    return wl_cos2pi(&c, u);
}

/* Key of a stream (seed_from_u64's PCG32 expansion). */
static void wl_key(uint64_t seed, uint32_t key[8]) {
    or_rng r;
    or_rng_init(&r, seed);
    memcpy(key, r.key, sizeof r.key);
}

/* Eight consecutive ChaCha12 blocks from `counter`, computed lane-parallel
 * (the same rounds as chacha12_block, laid out so the compiler vectorises
 * across the eight blocks). */
#define WL_LANES 8
#define WL_QR(a, b, c, d)                                                   \
    for (int l = 0; l < WL_LANES; l++) {                                    \
        x[a][l] += x[b][l]; x[d][l] = rotl32(x[d][l] ^ x[a][l], 16);      \
        x[c][l] += x[d][l]; x[b][l] = rotl32(x[b][l] ^ x[c][l], 12);      \
        x[a][l] += x[b][l]; x[d][l] = rotl32(x[d][l] ^ x[a][l], 8);       \
        x[c][l] += x[d][l]; x[b][l] = rotl32(x[b][l] ^ x[c][l], 7);       \
    }
static void chacha12_x8(const uint32_t key[8], uint64_t counter, uint32_t out[WL_LANES][16]) {
    uint32_t x[16][WL_LANES], s[16][WL_LANES];
    for (int l = 0; l < WL_LANES; l++) {
        s[0][l] = 0x61707865u; s[1][l] = 0x3320646eu; s[2][l] = 0x79622d32u; s[3][l] = 0x6b206574u;
        for (int i = 0; i < 8; i++) s[4 + i][l] = key[i];
        uint64_t c = counter + (uint64_t)l;
        s[12][l] = (uint32_t)c;
        s[13][l] = (uint32_t)(c >> 32);
        s[14][l] = 0;
        s[15][l] = 0;
    }
    memcpy(x, s, sizeof x);
    for (int r = 0; r < 6; r++) {
        WL_QR(0, 4, 8, 12) WL_QR(1, 5, 9, 13) WL_QR(2, 6, 10, 14) WL_QR(3, 7, 11, 15)
        WL_QR(0, 5, 10, 15) WL_QR(1, 6, 11, 12) WL_QR(2, 7, 8, 13) WL_QR(3, 4, 9, 14)
    }
    for (int i = 0; i < 16; i++)
        for (int l = 0; l < WL_LANES; l++) out[l][i] = x[i][l] + s[i][l];
}

/* u64 draws [0, n) of a fresh stream: next_u64 k is words (2k, 2k+1) of
 * block k / 8, exactly what BlockRng hands out from a fresh state. */
static void wl_u64_stream(const uint32_t key[8], uint64_t *out, size_t n) {
    uint32_t blk[WL_LANES][16];
    for (size_t b0 = 0; b0 * 8 < n; b0 += WL_LANES) {
        chacha12_x8(key, (uint64_t)b0, blk);
        for (size_t l = 0; l < WL_LANES; l++) {
            const size_t b = b0 + l;
            for (size_t k = 0; k < 8 && b * 8 + k < n; k++)
                out[b * 8 + k] = ((uint64_t)blk[l][2 * k + 1] << 32) | blk[l][2 * k];
        }
    }
}

typedef struct {
    uint64_t seed, row0, ncols;
    uint32_t fan_in;
    double sigma;
    uint32_t *col;
    float *w;
    size_t nrows, rows_per_item;
    wl_coeffs coeffs;
} wl_fanin_job;

/* Stable LSD radix sort of n keys below 2^bits, 11 bits per pass. */
static void wl_radix_sort(uint32_t *a, uint32_t *tmp, size_t n, int bits) {
    uint32_t cnt[2048];
    uint32_t *src = a, *dst = tmp;
    int passes = 0;
    for (int shift = 0; shift < bits; shift += 11, passes++) {
        memset(cnt, 0, sizeof cnt);
        for (size_t i = 0; i < n; i++) cnt[(src[i] >> shift) & 2047u]++;
        uint32_t sum = 0;
        for (int d = 0; d < 2048; d++) {
            uint32_t c = cnt[d];
            cnt[d] = sum;
            sum += c;
        }
        for (size_t i = 0; i < n; i++) dst[cnt[(src[i] >> shift) & 2047u]++] = src[i];
        uint32_t *t = src;
        src = dst;
        dst = t;
    }
    if (passes & 1) memcpy(a, src, n * sizeof(uint32_t));
}

static void wl_fanin_item(void *ctx, size_t item) {
    wl_fanin_job *j = (wl_fanin_job *)ctx;
    size_t r0 = item * j->rows_per_item, r1 = r0 + j->rows_per_item;
    if (r1 > j->nrows) r1 = j->nrows;
    uint64_t *u = (uint64_t *)malloc(sizeof(uint64_t) * 2 * j->fan_in + 64);
    uint32_t *tmp = (uint32_t *)malloc(sizeof(uint32_t) * j->fan_in + 64);
    int bits = 0;
    while (bits < 64 && ((j->ncols - 1) >> bits)) bits++;
    uint32_t key[8];
    for (size_t lr = r0; lr < r1; lr++) {
        const uint64_t r = j->row0 + lr;
        uint32_t *out = j->col + lr * j->fan_in;
        wl_key(j->seed ^ (r * WL_GOLDEN), key);
        wl_u64_stream(key, u, j->fan_in);
        for (uint32_t i = 0; i < j->fan_in; i++) out[i] = (uint32_t)(u[i] % j->ncols);
        wl_radix_sort(out, tmp, j->fan_in, bits);
        wl_key((j->seed ^ WL_WEIGHT_SALT) ^ (r * WL_GOLDEN), key);
        wl_u64_stream(key, u, 2 * (size_t)j->fan_in);
        float *wo = j->w + lr * j->fan_in;
        for (uint32_t i = 0; i < j->fan_in; i++) {
            double u1 = (double)(u[2 * i] >> 11) * (1.0 / 9007199254740992.0);
            double u2 = (double)(u[2 * i + 1] >> 11) * (1.0 / 9007199254740992.0);
            double z = sqrt(-2.0 * wl_log(&j->coeffs, 1.0 - u1)) * wl_cos2pi(&j->coeffs, u2);
            wo[i] = (float)(j->sigma * z);
        }
    }
    free(u);
    free(tmp);
}

void or_wl_fixed_fanin(uint64_t seed, uint64_t row0, size_t nrows, uint64_t ncols, uint32_t fan_in, float sigma,
                       uint32_t *col, float *w) {
    if (nrows == 0 || fan_in == 0 || ncols == 0) return;
    wl_fanin_job j = {.seed = seed, .row0 = row0, .ncols = ncols, .fan_in = fan_in, .sigma = (double)sigma,
                      .col = col, .w = w, .nrows = nrows, .rows_per_item = 64};
    wl_coeffs_init(&j.coeffs);
    par_for((nrows + j.rows_per_item - 1) / j.rows_per_item, wl_fanin_item, &j);
}

/* Per-cell initial state: cell c's stream seed ^ (c * 0x9E37...) gives
 * next_f32 f0, f1: v = v_lo + (v_hi - v_lo) f0, theta = theta0, spike = f1 < density. */
void or_wl_lif_state(uint64_t seed, uint64_t cell0, size_t n, float v_lo, float v_hi, float theta0, float density,
                     float *v, float *theta, uint8_t *spikes) {
    for (size_t i = 0; i < n; i++) {
        or_rng r;
        or_rng_init(&r, seed ^ ((cell0 + i) * WL_GOLDEN));
        float f0 = or_rng_next_f32(&r);
        float f1 = or_rng_next_f32(&r);
        v[i] = v_lo + (v_hi - v_lo) * f0;
        if (theta) theta[i] = theta0;
        if (spikes) spikes[i] = f1 < density;
    }
}

/* Recurrent ticks of a network whose rows are split into row blocks that
 * all read the same input spike words (the 4.3e9-synapse network needs two
 * blocks: CSR offsets are u32).  Each tick runs every block's fused
 * spike-SpMV + LIF (or_fused_spikes_lif, CpuParallel arm), then packs all
 * cells' spikes into x_spikes and records their count: or_recurrent_steps
 * with the rows partitioned, which changes no row's fold. */
void or_net_ticks(size_t nblocks, const uint32_t *const *row_ptr, const uint32_t *const *col,
                  const float *const *w, const size_t *block_rows, size_t n_total, uint32_t *x_spikes,
                  float *v, float *theta, uint8_t *spikes, float decay, float v_reset, float dtheta,
                  size_t steps, uint32_t *trace) {
    size_t words = or_packed_len(n_total);
    for (size_t t = 0; t < steps; t++) {
        size_t off = 0;
        for (size_t b = 0; b < nblocks; b++) {
            or_fused_spikes_lif(1, row_ptr[b], col[b], w[b], block_rows[b], x_spikes, v + off, theta + off,
                                spikes + off, decay, v_reset, dtheta);
            off += block_rows[b];
        }
        or_pack_spikes_into(spikes, n_total, x_spikes, words);
        if (trace) {
            uint32_t cnt = 0;
            for (size_t i = 0; i < n_total; i++) cnt += spikes[i] != 0;
            trace[t] = cnt;
        }
    }
}
