/*
 * sparsl_cuda.h -- C ABI of the B200 (sm_100a) substrate for sparsl.
 *
 * This is the library `src/backend/cuda.rs` of bharathvbcr/sparsl declares
 * but never provides (cuda.rs:23-44 lists the landing steps).  A Rust host
 * binds these symbols from `CudaDevice` / `CudaSparse` and adds one
 * `DeviceInner::Cuda` / `OpResident::Cuda` arm per dispatch site in
 * src/backend/mod.rs; the shapes arrive already validated, exactly as the
 * Metal substrate receives them (metal.rs:1048-1057).
 *
 * Conventions
 *  - Every entry point returns a status: SPARSL_OK, or an error whose static
 *    reason is available from sparsl_last_reason() and whose detail (copy it
 *    immediately; thread-local) from sparsl_last_error().  The statuses map
 *    one-to-one onto the reference's error enums:
 *      SPARSL_ERR_BACKEND     -> OpError::Backend / SparsePlanError::Backend
 *      SPARSL_ERR_EXECUTION   -> OpError::Execution { operation, detail }
 *      SPARSL_ERR_ALLOCATION  -> SparsePlanError::Allocation { what }
 *      SPARSL_ERR_INVALID     -> SparsePlanError::{EmptyRowPtr .. WeightsLen}
 *                                (detail code in sparsl_plan_error)
 *      SPARSL_ERR_LENGTH      -> OpError::{Length, TooShort, SizeOverflow}
 *      SPARSL_ERR_NO_TRANSPOSE-> OpError::TransposeNotPrepared
 *  - Host pointers are borrowed for the duration of the call only.  Calls
 *    with host buffers block until the device finished (bounded wait, see
 *    sparsl_set_timeout_ms) and check the canary tails of the buffers the
 *    device wrote.  There is no CPU fallback anywhere: with no usable GPU,
 *    sparsl_device_open fails.
 *  - bool arrays are uint8_t 0/1 (Rust bool), State arrays are float pairs
 *    [a0, b0, a1, b1, ...] (src/scan.rs:78-96, repr(C)).
 *  - Precision: 0 = f32, 1 = binary16, 2 = bfloat16 (WeightPrecision,
 *    src/backend/mod.rs:588-652).  The library quantises exactly as
 *    WeightPrecision::quantise (mod.rs:624-641) with the half.rs encoders.
 *  - Every floating-point result is bit-identical to the reference's
 *    CpuSequential arm on the same inputs (NaN payloads excepted; NaN class is
 *    preserved), because every output is one strict left fold with separate
 *    round-to-nearest multiply and add, as in mod.rs:2259-2267.
 */
#ifndef SPARSL_CUDA_H
#define SPARSL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SPARSL_OK = 0,
  SPARSL_ERR_BACKEND = 1,
  SPARSL_ERR_EXECUTION = 2,
  SPARSL_ERR_ALLOCATION = 3,
  SPARSL_ERR_INVALID = 4,
  SPARSL_ERR_LENGTH = 5,
  SPARSL_ERR_NO_TRANSPOSE = 6
};

/* SparsePlanError variants (src/backend/mod.rs:277-305), in validate_csr's
 * check order (mod.rs:2116-2182). */
enum {
  SPARSL_PLAN_OK = 0,
  SPARSL_PLAN_EMPTY_ROW_PTR = 1,
  SPARSL_PLAN_NONZERO_START = 2,
  SPARSL_PLAN_NOT_MONOTONIC = 3,
  SPARSL_PLAN_NNZ_MISMATCH = 4,
  SPARSL_PLAN_NCOLS_MISMATCH = 5,
  SPARSL_PLAN_COLUMN_OUT_OF_RANGE = 6,
  SPARSL_PLAN_ROW_UNSORTED = 7,
  SPARSL_PLAN_TOO_LARGE = 8,
  SPARSL_PLAN_WEIGHTS_LEN = 9
};

typedef struct sparsl_dev sparsl_dev;
typedef struct sparsl_op sparsl_op;
typedef struct sparsl_net sparsl_net;

/* Validated dimensions (SparseShape, mod.rs:457-503) or the first failure. */
typedef struct {
  int32_t code;          /* SPARSL_PLAN_* */
  uint64_t a, b, c;      /* error payload: index/edge/row, col/end, ncols */
  uint64_t nrows, ncols, nnz, max_row_nnz;
} sparsl_shape;

/* ---- diagnostics ------------------------------------------------------- */
const char *sparsl_last_error(void);   /* thread-local detail of the last failure */
const char *sparsl_last_reason(void);  /* static reason (&'static str) of the last failure */
const char *sparsl_version(void);
/* Completion deadline for host-facing calls (metal.rs:346-355 uses 60 s). */
void sparsl_set_timeout_ms(uint64_t ms);

/* ---- availability gate: Backend::unavailable_reason (mod.rs:106-112) ---- */
/* 0 when a usable sm_100 device exists, else SPARSL_ERR_BACKEND with a static
 * reason.  Replaces cuda::UNAVAILABLE_REASON (cuda.rs:47-48). */
int sparsl_cuda_probe(const char **reason);
int sparsl_device_count(void);

/* ---- Device (mod.rs:805-1230) ------------------------------------------ */
/* Device::try_new(Backend::Cuda) -> open_cuda (mod.rs:882-917). */
int sparsl_device_open(int ordinal, sparsl_dev **out);
void sparsl_device_close(sparsl_dev *dev);
/* Device::device_name (mod.rs:948-954). */
int sparsl_device_name(sparsl_dev *dev, char *buf, size_t cap);
/* Device::reset_metal analogue (mod.rs:825-843): clears the process-wide
 * quarantine only when no call is admitted and every dispatch that timed out
 * has since completed on the GPU (metal.rs:440-445); SPARSL_ERR_BACKEND
 * otherwise. */
int sparsl_device_reset(void);
int sparsl_quarantined(void);
/* Device::assoc_scan (mod.rs:1183-1197): in/out are n (a, b) pairs.
 * Bit-identical to assoc_scan_sequential (scan.rs:298-313).  From 2^23 maps
 * the copies run in 2^22-map chunks on two copy streams of the device,
 * overlapping each other and the scan (page-locked host memory lets them
 * run concurrently); the call returns when all of `out` is written. */
int sparsl_dev_assoc_scan(sparsl_dev *dev, const float *in, uint64_t n, float *out);
/* Device::lif_integrate (mod.rs:1202-1229). */
int sparsl_dev_lif_integrate(sparsl_dev *dev, float *v, float *theta, const float *currents,
                             uint8_t *spikes, uint64_t n, float decay, float v_reset,
                             float delta_theta);
/* The same over device arrays (each inside one allocation of this GPU),
 * enqueued on `stream` (cudaStream_t, NULL = the device's own) without
 * waiting: v, theta updated in place, spikes written as 0/1 bytes. */
int sparsl_dev_lif_integrate_device(sparsl_dev *dev, float *d_v, float *d_theta, const float *d_currents,
                                    uint8_t *d_spikes, uint64_t n, float decay, float v_reset,
                                    float delta_theta, void *stream);

/* ---- CSR gate: validate_csr (mod.rs:2116-2182) ---------------------------- */
int sparsl_validate_csr(const uint32_t *row_ptr, uint64_t row_ptr_len, const uint32_t *col,
                        uint64_t col_len, uint64_t csr_ncols, uint64_t ncols, sparsl_shape *out);

/* ---- narrow codecs (src/half.rs:49-219) ---------------------------------- */
void sparsl_f32_to_f16_bits(const float *in, uint16_t *out, uint64_t n);
void sparsl_f32_to_bf16_bits(const float *in, uint16_t *out, uint64_t n);
void sparsl_quantise(int precision, const float *in, float *out, uint64_t n);

/* ---- SparseOp (mod.rs:1281-2108) ---------------------------------------- */
/* SparseOp::prepare (mod.rs:1305-1371): validates (the gate above, first
 * failure wins, reported in *shape), quantises, uploads once and optionally
 * builds the stable reverse index (sparse.rs:361-427) on the GPU. */
int sparsl_op_prepare(sparsl_dev *dev, const uint32_t *row_ptr, uint64_t row_ptr_len,
                      const uint32_t *col, uint64_t col_len, uint64_t csr_ncols, uint64_t ncols,
                      const float *weights, uint64_t weights_len, int precision, int with_transpose,
                      sparsl_shape *shape, sparsl_op **out);
/* SparseOp::prepare (mod.rs:1305-1371) for a CSR whose arrays are already in
 * device memory of `dev` (d_row_ptr: row_ptr_len u32, d_col: col_len u32,
 * d_weights: weights_len f32): no extension in the reference, which only
 * takes host slices.  The same gate runs in the same order with the same
 * first-failure payload in *shape: the row_ptr checks on a host copy of
 * row_ptr (O(rows) bytes), the column-range and row-order checks on the GPU.
 * Narrow precisions are encoded on the GPU by the same encoder as
 * sparsl_f32_to_f16_bits / sparsl_f32_to_bf16_bits, so the operator is
 * bit-identical to one from sparsl_op_prepare on the same values.  Each
 * array must be device memory of this GPU lying inside one allocation
 * (else SPARSL_ERR_INVALID), and every write to it must have completed
 * before the call.  with_transpose builds the reverse index on the GPU, as
 * sparsl_op_prepare does.  The caller keeps ownership of its arrays. */
int sparsl_op_prepare_device(sparsl_dev *dev, const uint32_t *d_row_ptr, uint64_t row_ptr_len,
                             const uint32_t *d_col, uint64_t col_len, uint64_t csr_ncols,
                             uint64_t ncols, const float *d_weights, uint64_t weights_len,
                             int precision, int with_transpose, sparsl_shape *shape,
                             sparsl_op **out);
/* Extension, no counterpart in the reference (its operators always own
 * their arrays): sparsl_op_prepare_device in f32 precision, where the
 * operator uses the caller's row_ptr, col and weights in place instead of
 * copying them, for operators too large to hold twice (a 4.3e9-synapse
 * network's CSR is 34 GB).  Same gate, same products, bit for bit.
 * Requirements, each refused with SPARSL_ERR_INVALID:
 *  - each array starts on a 256-byte boundary;
 *  - each array is followed by 256 bytes of the same cudaMalloc allocation
 *    (not managed memory).
 * The caller keeps the arrays alive until sparsl_op_destroy, which never
 * frees them, and keeps row_ptr and col unchanged.  Forward products read
 * the weights in place.  sparsl_op_set_weights writes into d_weights.  The
 * reverse index keeps its own weight copy, refreshed by set_weights. */
int sparsl_op_prepare_device_borrowed(sparsl_dev *dev, const uint32_t *d_row_ptr,
                                      uint64_t row_ptr_len, const uint32_t *d_col,
                                      uint64_t col_len, uint64_t csr_ncols, uint64_t ncols,
                                      float *d_weights, uint64_t weights_len, int with_transpose,
                                      sparsl_shape *shape, sparsl_op **out);
/* Csc::from_csr_slices (sparse.rs:361-427) on the GPU, for a CSR in device
 * memory of `dev`: writes d_col_ptr[ncols + 1], and per slot d_row[col_len]
 * and d_edge_idx[col_len] -- each column's edges in CSR order, the same
 * arrays as the reference's counting sort.  The CSR passes the gate of
 * sparsl_validate_csr first (payload in *shape).  Every array must be
 * device memory of this GPU inside one allocation, with all writes to the
 * inputs complete.  Runs on the device's stream and returns when done. */
int sparsl_csc_from_csr_device(sparsl_dev *dev, const uint32_t *d_row_ptr, uint64_t row_ptr_len,
                               const uint32_t *d_col, uint64_t col_len, uint64_t ncols,
                               uint32_t *d_col_ptr, uint32_t *d_row, uint32_t *d_edge_idx,
                               sparsl_shape *shape);
void sparsl_op_destroy(sparsl_op *op);
int sparsl_op_shape(sparsl_op *op, sparsl_shape *out);
int sparsl_op_weight_precision(sparsl_op *op);    /* mod.rs:1582 */
/* Which device layouts an operator holds besides its CSR (a diagnostic; no
 * reference counterpart). */
enum {
  SPARSL_LAYOUT_ELL = 1,            /* uniform rows: TMA-streamed [nrows x L] */
  SPARSL_LAYOUT_ROW_ORDER = 2,      /* skewed rows: row folds in descending-length order */
  SPARSL_LAYOUT_SLICED_REVERSE = 4, /* transpose: sliced-ELL reverse index */
  SPARSL_LAYOUT_CSC = 8,            /* transpose: plain reverse index (hub columns) */
  SPARSL_LAYOUT_X_PANELS = 16,      /* uniform rows, x in <= 4 shared-memory panels: dense-x SpMV
                                       reads a tile-interleaved copy of col / values */
  SPARSL_LAYOUT_T_X_PANELS = 32,    /* the same for the transpose product, from the sliced-ELL
                                       reverse index (x of nrows values in <= 4 panels) */
  SPARSL_LAYOUT_ORDERED_COPY = 64   /* skewed rows: a tile-interleaved copy in descending-length
                                       order, used by every forward product whose operand is dense
                                       or a spike vector of at most 200 KB */
};
int sparsl_op_layouts(sparsl_op *op);
/* Test and diagnostic hook, no reference counterpart: forget the operator's
 * uniform-row layouts (TMA stream and x panels), its descending-length row
 * order and ordered copy, and its transpose x panels, so every later forward product runs on
 * the generic row-fold engine in natural row order and the transpose on the
 * reverse index itself.  The engine choice at prepare stays a function of the operator's
 * shape alone; this only lets a caller compare the engines on one operator.
 * Results are identical either way. */
int sparsl_op_force_plain_row_fold(sparsl_op *op);
/* Failure-detection test hooks, no reference counterpart.
 * sparsl_dev_test_expired_wait runs one look-back whose predecessor never
 * publishes: the device's bounded wait runs out (about 0.1 s), records the
 * look-back-timeout bit in the device error word and returns, and the call
 * reports SPARSL_ERR_EXECUTION.  The device stays usable.
 * sparsl_op_test_mark_canary overwrites one word of the operator's y canary
 * tail from the host (inside the allocation) and runs the canary check: the
 * call reports SPARSL_ERR_EXECUTION, and so does every later call on that
 * operator, whose tail stays marked. */
int sparsl_dev_test_expired_wait(sparsl_dev *dev);
int sparsl_op_test_mark_canary(sparsl_op *op);
int sparsl_op_has_transpose(sparsl_op *op);       /* mod.rs:1594 */
/* SparseOp::set_weights (mod.rs:1392-1409). */
int sparsl_op_set_weights(sparsl_op *op, const float *weights, uint64_t n);
/* SparseOp::spmv (mod.rs:1411-1429): y += A x.  This and spmv_spikes: a y in
 * pinned host memory the device can address (sparsl_host_alloc) is
 * accumulated into in place over PCIe; otherwise it is staged through a
 * device copy. */
int sparsl_op_spmv(sparsl_op *op, const float *x, uint64_t x_len, float *y, uint64_t y_len);
/* SparseOp::spmv_spikes (mod.rs:1449-1468). */
int sparsl_op_spmv_spikes(sparsl_op *op, const uint32_t *spikes, uint64_t words, float *y,
                          uint64_t y_len);
/* SparseOp::spmv_t (mod.rs:1486-1505): y += A^T x. */
int sparsl_op_spmv_t(sparsl_op *op, const float *x, uint64_t x_len, float *y, uint64_t y_len);
/* SparseOp::spmm (mod.rs:1528-1571): batch-minor X[ncols][n_vec], Y[nrows][n_vec].
 * For operators of 65,536 rows or more, Y moves in eight row ranges on two
 * copy streams, each range folded as soon as its rows are in. */
int sparsl_op_spmm(sparsl_op *op, const float *x, uint64_t x_len, uint64_t n_vec, float *y,
                   uint64_t y_len);
/* SparseOp::fused_spmv_lif (mod.rs:1609-1636).  This and the spike variant
 * below: when v, theta and the spike bytes are all pinned host memory the
 * device can address (sparsl_host_alloc), the tick reads and writes them in
 * place over PCIe and only the operand is copied; otherwise they are staged
 * through device copies. */
int sparsl_op_fused_lif(sparsl_op *op, const float *x, uint64_t x_len, float *v, float *theta,
                        uint8_t *spikes, uint64_t n, float decay, float v_reset, float delta_theta);
/* SparseOp::fused_spmv_spikes_lif (mod.rs:1644-1678). */
int sparsl_op_fused_spikes_lif(sparsl_op *op, const uint32_t *spikes_in, uint64_t words, float *v,
                               float *theta, uint8_t *spikes_out, uint64_t n, float decay,
                               float v_reset, float delta_theta);

/* ---- resident API (mod.rs:1680-1973) ------------------------------------ */
int sparsl_op_write_x(sparsl_op *op, const float *x, uint64_t len);              /* :1687 */
int sparsl_op_write_x_spikes(sparsl_op *op, const uint32_t *s, uint64_t words);  /* :1704 */
int sparsl_op_write_y(sparsl_op *op, const float *y, uint64_t len);              /* :1720 */
int sparsl_op_write_lif_state(sparsl_op *op, const float *v, const float *theta,
                              uint64_t n);                                        /* :1737 */
int sparsl_op_spmv_resident(sparsl_op *op);                                       /* :1756 */
int sparsl_op_fused_lif_resident(sparsl_op *op, float decay, float v_reset,
                                 float delta_theta);                              /* :1792 */
int sparsl_op_fused_spikes_lif_resident(sparsl_op *op, float decay, float v_reset,
                                        float delta_theta);                       /* :1827 */
int sparsl_op_pack_resident_spikes(sparsl_op *op);                                /* :1865 */
/* fused_spmv_spikes_lif_recurrent_steps (mod.rs:1889-1932).  Also records
 * the spike count of every tick in a device-side trace (see below). */
int sparsl_op_recurrent_steps(sparsl_op *op, float decay, float v_reset, float delta_theta,
                              uint64_t steps);
int sparsl_op_sync_y(sparsl_op *op, float *y, uint64_t len);                      /* :1937 */
int sparsl_op_sync_lif_state(sparsl_op *op, float *v, float *theta, uint8_t *spikes,
                             uint64_t n);                                         /* :1960 */
int sparsl_op_sync_x_spikes(sparsl_op *op, uint32_t *s, uint64_t words);

/* ---- tick trace (extension; no reference counterpart) -------------------- */
/* Spike counts of the ticks run by the last sparsl_op_recurrent_steps call. */
int sparsl_op_spike_trace(sparsl_op *op, uint32_t *out, uint64_t cap, uint64_t *n_out);
/* Ascending indices of the cells that fired in the last recurrent tick, as
 * compacted on the device by warp ballots and a decoupled look-back. */
int sparsl_op_spike_indices(sparsl_op *op, uint32_t *out, uint64_t cap, uint64_t *count);

/* ---- zero-copy interop: bound buffers and event handoff ------------------ */
/* CUDA analogue of SparseOp::bind_mtl_x / bind_mtl_y / unbind_mtl_* /
 * mtl_*_gpu_address / alloc_mtl_f32 (mod.rs:1975-2066, metal.rs:1834-1916).
 * A bound caller buffer (device memory of the operator's GPU holding at least
 * ncols (x) or nrows (y) f32 up to the end of its allocation; else
 * SPARSL_ERR_BACKEND or SPARSL_ERR_LENGTH, validate_external_vec
 * metal.rs:1805-1832) replaces the operator's own x / y:
 *  - sparsl_op_spmv and sparsl_op_fused_lif read a bound x instead of the
 *    host slice; sparsl_op_spmv accumulates into a bound y and copies it
 *    into the host slice afterwards;
 *  - spmv_resident, fused_lif_resident and sync_y use the bound buffers;
 *  - write_x / write_y are refused (SPARSL_ERR_BACKEND) while bound.
 * The caller keeps the buffer alive while it is bound. */
int sparsl_op_bind_x(sparsl_op *op, const float *d_x);
int sparsl_op_bind_y(sparsl_op *op, float *d_y);
int sparsl_op_unbind_x(sparsl_op *op);
int sparsl_op_unbind_y(sparsl_op *op);
int sparsl_op_x_address(sparsl_op *op, uint64_t *out); /* active x: bound or owned */
int sparsl_op_y_address(sparsl_op *op, uint64_t *out);
/* n f32 of device memory on the operator's GPU, filled from `data` (NULL:
 * uninitialised); free with sparsl_device_free. */
int sparsl_op_alloc_f32(sparsl_op *op, const float *data, uint64_t n, float **out);
/* wait_shared_event / signal_shared_event (metal.rs:1918-1953) with a CUDA
 * event (cudaEvent_t) in place of an MTLSharedEvent:
 *  - wait: the operator's stream waits for the event on the device, and the
 *    host polls it for up to timeout_ms (SPARSL_ERR_EXECUTION on expiry).
 *    NULL returns at once, like a value of 0.
 *  - signal: records the event on the operator's stream, so it completes
 *    after all of the operator's work enqueued before it. */
int sparsl_op_wait_event(sparsl_op *op, void *event, uint64_t timeout_ms);
int sparsl_op_signal_event(sparsl_op *op, void *event);

/* ---- zero-copy device-pointer entry points (extension) ------------------- */
/* Operands are device pointers and the work is only enqueued on `stream`
 * (cudaStream_t, or NULL for the operator's own stream).  No wait, no canary
 * check. */
int sparsl_op_spmv_device(sparsl_op *op, const float *d_x, float *d_y, void *stream);
int sparsl_op_spmv_spikes_device(sparsl_op *op, const uint32_t *d_spikes, float *d_y, void *stream);
int sparsl_op_spmv_t_device(sparsl_op *op, const float *d_x, float *d_y, void *stream);
int sparsl_op_spmm_device(sparsl_op *op, const float *d_x, uint64_t n_vec, float *d_y, void *stream);
int sparsl_dev_assoc_scan_device(sparsl_dev *dev, const float *d_in, uint64_t n, float *d_out,
                                 void *stream);
/* ---- a scan split into runs across devices (extension) ------------------- */
/* The pieces of an exact scan whose maps are split into consecutive runs,
 * one per device (the speculate/verify rule of the single-device scan,
 * applied across devices; the host exchanges the boundary states).
 *  - assoc_scan_from: the scan of a run that continues a longer sequence
 *    whose state before d_in[0] is entry[0..1] (NULL: the run starts the
 *    sequence and its first map is copied, scan.rs:280-286).
 *  - scan_fold: the state after folding d_in[0..n) (from entry, or from a
 *    copy of d_in[0]), into state[0..1] (host memory); used to guess a run's
 *    entry state from the maps before it.  Synchronous, one thread.
 *  - scan_rejoin: given a run's exact entry state, rewrites d_out from the
 *    start until it rejoins the stored trajectory bit for bit; returns the
 *    run's exit state and the number of rewritten maps.  Synchronous, one
 *    thread, at most n steps. */
int sparsl_dev_assoc_scan_from_device(sparsl_dev *dev, const float *d_in, uint64_t n, float *d_out,
                                      const float *entry, void *stream);
int sparsl_dev_scan_fold_device(sparsl_dev *dev, const float *d_in, uint64_t n, const float *entry,
                                float *state, void *stream);
int sparsl_dev_scan_rejoin_device(sparsl_dev *dev, const float *d_in, float *d_out, uint64_t n,
                                  const float *entry, float *exit_state, uint64_t *rewritten,
                                  void *stream);
/*  - scan_table: the transfer table of d_in[0..n) for the multiplier chain:
 *    nibble m (m = 0..7) is the bit pattern of the multiplier leaving the run
 *    when m * 2^-149 entered it, or 8 when that is not one of {0..7} * 2^-149
 *    (on multipliers in [0.9, 1] the f32 chain settles on such a value and
 *    stays there, so runs compose by their tables).  Synchronous.
 *  - scan_settle: the multiplier chain from a copy of d_in[0] up to the first
 *    value in {0..7} * 2^-149 (or the end of the run): *multiplier, and in
 *    *folded the number of maps folded so far. */
int sparsl_dev_scan_table_device(sparsl_dev *dev, const float *d_in, uint64_t n, uint32_t *table,
                                 void *stream);
/*  The same steps with no host round trip, for a host that all-gathers
 *  device buffers (NCCL); all three only enqueue work on `stream`:
 *  - scan_publish: writes the run's blob of 2*halo + 4 floats: its last
 *    `halo` maps (identity maps in front when the run is shorter), then the
 *    words {maps in that tail, the run's multiplier table, and on the first
 *    run (first != 0) its exit multiplier bits (8 = not settled), 0}.
 *  - scan_entry: from every run's blob, gathered in run order
 *    (world x (2*halo + 4) floats), writes run `rank`'s guessed entry state
 *    (2 floats, device memory): the offset folded over the halo, the
 *    multiplier exact when it has settled.
 *  - assoc_scan_after: the scan of the run from an entry state in device
 *    memory.
 *  halo is 1..4096 maps; world <= 64.  publish uses per-device scratch, so
 *  order these calls of one device on one stream. */
int sparsl_dev_scan_publish_device(sparsl_dev *dev, const float *d_in, uint64_t n, int first,
                                   uint32_t halo, float *d_blob, void *stream);
int sparsl_dev_scan_entry_device(sparsl_dev *dev, const float *d_gathered, uint32_t world,
                                 uint32_t rank, uint32_t halo, float *d_entry, void *stream);
int sparsl_dev_assoc_scan_after_device(sparsl_dev *dev, const float *d_in, uint64_t n, float *d_out,
                                       const float *d_entry, void *stream);
int sparsl_dev_scan_settle_device(sparsl_dev *dev, const float *d_in, uint64_t n, float *multiplier,
                                  uint64_t *folded, void *stream);
/* Enqueue recurrent ticks on the operator's stream without waiting. */
int sparsl_op_recurrent_steps_async(sparsl_op *op, float decay, float v_reset, float delta_theta,
                                    uint64_t steps);
void *sparsl_op_stream(sparsl_op *op);
void *sparsl_dev_stream(sparsl_dev *dev);
int sparsl_op_wait(sparsl_op *op);   /* bounded wait + device error word check */
int sparsl_dev_wait(sparsl_dev *dev);
/* Elements the last device scan had to replay serially (repair statistics). */
int sparsl_dev_scan_stats(sparsl_dev *dev, uint64_t *repaired, uint64_t *segments);

/* ---- allocation-free scan (no counterpart in the reference) -------------- */
/* The exact affine-map scan for callers that cannot allocate device memory:
 * a host whose allocator already owns all of HBM, or one that only lends this
 * library buffers it holds.  Scratch lives in a static device array of about
 * 256 KiB that every GPU loading the library keeps until exit, so n is capped
 * at 4,194,304 maps (larger n returns SPARSL_ERR_LENGTH).  d_in / d_out are
 * caller-owned device buffers of n (a, b) pairs on device `ordinal`, each
 * inside one allocation (checked; SPARSL_ERR_INVALID otherwise); the work
 * runs on `stream` (cudaStream_t, NULL = legacy default stream) and the call
 * waits for it with a bounded poll (timeout_ms, 0 = the process-wide
 * sparsl_set_timeout_ms value).  It calls no cudaMalloc, cudaFree or
 * allocating routine.  The first call on a device looks up the array's device
 * address.  The call polls the stream and reads the device error word back,
 * so it cannot be captured into a CUDA graph: on a capturing stream it
 * returns SPARSL_ERR_INVALID.  All calls share the one array: calls that
 * overlap on a GPU race, so serialize them.  Like every entry point it is
 * refused while the backend is quarantined.  A timeout quarantines the
 * backend: the scan may then still be running on the shared array, and a
 * later call's clearing of the array would race with it, so let the stream
 * drain before sparsl_device_reset.  A device fault or a set device error
 * word (expired bounded wait, repair limit) also quarantines and returns
 * SPARSL_ERR_EXECUTION.  Results are bit-identical to sparsl_dev_assoc_scan. */
int sparsl_dev_assoc_scan_noalloc(int ordinal, const float *d_in, uint64_t n, float *d_out,
                                  void *stream, uint64_t timeout_ms);

/* ---- pinned host memory (for end-to-end copies at DMA speed) ------------- */
void *sparsl_host_alloc(uint64_t bytes);
void sparsl_host_free(void *p);
void *sparsl_device_alloc(sparsl_dev *dev, uint64_t bytes);
void sparsl_device_free(void *p);
int sparsl_memcpy(void *dst, const void *src, uint64_t bytes); /* cudaMemcpyDefault, synchronous */

/* ---- multi-GPU network tick (extension; the reference is single device) -- */
/* One rank's share of a recurrent LIF network: `blocks` are row-block
 * operators over the global spike vector (ncols == n_global), together
 * covering rows [row_offset, row_offset + local_rows), each starting on a
 * multiple of 32.  Every tick runs the fused spike kernel on each block, then
 * all-gathers the packed spike words of all ranks with NCCL (in place, one
 * ncclAllGather per tick), then counts the global spikes into a trace.  With
 * nranks == 1 no NCCL is loaded.  nccl_id is 128 bytes from
 * sparsl_nccl_unique_id on rank 0, distributed by the caller. */
int sparsl_nccl_unique_id(uint8_t out[128]);
int sparsl_net_create(sparsl_dev *dev, sparsl_op *const *blocks, uint32_t n_blocks,
                      uint64_t row_offset, uint64_t n_global, int rank, int nranks,
                      const uint8_t *nccl_id, sparsl_net **out);
void sparsl_net_destroy(sparsl_net *net);
int sparsl_net_write_state(sparsl_net *net, const uint32_t *x_spikes_global, uint64_t words,
                           const float *v_local, const float *theta_local, uint64_t local_rows);
int sparsl_net_steps(sparsl_net *net, float decay, float v_reset, float delta_theta,
                     uint64_t steps);
int sparsl_net_steps_async(sparsl_net *net, float decay, float v_reset, float delta_theta,
                           uint64_t steps);
int sparsl_net_wait(sparsl_net *net);
void *sparsl_net_stream(sparsl_net *net);
int sparsl_net_read_state(sparsl_net *net, uint32_t *x_spikes_global, uint64_t words, float *v_local,
                          float *theta_local, uint64_t local_rows);
int sparsl_net_trace(sparsl_net *net, uint32_t *out, uint64_t cap, uint64_t *n_out);
/* sparsl_net_write_state + sparsl_net_steps + sparsl_net_read_state in one
 * call, over the same host buffers (read, then overwritten with the state
 * after the last tick; the network counterpart of the resident
 * write_lif_state / recurrent_steps / sync_lif_state sequence,
 * mod.rs:1737, :1889-1932, :1960).  When v_local and theta_local are pinned
 * host memory the device can address (sparsl_host_alloc), the first tick's
 * kernels read them over PCIe and the last tick's kernels write the new
 * state back into them (as well as into the device copy), so only the spike
 * vector is copied.  Otherwise each block's v and theta are copied in on
 * their own stream, its first tick waits for them alone, and its copy back
 * starts when its last tick kernel ends.  Blocking, like sparsl_net_steps;
 * the trace as after it. */
int sparsl_net_steps_host(sparsl_net *net, uint32_t *x_spikes_global, uint64_t words, float *v_local,
                          float *theta_local, uint64_t local_rows, float decay, float v_reset,
                          float delta_theta, uint64_t steps);
/* Bracket the fused tick kernels of each of the next (up to max_ticks) ticks
 * with CUDA events on the net's stream; 0 turns timing off. */
int sparsl_net_set_timing(sparsl_net *net, uint64_t max_ticks);
/* Sum of those kernel durations over the ticks of the last steps call. */
int sparsl_net_kernel_ms(sparsl_net *net, double *total_ms, uint64_t *ticks);
/* How the ranks exchange the spike vector after each tick (nranks > 1):
 * SPARSL_NET_EXCHANGE_PEER (default): the tick kernels store their packed
 * words straight into every peer GPU's copy over NVLink (cudaIpc mappings
 * made at create), and one small kernel per tick publishes a flag and the
 * spike count to each peer and waits, bounded, for theirs.
 * SPARSL_NET_EXCHANGE_NCCL: an in-place ncclAllGather of the packed words,
 * then a popcount (the plain-collective baseline).  Every rank must choose
 * the same mode; the trace and state are identical either way. */
enum { SPARSL_NET_EXCHANGE_PEER = 0, SPARSL_NET_EXCHANGE_NCCL = 1 };
int sparsl_net_set_exchange(sparsl_net *net, int mode);
/* The same durations per tick (ms): out[t] for the first min(cap, n) timed
 * ticks of the last steps call; *n_out = the number timed. */
int sparsl_net_tick_ms(sparsl_net *net, float *out, uint64_t cap, uint64_t *n_out);

#ifdef __cplusplus
}
#endif
#endif /* SPARSL_CUDA_H */
