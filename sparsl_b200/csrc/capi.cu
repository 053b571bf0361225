// Runtime and C ABI of libsparsl_cuda (declared in include/sparsl_cuda.h).
//
// Mirrors the reference's substrate contract (src/backend/metal.rs):
//  * one stream, one event and one mutex per operator (metal.rs:30-34);
//  * every device buffer a kernel writes carries a 64-word canary tail that is
//    checked after each host-facing dispatch (metal.rs:321-344);
//  * completion is awaited with a deadline, never unbounded; a timeout or a
//    sticky device error quarantines the backend process-wide and new calls
//    are refused until sparsl_device_reset (metal.rs:346-445);
//  * no CPU fallback: every entry point either runs on the GPU or fails.
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <nccl.h>

#include "../../include/sparsl_cuda.h"
#include "common.cuh"
#include "csc.cuh"
#include "ell.cuh"
#include "panel.cuh"
#include "host.hpp"
#include "misc.cuh"
#include "net.cuh"
#include "rows.cuh"
#include "scan.cuh"
#include "sell.cuh"
#include "validate.cuh"

using namespace sparsl;

namespace {

thread_local std::string t_err;
thread_local const char* t_reason = "";
std::atomic<uint64_t> g_timeout_ms{60000};
std::atomic<bool> g_quarantine{false};
std::atomic<int> g_admitted{0};
// Dispatches that timed out, as events recorded behind their work: the
// quarantine may be cleared only once every one of them has completed
// (metal.rs:440-445, TIMED_OUT_COMMANDS).
std::mutex g_timed_out_mu;
std::vector<cudaEvent_t> g_timed_out;

void retain_timed_out(cudaStream_t s) {
  cudaEvent_t e = nullptr;
  if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  if (cudaEventRecord(e, s) != cudaSuccess) {
    cudaGetLastError();
    cudaEventDestroy(e);
    return;
  }
  std::lock_guard<std::mutex> lk(g_timed_out_mu);
  g_timed_out.push_back(e);
}

int fail(int code, const char* reason, const std::string& detail) {
  t_reason = reason;
  t_err = detail;
  return code;
}

int fail_cuda(const char* operation, cudaError_t e) {
  return fail(SPARSL_ERR_EXECUTION, operation, std::string(operation) + ": " + cudaGetErrorString(e));
}

// Admission: refuse new work while quarantined, count work in flight.
struct Admission {
  bool ok;
  Admission() {
    g_admitted.fetch_add(1);
    ok = !g_quarantine.load();
  }
  ~Admission() { g_admitted.fetch_sub(1); }
};

#define ADMIT()                                                                                   \
  Admission adm_;                                                                                 \
  if (!adm_.ok)                                                                                   \
    return fail(SPARSL_ERR_BACKEND, "CUDA backend is quarantined after a failed or timed-out dispatch", \
                "CUDA backend is quarantined; call sparsl_device_reset once no work is in flight")

#define CK(op, expr)                        \
  do {                                      \
    cudaError_t ck_e_ = (expr);             \
    if (ck_e_ != cudaSuccess) return fail_cuda(op, ck_e_); \
  } while (0)

constexpr size_t kAlign = 256;
inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline uint64_t packed_len(uint64_t n) { return (n + 31) / 32; }

// A device allocation with an optional canary tail after its payload.
struct DBuf {
  void* p = nullptr;
  size_t bytes = 0;  // payload capacity
  bool guarded = false;
  bool borrowed = false;  // the caller's memory: never freed here
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
  const uint32_t* canary() const { return reinterpret_cast<const uint32_t*>(static_cast<char*>(p) + round_up(bytes, kAlign)); }
};

cudaError_t dalloc(DBuf& b, size_t bytes, bool guard, cudaStream_t s) {
  b.bytes = std::max<size_t>(bytes, 16);
  b.guarded = guard;
  const size_t total = round_up(b.bytes, kAlign) + (guard ? kCanaryWords * 4 : 0) + kAlign;
  cudaError_t e = cudaMalloc(&b.p, total);
  if (e != cudaSuccess) {
    b.p = nullptr;
    return e;
  }
  if (guard) {
    e = launch_fill(const_cast<uint32_t*>(b.canary()), kCanaryWords, kCanaryBits, s);
  }
  return e;
}

void dfree(DBuf& b) {
  if (b.p && !b.borrowed) cudaFree(b.p);
  b.p = nullptr;
  b.bytes = 0;
  b.borrowed = false;
}

// Grow-only buffer.
cudaError_t ensure(DBuf& b, size_t bytes, bool guard, cudaStream_t s) {
  if (b.p && b.bytes >= bytes) return cudaSuccess;
  if (b.p) {
    cudaStreamSynchronize(s);
    dfree(b);
  }
  return dalloc(b, bytes, guard, s);
}

std::string describe_dev_err(uint32_t bits) {
  std::string d;
  if (bits & DEVERR_LOOKBACK_TIMEOUT) d += "a bounded look-back wait expired; ";
  if (bits & DEVERR_CANARY) d += "a canary tail was overwritten (out-of-bounds device write); ";
  if (bits & DEVERR_REPAIR_LIMIT) d += "scan repair exceeded its bound; ";
  if (bits & DEVERR_PEER_TIMEOUT) d += "a peer GPU did not publish its tick in time; ";
  return d.empty() ? std::string("device error word set") : d;
}

// Bounded wait for everything enqueued on `s` so far, then the device error
// word.  `err_h` is pinned host memory the error word was copied into.
int wait_bounded(cudaStream_t s, cudaEvent_t ev, uint32_t* err_d, uint32_t* err_h, const char* operation) {
  cudaError_t e = cudaMemcpyAsync(err_h, err_d, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaEventRecord(ev, s);
  if (e != cudaSuccess) {
    g_quarantine.store(true);
    return fail_cuda(operation, e);
  }
  const auto t0 = std::chrono::steady_clock::now();
  const auto limit = std::chrono::milliseconds(g_timeout_ms.load());
  uint64_t polls = 0;
  for (;;) {
    e = cudaEventQuery(ev);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      g_quarantine.store(true);
      return fail(SPARSL_ERR_EXECUTION, operation,
                  std::string(operation) + ": device execution failed: " + cudaGetErrorString(e) +
                      "; backend quarantined");
    }
    if (std::chrono::steady_clock::now() - t0 > limit) {
      g_quarantine.store(true);
      retain_timed_out(s);
      return fail(SPARSL_ERR_EXECUTION, operation,
                  std::string(operation) + ": did not complete within " + std::to_string(g_timeout_ms.load()) +
                      " ms; backend quarantined");
    }
    // About a millisecond of spinning, so calls that finish within it return
    // as soon as they complete; then short sleeps (metal.rs:3108-3152).
    if (++polls > 2000) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  const uint32_t bits = *err_h;
  if (bits) {
    *err_h = 0;
    cudaMemsetAsync(err_d, 0, sizeof(uint32_t), s);
    cudaStreamSynchronize(s);
    return fail(SPARSL_ERR_EXECUTION, operation, std::string(operation) + ": " + describe_dev_err(bits));
  }
  return SPARSL_OK;
}

struct ErrWord {
  uint32_t* d = nullptr;
  uint32_t* h = nullptr;
  cudaError_t init() {
    cudaError_t e = cudaMalloc(&d, 64);
    if (e != cudaSuccess) return e;
    e = cudaMemset(d, 0, 64);
    if (e != cudaSuccess) return e;
    return cudaHostAlloc(&h, 64, cudaHostAllocDefault);
  }
  void release() {
    if (d) cudaFree(d);
    if (h) cudaFreeHost(h);
    d = h = nullptr;
  }
};

// ---- NCCL, loaded on demand so single-GPU users never need it ----
struct NcclApi {
  bool loaded = false;
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
std::mutex g_nccl_mu;
NcclApi g_nccl;

const char* nccl_load() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.loaded) return nullptr;
  // Reuse the NCCL the process already has (a framework that links it), so
  // one communicator library serves every caller; otherwise load it.
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return "libnccl.so.2 could not be loaded";
  auto sym = [&](const char* n) { return dlsym(h, n); };
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(sym("ncclGetUniqueId"));
  g_nccl.CommInitRankConfig = reinterpret_cast<decltype(g_nccl.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
  g_nccl.CommGetAsyncError = reinterpret_cast<decltype(g_nccl.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
  g_nccl.AllGather = reinterpret_cast<decltype(g_nccl.AllGather)>(sym("ncclAllGather"));
  g_nccl.CommFinalize = reinterpret_cast<decltype(g_nccl.CommFinalize)>(sym("ncclCommFinalize"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(sym("ncclCommDestroy"));
  g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(sym("ncclCommAbort"));
  g_nccl.GetErrorString = reinterpret_cast<decltype(g_nccl.GetErrorString)>(sym("ncclGetErrorString"));
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRankConfig || !g_nccl.CommGetAsyncError || !g_nccl.AllGather ||
      !g_nccl.CommFinalize || !g_nccl.CommDestroy || !g_nccl.CommAbort || !g_nccl.GetErrorString)
    return "libnccl.so.2 lacks a required symbol";
  g_nccl.handle = h;
  g_nccl.loaded = true;
  return nullptr;
}

// The communicator is non-blocking (so a rank that never joins cannot hang
// init), which means any NCCL call may return ncclInProgress with its work
// still being set up on NCCL's own threads (the first collective connects the
// peers).  Nothing else may be issued on the communicator or the stream until
// that finishes: poll its state, bounded by the library timeout.
ncclResult_t nccl_settle(ncclComm_t comm, ncclResult_t r) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(g_timeout_ms.load())) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (g_nccl.CommGetAsyncError(comm, &r) != ncclSuccess) return ncclSystemError;
  }
  return r;
}

}  // namespace

namespace sparsl {
// Lets other translation units report through sparsl_last_error and share
// the process-wide admission and quarantine state.
int record_error(int code, const char* message) { return fail(code, message, message); }
int record_error_detail(int code, const char* reason, const std::string& detail) { return fail(code, reason, detail); }
int check_device_array(const void* p, uint64_t bytes, int ordinal, const char* what);  // defined below
bool admission_enter() {
  g_admitted.fetch_add(1);
  return !g_quarantine.load();
}
void admission_leave() { g_admitted.fetch_sub(1); }
void quarantine_backend() { g_quarantine.store(true); }
uint64_t timeout_ms_setting() { return g_timeout_ms.load(); }
}  // namespace sparsl

// ==========================================================================
// Device
// ==========================================================================
struct sparsl_dev {
  int ordinal = 0;
  std::string name;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev = nullptr;
  std::mutex mu;
  ErrWord err;
  DBuf scan_in, scan_out, scan_scr;
  uint64_t scan_cap = 0;
  ScanScratch sc{};
  bool scan_dirty = false;
  DBuf lv, lth, lcur, lspk;
  DBuf vscratch;  // device CSR validation results, scan walk state
  DBuf tscratch;  // scan transfer tables
  DBuf cscratch;  // reverse-index sort scratch (sparsl_csc_from_csr_device)
  // Copy streams of the chunked host-buffer scan (created on first use).
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t up_ev = nullptr, scan_ev = nullptr, down_ev = nullptr;
};

namespace {
int dev_scan_prepare(sparsl_dev* d, uint64_t n) {
  if (d->scan_cap >= n && !d->scan_dirty && d->scan_scr.p) return SPARSL_OK;
  const uint64_t cap = std::max<uint64_t>(n, d->scan_cap);
  const size_t bytes = scan_scratch_bytes(cap);
  if (!d->scan_scr.p || d->scan_scr.bytes < bytes) {
    cudaStreamSynchronize(d->stream);
    dfree(d->scan_scr);
    if (dalloc(d->scan_scr, bytes, false, d->stream) != cudaSuccess)
      return fail(SPARSL_ERR_ALLOCATION, "scan scratch", "device allocation failed for scan scratch");
  }
  CK("assoc_scan", cudaMemsetAsync(d->scan_scr.p, 0, d->scan_scr.bytes, d->stream));
  d->sc = scan_scratch_carve(d->scan_scr.p, cap);
  d->scan_cap = cap;
  d->scan_dirty = false;
  return SPARSL_OK;
}
}  // namespace

// ==========================================================================
// Operator
// ==========================================================================
struct sparsl_op {
  sparsl_dev* dev = nullptr;
  uint32_t nrows = 0, ncols = 0, nnz = 0, max_row_nnz = 0;
  int precision = 0;
  bool has_t = false;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev = nullptr;
  std::mutex mu;
  ErrWord err;
  DBuf row_ptr, col, w;
  DBuf col_ptr, csc_row, csc_eidx;
  DBuf w_csc;  // the weights in reverse-index order: w_csc[k] = w[csc_eidx[k]]
  // Sliced-ELL copy of the reverse index for the transpose product (when its
  // padding stays bounded): slice offsets, row and edge index per entry, the
  // weights in that order, and the slice counter.
  bool sell_ok = false;
  uint32_t sell_slices = 0;
  uint64_t sell_total = 0;
  DBuf sell_ptr, sell_row, sell_eidx, w_sell, sell_ctr;
  // Uniform row length: TMA tensor maps over col / w as [nrows x L] matrices.
  EllMaps ell;
  // Uniform row length and x within kPanelMaxPanels shared-memory panels:
  // the tile-interleaved copy of col / w for the dense-x SpMV (panel.cu).
  PanelOp panel;
  DBuf pcol, pw, psplit;
  // The same for the transpose product, built from the sliced-ELL reverse
  // index when x (one value per row) fits the panels.
  PanelOp tpanel;
  DBuf tcol, tw, tsplit, ttoff;
  // Skewed rows: the rows in descending-length order, tile-interleaved, for
  // dense-x SpMV at high occupancy (panel.cu); its order is spmm_order.
  OrderedOp ordered;
  DBuf ocol, ow, olen, otoff;
  uint32_t ell_epoch = 0;  // tag of the last compacting TMA launch's flags
  // resident scratch (the write / step / sync API)
  DBuf rx, rxs[2], ry, rv, rth, rspk;
  int cur = 0;
  // compaction + trace
  DBuf idx_list, tile_flags, ticket, trace;
  // Recurrent ticks on the TMA path compact the spikes on a side stream,
  // concurrently with the next tick; done[b] marks the compaction that last
  // read spike buffer b (created on first use).
  cudaStream_t side = nullptr;
  cudaEvent_t tick_ev = nullptr, done_ev[2] = {nullptr, nullptr};
  // SpMM work units (rows by descending length unless all rows are equal)
  DBuf spmm_order, spmm_units, spmm_ctr;
  // Skewed row lengths: forward row folds walk rows in row_order (rows of
  // 32 or more entries by descending length, then the rest in index order).
  bool row_ordered = false;
  DBuf row_order;

  uint32_t spmm_nunits = 0, spmm_rows_per_unit = 1;
  // Row ranges of the host-buffer SpMM pipeline (empty: one launch): range k
  // is rows [range_row[k], range_row[k+1]) and units [range_unit[k],
  // range_unit[k+1]) of spmm_runits / spmm_rorder (of the plain units when
  // rows are equal).  Copy streams and events are created on first use.
  DBuf spmm_rorder, spmm_runits;
  std::vector<uint32_t> spmm_range_unit;
  std::vector<uint64_t> spmm_range_row;
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t up_ev = nullptr, fold_ev = nullptr, down_ev = nullptr;
  uint64_t trace_cap = 0, last_steps = 0;
  // staging for host-slice calls (kept apart from resident state, as the
  // reference CPU arm's slice API never touches its resident scratch)
  DBuf sx, sbits, sy, sv, sth, sspk;
  // Caller-owned device buffers bound as the SpMV x (ncols f32) and y
  // (nrows f32) in place of the operator's own (zero-copy interop).
  const float* ext_x = nullptr;
  float* ext_y = nullptr;
  uint64_t words() const { return packed_len(ncols); }
  const float* x_active() const { return ext_x ? ext_x : rx.as<float>(); }
  float* y_active() const { return ext_y ? ext_y : ry.as<float>(); }
};

namespace {

int wait_op(sparsl_op* op, const char* operation) {
  return wait_bounded(op->stream, op->ev, op->err.d, op->err.h, operation);
}

// Check every guarded buffer of the operator on its stream.
cudaError_t check_canaries(sparsl_op* op) {
  CanarySet set;
  auto add = [&](const DBuf& b) {
    if (b.p && b.guarded && set.count < CanarySet::kMax) set.ptr[set.count++] = b.canary();
  };
  add(op->ry);
  add(op->rv);
  add(op->rth);
  add(op->rspk);
  add(op->rxs[0]);
  add(op->rxs[1]);
  add(op->idx_list);
  add(op->trace);
  add(op->sy);
  add(op->sv);
  add(op->sth);
  add(op->sspk);
  return launch_canary_check(set, op->err.d, op->stream);
}

int finish(sparsl_op* op, const char* operation) {
  cudaError_t e = check_canaries(op);
  if (e != cudaSuccess) return fail_cuda(operation, e);
  return wait_op(op, operation);
}

int wkind_of(int precision) { return precision == 1 ? W_F16 : precision == 2 ? W_BF16 : W_F32; }

RowLaunch fwd_launch(sparsl_op* op) {
  RowLaunch p;
  p.ptr = op->row_ptr.as<uint32_t>();
  p.idx = op->col.as<uint32_t>();
  p.w = op->w.p;
  p.wkind = wkind_of(op->precision);
  p.nlines = op->nrows;
  p.err = op->err.d;
  p.tile_ticket = op->ticket.as<uint32_t>();
  return p;
}

// Forward launches take the TMA-pipelined kernel when the operator's rows all
// have the same length, the generic row-fold kernel otherwise.
cudaError_t launch_fwd(sparsl_op* op, const RowLaunch& p, cudaStream_t s) {
  if (op->panel.ok && p.xmode == X_DENSE && p.epilogue == EPI_ACCUM && !p.eidx && !p.out_bits && !p.idx_list)
    return launch_panel_spmv(op->panel, p.x, p.y, s);
  if (!op->ell.ok && op->row_ordered && !p.eidx) {
    // Skewed rows: warps fold rows in descending-length order; the packed
    // spike words (and from them the index list) come from the spike bytes.
    cudaError_t e;
    const bool bits = p.xmode != X_DENSE;
    if (op->ordered.ok && (!bits || (uint64_t)p.xbits_words * 4 <= kOrderedBitsMaxBytes)) {
      // The ordered fold: long rows a warp each, the rest 32 rows of similar
      // length per warp, no staging; a spike operand sits in shared memory.
      const bool lif = p.epilogue == EPI_LIF;
      e = launch_ordered_fold(op->ordered, bits ? nullptr : p.x, bits ? p.xbits : nullptr, bits ? p.xbits_words : 0,
                              lif ? nullptr : p.y, lif ? p.v : nullptr, lif ? p.theta : nullptr,
                              lif ? p.spikes : nullptr, p.decay, p.v_reset, p.dtheta, s,
                              LifHostState{p.v_src, p.theta_src, p.v_mirror, p.theta_mirror});
    } else {
      RowLaunch q = p;
      q.order = op->row_order.as<uint32_t>();
      q.out_bits = nullptr;
      q.idx_list = nullptr;
      q.idx_count = nullptr;
      e = launch_rows(q, s);
    }
    if (e != cudaSuccess || !p.out_bits) return e;
    const uint64_t words = ((uint64_t)p.nlines + 31) / 32;
    e = launch_pack(p.spikes, p.nlines, p.out_bits, words, s);
    if (e != cudaSuccess || !p.idx_list) return e;
    return launch_compact_bits(p.out_bits, words, p.idx_list, p.idx_count, p.idx_base, s);
  }
  if (!op->ell.ok) return launch_rows(p, s);
  if (!p.idx_list) return launch_ell(op->ell, p, s);
  if (p.out_bits && p.epilogue == EPI_LIF) {
    // A recurrent tick: the streaming kernel only writes the packed spikes,
    // and one small kernel turns them into the ascending index list.
    RowLaunch q = p;
    q.idx_list = nullptr;
    q.idx_count = nullptr;
    cudaError_t e = launch_ell(op->ell, q, s);
    if (e != cudaSuccess) return e;
    return launch_compact_bits(p.out_bits, ((uint64_t)p.nlines + 31) / 32, p.idx_list, p.idx_count, p.idx_base, s);
  }
  // Compacting launches tag their look-back flags with a fresh epoch; the
  // flags are cleared only when the 30-bit tag wraps.
  RowLaunch q = p;
  if (++op->ell_epoch >= (1u << 30)) {
    cudaError_t e = cudaMemsetAsync(op->tile_flags.p, 0, op->tile_flags.bytes, s);
    if (e != cudaSuccess) return e;
    op->ell_epoch = 1;
  }
  q.epoch = op->ell_epoch;
  return launch_ell(op->ell, q, s);
}

void set_bits_mode(RowLaunch& p, const uint32_t* bits, uint64_t words) {
  p.xbits = bits;
  p.xbits_words = (uint32_t)words;
  p.xmode = words <= kBitsSmemMaxWords ? X_BITS_SMEM : X_BITS_GLOBAL;
}

int check_len(const char* what, uint64_t got, uint64_t expected) {
  if (got == expected) return SPARSL_OK;
  return fail(SPARSL_ERR_LENGTH, what,
              std::string("`") + what + "` must have length " + std::to_string(expected) + ", got " +
                  std::to_string(got));
}
int check_min(const char* what, uint64_t got, uint64_t min) {
  if (got >= min) return SPARSL_OK;
  return fail(SPARSL_ERR_LENGTH, what,
              std::string("`") + what + "` must have length >= " + std::to_string(min) + ", got " +
                  std::to_string(got));
}

#define TRY(expr)                 \
  do {                            \
    int try_rc_ = (expr);         \
    if (try_rc_ != SPARSL_OK) return try_rc_; \
  } while (0)

#define ALLOC(buf, bytes, guard, what)                                                     \
  do {                                                                                     \
    if (ensure((buf), (bytes), (guard), op->stream) != cudaSuccess)                        \
      return fail(SPARSL_ERR_ALLOCATION, what, std::string("device allocation failed for ") + what); \
  } while (0)

int ensure_trace(sparsl_op* op, uint64_t steps) {
  if (op->trace.p && op->trace_cap >= steps) return SPARSL_OK;
  uint64_t cap = std::max<uint64_t>(steps, std::max<uint64_t>(1024, op->trace_cap * 2));
  ALLOC(op->trace, cap * 4, true, "spike trace");
  op->trace_cap = cap;
  return SPARSL_OK;
}

}  // namespace

// ==========================================================================
// C ABI
// ==========================================================================
extern "C" {

const char* sparsl_last_error(void) { return t_err.c_str(); }
const char* sparsl_last_reason(void) { return t_reason; }
const char* sparsl_version(void) { return "sparsl-cuda 0.1.0 (sm_100a)"; }
void sparsl_set_timeout_ms(uint64_t ms) { g_timeout_ms.store(ms ? ms : 1); }

int sparsl_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int sparsl_cuda_probe(const char** reason) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  const char* why = nullptr;
  if (e != cudaSuccess || n == 0) {
    why = "no CUDA device is visible to this process";
  } else {
    int sm100 = 0;
    for (int i = 0; i < n; ++i) {
      int major = 0, minor = 0;
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, i);
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, i);
      if (major == 10 && minor == 0) sm100 = 1;
    }
    if (!sm100) why = "no sm_100 (B200-class) device: this library is built for sm_100a only";
  }
  if (!why && g_quarantine.load()) why = "CUDA backend is quarantined after a failed or timed-out dispatch";
  if (reason) *reason = why;
  if (why) return fail(SPARSL_ERR_BACKEND, why, why);
  return SPARSL_OK;
}

int sparsl_device_open(int ordinal, sparsl_dev** out) {
  if (!out) return fail(SPARSL_ERR_INVALID, "null output", "sparsl_device_open: out is null");
  *out = nullptr;
  const char* why = nullptr;
  TRY(sparsl_cuda_probe(&why));
  int n = 0;
  cudaGetDeviceCount(&n);
  if (ordinal < 0 || ordinal >= n) return fail(SPARSL_ERR_BACKEND, "no such CUDA device", "ordinal out of range");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, ordinal);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, ordinal);
  if (major != 10 || minor != 0)
    return fail(SPARSL_ERR_BACKEND, "device is not sm_100", "the requested device is not sm_100 (B200-class)");
  CK("device_open", cudaSetDevice(ordinal));
  auto* d = new sparsl_dev();
  d->ordinal = ordinal;
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, ordinal);
  d->name = prop.name;
  d->sm_count = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = d->err.init();
  if (e != cudaSuccess) {
    delete d;
    return fail_cuda("device_open", e);
  }
  *out = d;
  return SPARSL_OK;
}

void sparsl_device_close(sparsl_dev* d) {
  if (!d) return;
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  dfree(d->scan_in);
  dfree(d->scan_out);
  dfree(d->scan_scr);
  dfree(d->lv);
  dfree(d->lth);
  dfree(d->lcur);
  dfree(d->lspk);
  dfree(d->vscratch);
  dfree(d->tscratch);
  dfree(d->cscratch);
  d->err.release();
  for (cudaStream_t st : {d->up, d->down})
    if (st) {
      cudaStreamSynchronize(st);
      cudaStreamDestroy(st);
    }
  for (cudaEvent_t e : {d->up_ev, d->scan_ev, d->down_ev})
    if (e) cudaEventDestroy(e);
  cudaEventDestroy(d->ev);
  cudaStreamDestroy(d->stream);
  delete d;
}

int sparsl_device_name(sparsl_dev* d, char* buf, size_t cap) {
  if (!d || !buf || cap == 0) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_device_name");
  std::snprintf(buf, cap, "%s", d->name.c_str());
  return SPARSL_OK;
}

int sparsl_device_reset(void) {
  // Refuse while any call is admitted (mod.rs:825-843) or while a dispatch
  // that timed out is still running on the GPU (metal.rs:440-445).
  if (g_admitted.load() > 0)
    return fail(SPARSL_ERR_BACKEND, "reset refused: admissions outstanding",
                "reset refused: a call is still admitted");
  {
    std::lock_guard<std::mutex> lk(g_timed_out_mu);
    for (cudaEvent_t e : g_timed_out) {
      const cudaError_t q = cudaEventQuery(e);
      if (q == cudaErrorNotReady)
        return fail(SPARSL_ERR_BACKEND, "reset refused: a timed-out dispatch is still running",
                    "reset refused: a dispatch that timed out has not completed on the GPU yet");
      if (q != cudaSuccess) cudaGetLastError();
    }
    for (cudaEvent_t e : g_timed_out) cudaEventDestroy(e);
    g_timed_out.clear();
  }
  g_quarantine.store(false);
  return SPARSL_OK;
}

int sparsl_quarantined(void) { return g_quarantine.load() ? 1 : 0; }

int sparsl_validate_csr(const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* col, uint64_t col_len,
                        uint64_t csr_ncols, uint64_t ncols, sparsl_shape* out) {
  PlanResult r = validate_csr(row_ptr, row_ptr_len, col, col_len, csr_ncols, ncols);
  if (out) {
    out->code = r.code;
    out->a = r.a;
    out->b = r.b;
    out->c = r.c;
    out->nrows = r.nrows;
    out->ncols = r.ncols;
    out->nnz = r.nnz;
    out->max_row_nnz = r.max_row_nnz;
  }
  if (r.code != PLAN_OK) return fail(SPARSL_ERR_INVALID, "invalid CSR", "CSR failed validation");
  return SPARSL_OK;
}

void sparsl_f32_to_f16_bits(const float* in, uint16_t* out, uint64_t n) { encode_narrow(1, in, out, n); }
void sparsl_f32_to_bf16_bits(const float* in, uint16_t* out, uint64_t n) { encode_narrow(2, in, out, n); }
void sparsl_quantise(int precision, const float* in, float* out, uint64_t n) { quantise(precision, in, out, n); }

// ---- device-level ops ----------------------------------------------------
int sparsl_dev_assoc_scan(sparsl_dev* d, const float* in, uint64_t n, float* out) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "assoc_scan: null device");
  if (n == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(d->mu);
  CK("assoc_scan", cudaSetDevice(d->ordinal));
  const size_t bytes = n * 8;
  if (ensure(d->scan_in, bytes, false, d->stream) != cudaSuccess ||
      ensure(d->scan_out, bytes, true, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "scan buffers", "device allocation failed for scan buffers");
  TRY(dev_scan_prepare(d, n));
  if (n < 2 * kScanPipeChunk) {
    CK("assoc_scan", cudaMemcpyAsync(d->scan_in.p, in, bytes, cudaMemcpyHostToDevice, d->stream));
    CK("assoc_scan", launch_scan(d->scan_in.as<float>(), d->scan_out.as<float>(), n, d->sc, d->err.d, d->stream));
    CK("assoc_scan", cudaMemcpyAsync(out, d->scan_out.p, bytes, cudaMemcpyDeviceToHost, d->stream));
  } else {
    // Chunked: chunk k's upload, chunk k-1's scan and chunk k-2's download
    // overlap (copy engines in both directions, the SMs).  Chunk k continues
    // from the last state chunk k-1 wrote (device memory, same stream), so
    // the result is the same single left fold.
    if (!d->up) {
      CK("assoc_scan", cudaStreamCreateWithFlags(&d->up, cudaStreamNonBlocking));
      CK("assoc_scan", cudaStreamCreateWithFlags(&d->down, cudaStreamNonBlocking));
      for (cudaEvent_t* e : {&d->up_ev, &d->scan_ev, &d->down_ev})
        CK("assoc_scan", cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    }
    CK("assoc_scan", cudaEventRecord(d->scan_ev, d->stream));  // after the scratch reset
    CK("assoc_scan", cudaStreamWaitEvent(d->up, d->scan_ev, 0));
    float* din = d->scan_in.as<float>();
    float* dout = d->scan_out.as<float>();
    for (uint64_t s0 = 0; s0 < n; s0 += kScanPipeChunk) {
      const uint64_t m = std::min<uint64_t>(kScanPipeChunk, n - s0);
      CK("assoc_scan", cudaMemcpyAsync(din + 2 * s0, in + 2 * s0, m * 8, cudaMemcpyHostToDevice, d->up));
      CK("assoc_scan", cudaEventRecord(d->up_ev, d->up));
      CK("assoc_scan", cudaStreamWaitEvent(d->stream, d->up_ev, 0));
      CK("assoc_scan", launch_scan(din + 2 * s0, dout + 2 * s0, m, d->sc, d->err.d, d->stream, nullptr,
                                   s0 ? dout + 2 * (s0 - 1) : nullptr));
      CK("assoc_scan", cudaEventRecord(d->scan_ev, d->stream));
      CK("assoc_scan", cudaStreamWaitEvent(d->down, d->scan_ev, 0));
      CK("assoc_scan", cudaMemcpyAsync(out + 2 * s0, dout + 2 * s0, m * 8, cudaMemcpyDeviceToHost, d->down));
    }
    CK("assoc_scan", cudaEventRecord(d->down_ev, d->down));
    CK("assoc_scan", cudaStreamWaitEvent(d->stream, d->down_ev, 0));
  }
  CanarySet set;
  set.ptr[set.count++] = d->scan_out.canary();
  CK("assoc_scan", launch_canary_check(set, d->err.d, d->stream));
  int rc = wait_bounded(d->stream, d->ev, d->err.d, d->err.h, "assoc_scan");
  if (rc != SPARSL_OK) d->scan_dirty = true;
  return rc;
}

int sparsl_dev_assoc_scan_device(sparsl_dev* d, const float* d_in, uint64_t n, float* d_out, void* stream) {
  return sparsl_dev_assoc_scan_from_device(d, d_in, n, d_out, nullptr, stream);
}

namespace {
int dev_scan(sparsl_dev* d, const float* d_in, uint64_t n, float* d_out, const float* entry, const float* entry_dev,
             void* stream) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "assoc_scan: null device");
  if (n == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(d->mu);
  CK("assoc_scan", cudaSetDevice(d->ordinal));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
  if (d->scan_cap < n || d->scan_dirty) {
    cudaStreamSynchronize(s);
    TRY(dev_scan_prepare(d, n));
    CK("assoc_scan", cudaStreamSynchronize(d->stream));
  }
  CK("assoc_scan", launch_scan(d_in, d_out, n, d->sc, d->err.d, s, entry, entry_dev));
  return SPARSL_OK;
}
}  // namespace

int sparsl_dev_assoc_scan_from_device(sparsl_dev* d, const float* d_in, uint64_t n, float* d_out, const float* entry,
                                      void* stream) {
  return dev_scan(d, d_in, n, d_out, entry, nullptr, stream);
}

int sparsl_dev_assoc_scan_after_device(sparsl_dev* d, const float* d_in, uint64_t n, float* d_out,
                                       const float* d_entry, void* stream) {
  if (!d_entry) return fail(SPARSL_ERR_INVALID, "null argument", "assoc_scan_after: a device entry state is required");
  return dev_scan(d, d_in, n, d_out, nullptr, d_entry, stream);
}

namespace {
// Lazily allocated per-device scratch of the split-scan pieces.
constexpr uint32_t kTabBlk = 1184;
int dev_split_scratch(sparsl_dev* d) {
  if (!d->tscratch.p && dalloc(d->tscratch, (kTabBlk + 64) * 4, false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "table scratch", "device allocation failed for scan table scratch");
  if (!d->vscratch.p && dalloc(d->vscratch, 32, false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "walk scratch", "device allocation failed for scan walk scratch");
  return SPARSL_OK;
}
}  // namespace

int sparsl_dev_scan_publish_device(sparsl_dev* d, const float* d_in, uint64_t n, int first, uint32_t halo,
                                   float* d_blob, void* stream) {
  ADMIT();
  if (!d || !d_in || !d_blob) return fail(SPARSL_ERR_INVALID, "null argument", "scan_publish: null argument");
  if (n == 0) return fail(SPARSL_ERR_LENGTH, "empty run", "scan_publish: a run needs at least one map");
  if (halo == 0 || halo > 4096) return fail(SPARSL_ERR_LENGTH, "halo", "scan_publish: halo must be 1..4096 maps");
  std::lock_guard<std::mutex> lk(d->mu);
  CK("scan_publish", cudaSetDevice(d->ordinal));
  TRY(dev_split_scratch(d));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
  CK("scan_publish", launch_scan_publish(d_in, n, first ? 1 : 0, halo, d_blob, d->tscratch.as<uint32_t>(), kTabBlk,
                                         d->vscratch.as<float>(), d->vscratch.as<unsigned long long>() + 1, s));
  return SPARSL_OK;
}

int sparsl_dev_scan_entry_device(sparsl_dev* d, const float* d_gathered, uint32_t world, uint32_t rank,
                                 uint32_t halo, float* d_entry, void* stream) {
  ADMIT();
  if (!d || !d_gathered || !d_entry) return fail(SPARSL_ERR_INVALID, "null argument", "scan_entry: null argument");
  if (rank == 0 || rank >= world || world > 64)
    return fail(SPARSL_ERR_INVALID, "rank", "scan_entry: needs 0 < rank < world <= 64");
  if (halo == 0 || halo > 4096) return fail(SPARSL_ERR_LENGTH, "halo", "scan_entry: halo must be 1..4096 maps");
  std::lock_guard<std::mutex> lk(d->mu);
  CK("scan_entry", cudaSetDevice(d->ordinal));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
  CK("scan_entry", launch_scan_entry(d_gathered, world, rank, halo, d_entry, s));
  return SPARSL_OK;
}

namespace {
int dev_scan_walk(sparsl_dev* d, const float* d_in, float* d_out, uint64_t n, const float* entry, int repair,
                  float* state, uint64_t* rewritten, void* stream, const char* what) {
  ADMIT();
  if (!d || !state) return fail(SPARSL_ERR_INVALID, "null argument", std::string(what) + ": null argument");
  if (n == 0) return fail(SPARSL_ERR_LENGTH, "empty run", std::string(what) + ": a run needs at least one map");
  std::lock_guard<std::mutex> lk(d->mu);
  CK(what, cudaSetDevice(d->ordinal));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
  if (!d->vscratch.p && dalloc(d->vscratch, 32, false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "walk scratch", "device allocation failed for scan walk scratch");
  float* dstate = d->vscratch.as<float>();
  unsigned long long* dstats = d->vscratch.as<unsigned long long>() + 1;
  CK(what, launch_scan_walk(d_in, d_out, n, entry, repair, dstate, dstats, s));
  unsigned long long h[2] = {0, 0};
  CK(what, cudaMemcpyAsync(h, d->vscratch.p, 16, cudaMemcpyDeviceToHost, s));
  CK(what, cudaStreamSynchronize(s));
  std::memcpy(state, h, 8);
  if (rewritten) *rewritten = h[1];
  return SPARSL_OK;
}
}  // namespace

int sparsl_dev_scan_fold_device(sparsl_dev* d, const float* d_in, uint64_t n, const float* entry, float* state,
                                void* stream) {
  return dev_scan_walk(d, d_in, nullptr, n, entry, 0, state, nullptr, stream, "scan_fold");
}

int sparsl_dev_scan_rejoin_device(sparsl_dev* d, const float* d_in, float* d_out, uint64_t n, const float* entry,
                                  float* exit_state, uint64_t* rewritten, void* stream) {
  if (!entry) return fail(SPARSL_ERR_INVALID, "null argument", "scan_rejoin: an entry state is required");
  return dev_scan_walk(d, d_in, d_out, n, entry, 1, exit_state, rewritten, stream, "scan_rejoin");
}

int sparsl_dev_scan_settle_device(sparsl_dev* d, const float* d_in, uint64_t n, float* multiplier,
                                  uint64_t* folded, void* stream) {
  float st[2] = {0.f, 0.f};
  TRY(dev_scan_walk(d, d_in, nullptr, n, nullptr, 2, st, folded, stream, "scan_settle"));
  if (multiplier) *multiplier = st[0];
  return SPARSL_OK;
}

int sparsl_dev_scan_table_device(sparsl_dev* d, const float* d_in, uint64_t n, uint32_t* table, void* stream) {
  ADMIT();
  if (!d || !table) return fail(SPARSL_ERR_INVALID, "null argument", "scan_table: null argument");
  if (n == 0) {
    *table = 0x76543210u;  // the identity table
    return SPARSL_OK;
  }
  std::lock_guard<std::mutex> lk(d->mu);
  CK("scan_table", cudaSetDevice(d->ordinal));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
  TRY(dev_split_scratch(d));
  uint32_t* out = d->tscratch.as<uint32_t>() + kTabBlk;
  CK("scan_table", launch_scan_table(d_in, n, d->tscratch.as<uint32_t>(), kTabBlk, out, s));
  CK("scan_table", cudaMemcpyAsync(table, out, 4, cudaMemcpyDeviceToHost, s));
  CK("scan_table", cudaStreamSynchronize(s));
  return SPARSL_OK;
}

int sparsl_dev_scan_stats(sparsl_dev* d, uint64_t* repaired, uint64_t* segments) {
  if (!d || !d->scan_scr.p) return fail(SPARSL_ERR_INVALID, "no scan has run", "no scan has run");
  std::lock_guard<std::mutex> lk(d->mu);
  uint32_t st[2] = {0, 0};
  CK("scan_stats", cudaSetDevice(d->ordinal));
  CK("scan_stats", cudaMemcpyAsync(st, d->sc.repair_stats, 8, cudaMemcpyDeviceToHost, d->stream));
  CK("scan_stats", cudaStreamSynchronize(d->stream));
  if (repaired) *repaired = st[0];
  if (segments) *segments = st[1];
  return SPARSL_OK;
}

int sparsl_dev_lif_integrate(sparsl_dev* d, float* v, float* theta, const float* cur, uint8_t* spk, uint64_t n,
                             float decay, float v_reset, float dtheta) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "lif_integrate: null device");
  if (n == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(d->mu);
  CK("lif_integrate", cudaSetDevice(d->ordinal));
  if (ensure(d->lv, n * 4, true, d->stream) != cudaSuccess || ensure(d->lth, n * 4, true, d->stream) != cudaSuccess ||
      ensure(d->lcur, n * 4, false, d->stream) != cudaSuccess || ensure(d->lspk, n, true, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "lif buffers", "device allocation failed for LIF buffers");
  CK("lif_integrate", cudaMemcpyAsync(d->lv.p, v, n * 4, cudaMemcpyHostToDevice, d->stream));
  CK("lif_integrate", cudaMemcpyAsync(d->lth.p, theta, n * 4, cudaMemcpyHostToDevice, d->stream));
  CK("lif_integrate", cudaMemcpyAsync(d->lcur.p, cur, n * 4, cudaMemcpyHostToDevice, d->stream));
  CK("lif_integrate", launch_lif_integrate(d->lv.as<float>(), d->lth.as<float>(), d->lcur.as<float>(),
                                           d->lspk.as<uint8_t>(), n, decay, v_reset, dtheta, d->stream));
  CK("lif_integrate", cudaMemcpyAsync(v, d->lv.p, n * 4, cudaMemcpyDeviceToHost, d->stream));
  CK("lif_integrate", cudaMemcpyAsync(theta, d->lth.p, n * 4, cudaMemcpyDeviceToHost, d->stream));
  CK("lif_integrate", cudaMemcpyAsync(spk, d->lspk.p, n, cudaMemcpyDeviceToHost, d->stream));
  CanarySet set;
  set.ptr[set.count++] = d->lv.canary();
  set.ptr[set.count++] = d->lth.canary();
  set.ptr[set.count++] = d->lspk.canary();
  CK("lif_integrate", launch_canary_check(set, d->err.d, d->stream));
  return wait_bounded(d->stream, d->ev, d->err.d, d->err.h, "lif_integrate");
}

int sparsl_dev_lif_integrate_device(sparsl_dev* d, float* d_v, float* d_theta, const float* d_cur, uint8_t* d_spk,
                                    uint64_t n, float decay, float v_reset, float dtheta, void* stream) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "lif_integrate: null device");
  if (n == 0) return SPARSL_OK;
  CK("lif_integrate", cudaSetDevice(d->ordinal));
  TRY(sparsl::check_device_array(d_v, n * 4, d->ordinal, "v"));
  TRY(sparsl::check_device_array(d_theta, n * 4, d->ordinal, "theta"));
  TRY(sparsl::check_device_array(d_cur, n * 4, d->ordinal, "currents"));
  TRY(sparsl::check_device_array(d_spk, n, d->ordinal, "spikes"));
  CK("lif_integrate", launch_lif_integrate(d_v, d_theta, d_cur, d_spk, n, decay, v_reset, dtheta,
                                           stream ? static_cast<cudaStream_t>(stream) : d->stream));
  return SPARSL_OK;
}

void* sparsl_dev_stream(sparsl_dev* d) { return d ? d->stream : nullptr; }
int sparsl_dev_test_expired_wait(sparsl_dev* d) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "test_expired_wait: null device");
  std::lock_guard<std::mutex> lk(d->mu);
  CK("test_expired_wait", cudaSetDevice(d->ordinal));
  if (ensure(d->vscratch, 32, false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "validation scratch", "device allocation failed for validation scratch");
  CK("test_expired_wait", launch_expired_wait(d->vscratch.p, d->err.d, d->stream));
  return wait_bounded(d->stream, d->ev, d->err.d, d->err.h, "test_expired_wait");
}

int sparsl_dev_wait(sparsl_dev* d) {
  if (!d) return fail(SPARSL_ERR_INVALID, "null device", "null device");
  cudaSetDevice(d->ordinal);
  return wait_bounded(d->stream, d->ev, d->err.d, d->err.h, "device wait");
}

// ---- operator ------------------------------------------------------------
namespace {

// Where an operator's CSR comes from.  row_ptr is always readable on the
// host (the device-source entry copies it there first: O(rows) bytes);
// col and weights are host pointers, or device pointers when `device`.
struct PrepSrc {
  const uint32_t* row_ptr;
  const uint32_t* d_row_ptr;  // device row_ptr (device sources), else null
  const uint32_t* col;
  const float* weights;
  bool device;
  bool borrow = false;  // device f32 sources the operator uses in place
};

void to_shape(const PlanResult& r, sparsl_shape* out) {
  out->code = r.code;
  out->a = r.a;
  out->b = r.b;
  out->c = r.c;
  out->nrows = r.nrows;
  out->ncols = r.ncols;
  out->nnz = r.nnz;
  out->max_row_nnz = r.max_row_nnz;
}

// The argument checks that follow validate_csr in SparseOp::prepare
// (src/backend/mod.rs:1305-1320): one weight per non-zero, a known precision.
int check_prepare_args(const sparsl_shape& sh, uint64_t weights_len, int precision, sparsl_shape* shape) {
  if (weights_len != sh.nnz) {
    if (shape) {
      shape->code = SPARSL_PLAN_WEIGHTS_LEN;
      shape->a = sh.nnz;
      shape->b = weights_len;
    }
    return fail(SPARSL_ERR_INVALID, "weights length", "weights must have one entry per non-zero");
  }
  if (precision < 0 || precision > 2) return fail(SPARSL_ERR_INVALID, "precision", "unknown weight precision");
  return SPARSL_OK;
}

// cuMemGetAddressRange through the runtime's driver entry point.
typedef int (*AddrRangeFn)(unsigned long long*, size_t*, unsigned long long);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<AddrRangeFn>(p);
    return (AddrRangeFn) nullptr;
  }();
  return fn;
}

// A caller's device array must be device (or managed) memory of this GPU
// and lie inside one allocation, so no kernel reading it leaves the
// allocation whatever the caller passed.
int check_device_span(const void* p, uint64_t bytes, int ordinal, const char* what) {
  if (bytes == 0) return SPARSL_OK;
  if (!p) return fail(SPARSL_ERR_INVALID, "null device array", std::string(what) + ": null device pointer");
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(SPARSL_ERR_INVALID, "not device memory", std::string(what) + ": not a device pointer");
  }
  if ((at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged) ||
      (at.type == cudaMemoryTypeDevice && at.device != ordinal))
    return fail(SPARSL_ERR_INVALID, "not device memory",
                std::string(what) + ": not device memory of GPU " + std::to_string(ordinal));
  if (at.type == cudaMemoryTypeDevice) {
    AddrRangeFn fn = addr_range_fn();
    unsigned long long base = 0;
    size_t size = 0;
    if (!fn || fn(&base, &size, reinterpret_cast<unsigned long long>(p)) != 0)
      return fail(SPARSL_ERR_INVALID, "not device memory", std::string(what) + ": no allocation holds it");
    const unsigned long long a = reinterpret_cast<unsigned long long>(p);
    if (a + bytes < a || a + bytes > base + size)
      return fail(SPARSL_ERR_INVALID, "device array too short",
                  std::string(what) + ": the array runs past the end of its allocation");
  }
  return SPARSL_OK;
}

}  // namespace
}  // extern "C"

// C++ linkage: shared with the allocation-free entry point (noalloc.cu).
namespace sparsl {
int check_device_array(const void* p, uint64_t bytes, int ordinal, const char* what) {
  return check_device_span(p, bytes, ordinal, what);
}
std::string describe_device_error(uint32_t bits) { return describe_dev_err(bits); }
}  // namespace sparsl

extern "C" {
namespace {

int prepare_body(sparsl_dev* d, const PrepSrc& src, const sparsl_shape& sh, int precision, int with_transpose,
                 sparsl_op** out);

// Device temporaries of one call, freed when it returns.
struct TmpBufs {
  DBuf row, eidx, keys, scratch, depth;
  ~TmpBufs() {
    for (DBuf* b : {&row, &eidx, &keys, &scratch, &depth}) dfree(*b);
  }
};

// The CSR gate (validate_csr) for arrays in device memory; `rp` receives
// the host copy of row_ptr.  Returns a status only for a CUDA failure; the
// gate's verdict is in *sh.
int gate_device(sparsl_dev* d, const uint32_t* d_row_ptr, uint64_t row_ptr_len, const uint32_t* d_col,
                uint64_t col_len, uint64_t csr_ncols, uint64_t ncols, std::vector<uint32_t>& rp, sparsl_shape* sh) {
  rp.assign(row_ptr_len, 0u);
  std::lock_guard<std::mutex> lk(d->mu);
  if (row_ptr_len)
    CK("validate", cudaMemcpyAsync(rp.data(), d_row_ptr, row_ptr_len * 4, cudaMemcpyDeviceToHost, d->stream));
  CK("validate", cudaStreamSynchronize(d->stream));
  if (!d->vscratch.p && dalloc(d->vscratch, 32, false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "validation scratch", "device allocation failed for validation scratch");
  PlanResult r{};
  CK("validate", validate_csr_device(rp.data(), row_ptr_len, d_row_ptr, d_col, col_len, csr_ncols, ncols,
                                     d->vscratch.as<unsigned long long>(), d->stream, &r));
  to_shape(r, sh);
  return SPARSL_OK;
}

}  // namespace

int sparsl_op_prepare(sparsl_dev* d, const uint32_t* row_ptr, uint64_t row_ptr_len, const uint32_t* col,
                      uint64_t col_len, uint64_t csr_ncols, uint64_t ncols, const float* weights,
                      uint64_t weights_len, int precision, int with_transpose, sparsl_shape* shape,
                      sparsl_op** out) {
  ADMIT();
  if (!out || !d) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_op_prepare: null argument");
  *out = nullptr;
  sparsl_shape sh{};
  int rc = sparsl_validate_csr(row_ptr, row_ptr_len, col, col_len, csr_ncols, ncols, &sh);
  if (shape) *shape = sh;
  if (rc != SPARSL_OK) return rc;
  TRY(check_prepare_args(sh, weights_len, precision, shape));
  return prepare_body(d, PrepSrc{row_ptr, nullptr, col, weights, false}, sh, precision, with_transpose, out);
}

int sparsl_op_prepare_device(sparsl_dev* d, const uint32_t* d_row_ptr, uint64_t row_ptr_len, const uint32_t* d_col,
                             uint64_t col_len, uint64_t csr_ncols, uint64_t ncols, const float* d_weights,
                             uint64_t weights_len, int precision, int with_transpose, sparsl_shape* shape,
                             sparsl_op** out) {
  ADMIT();
  if (!out || !d) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_op_prepare_device: null argument");
  *out = nullptr;
  CK("prepare_device", cudaSetDevice(d->ordinal));
  TRY(check_device_span(d_row_ptr, row_ptr_len * 4, d->ordinal, "row_ptr"));
  TRY(check_device_span(d_col, col_len * 4, d->ordinal, "col"));
  TRY(check_device_span(d_weights, weights_len * 4, d->ordinal, "weights"));
  std::vector<uint32_t> rp;
  sparsl_shape sh{};
  TRY(gate_device(d, d_row_ptr, row_ptr_len, d_col, col_len, csr_ncols, ncols, rp, &sh));
  if (shape) *shape = sh;
  if (sh.code != PLAN_OK) return fail(SPARSL_ERR_INVALID, "invalid CSR", "CSR failed validation");
  TRY(check_prepare_args(sh, weights_len, precision, shape));
  return prepare_body(d, PrepSrc{rp.data(), d_row_ptr, d_col, d_weights, true}, sh, precision, with_transpose, out);
}

namespace {
// A borrowed array must meet what the operator's own arrays guarantee every
// kernel: a kAlign-aligned start and kAlign bytes of the same allocation
// after its end (vector loads and staged tiles may read into that slack).
// Managed memory is refused: its allocation extent cannot be checked.
int check_borrowable(const void* p, uint64_t bytes, int ordinal, const char* what) {
  cudaPointerAttributes at{};
  if (p && cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type == cudaMemoryTypeManaged)
    return fail(SPARSL_ERR_INVALID, "not device memory", std::string(what) + ": managed memory cannot be borrowed");
  cudaGetLastError();
  int rc = check_device_span(p, bytes + kAlign, ordinal, what);
  if (rc != SPARSL_OK && std::string(sparsl_last_reason()) == "device array too short")
    return fail(SPARSL_ERR_INVALID, "device array too short",
                std::string(what) + ": a borrowed array must be followed by 256 bytes of its allocation");
  if (rc != SPARSL_OK) return rc;
  if (reinterpret_cast<uintptr_t>(p) % kAlign)
    return fail(SPARSL_ERR_INVALID, "misaligned device array",
                std::string(what) + ": a borrowed array must start on a 256-byte boundary");
  return SPARSL_OK;
}
}  // namespace

int sparsl_op_prepare_device_borrowed(sparsl_dev* d, const uint32_t* d_row_ptr, uint64_t row_ptr_len,
                                      const uint32_t* d_col, uint64_t col_len, uint64_t csr_ncols, uint64_t ncols,
                                      float* d_weights, uint64_t weights_len, int with_transpose,
                                      sparsl_shape* shape, sparsl_op** out) {
  ADMIT();
  if (!out || !d) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_op_prepare_device_borrowed: null argument");
  *out = nullptr;
  CK("prepare_device", cudaSetDevice(d->ordinal));
  TRY(check_borrowable(d_row_ptr, row_ptr_len * 4, d->ordinal, "row_ptr"));
  TRY(check_borrowable(d_col, col_len * 4, d->ordinal, "col"));
  TRY(check_borrowable(d_weights, weights_len * 4, d->ordinal, "weights"));
  std::vector<uint32_t> rp;
  sparsl_shape sh{};
  TRY(gate_device(d, d_row_ptr, row_ptr_len, d_col, col_len, csr_ncols, ncols, rp, &sh));
  if (shape) *shape = sh;
  if (sh.code != PLAN_OK) return fail(SPARSL_ERR_INVALID, "invalid CSR", "CSR failed validation");
  TRY(check_prepare_args(sh, weights_len, 0, shape));
  PrepSrc src{rp.data(), d_row_ptr, d_col, d_weights, true};
  src.borrow = true;
  return prepare_body(d, src, sh, 0, with_transpose, out);
}

int sparsl_csc_from_csr_device(sparsl_dev* d, const uint32_t* d_row_ptr, uint64_t row_ptr_len, const uint32_t* d_col,
                               uint64_t col_len, uint64_t ncols, uint32_t* d_col_ptr, uint32_t* d_row,
                               uint32_t* d_edge_idx, sparsl_shape* shape) {
  ADMIT();
  if (!d) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_csc_from_csr_device: null device");
  CK("csc_from_csr", cudaSetDevice(d->ordinal));
  TRY(check_device_span(d_row_ptr, row_ptr_len * 4, d->ordinal, "row_ptr"));
  TRY(check_device_span(d_col, col_len * 4, d->ordinal, "col"));
  std::vector<uint32_t> rp;
  sparsl_shape sh{};
  TRY(gate_device(d, d_row_ptr, row_ptr_len, d_col, col_len, ncols, ncols, rp, &sh));
  if (shape) *shape = sh;
  if (sh.code != PLAN_OK) return fail(SPARSL_ERR_INVALID, "invalid CSR", "CSR failed validation");
  // The gate bounds ncols and nnz by 2^32 - 1, so these sizes cannot overflow.
  TRY(check_device_span(d_col_ptr, (ncols + 1) * 4, d->ordinal, "col_ptr"));
  TRY(check_device_span(d_row, col_len * 4, d->ordinal, "row"));
  TRY(check_device_span(d_edge_idx, col_len * 4, d->ordinal, "edge_idx"));
  std::lock_guard<std::mutex> lk(d->mu);
  // The sort's scratch is kept on the device and grows only, so repeated
  // builds of similar size allocate nothing.
  if (ensure(d->cscratch, csc_scratch_bytes(sh.nnz), false, d->stream) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "reverse index", "device allocation failed for the reverse index");
  CK("csc_from_csr", csc_build(d_row_ptr, sh.nrows, d_col, sh.nnz, ncols, d_col_ptr, d_row, d_edge_idx, nullptr,
                               d->cscratch.p, d->err.d, d->stream));
  return wait_bounded(d->stream, d->ev, d->err.d, d->err.h, "csc_from_csr");
}

namespace {
int prepare_body(sparsl_dev* d, const PrepSrc& src, const sparsl_shape& sh, int precision, int with_transpose,
                 sparsl_op** out) {
  const uint32_t* row_ptr = src.row_ptr;
  int rc = SPARSL_OK;
  CK("prepare", cudaSetDevice(d->ordinal));
  auto* op = new sparsl_op();
  op->dev = d;
  op->nrows = (uint32_t)sh.nrows;
  op->ncols = (uint32_t)sh.ncols;
  op->nnz = (uint32_t)sh.nnz;
  op->max_row_nnz = (uint32_t)sh.max_row_nnz;
  op->precision = precision;
  op->has_t = with_transpose != 0;
  auto bail = [&](int code) {
    sparsl_op_destroy(op);
    return code;
  };
  if (cudaStreamCreateWithFlags(&op->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&op->ev, cudaEventDisableTiming) != cudaSuccess || op->err.init() != cudaSuccess)
    return bail(fail(SPARSL_ERR_BACKEND, "stream creation failed", "could not create operator stream"));
  const uint64_t nnz = sh.nnz, nrows = sh.nrows, nc = sh.ncols;
  const uint64_t words = packed_len(nc);
  const size_t wbytes = precision == 0 ? 4 : 2;
  // Every array gets 16 bytes of slack so vector loads near the end stay in bounds.
#define PALLOC(buf, bytes, guard, what)                                                    \
  do {                                                                                     \
    if (dalloc((buf), (bytes) + 16, (guard), op->stream) != cudaSuccess)                   \
      return bail(fail(SPARSL_ERR_ALLOCATION, what, std::string("device allocation failed for ") + what)); \
  } while (0)
  const bool borrow = src.borrow && nnz > 0;
  auto lend = [](DBuf& b, const void* p, size_t bytes) {
    b.p = const_cast<void*>(p);
    b.bytes = bytes;
    b.borrowed = true;
  };
  if (borrow) {
    lend(op->row_ptr, src.d_row_ptr, (nrows + 1) * 4);
    lend(op->col, src.col, nnz * 4);
    lend(op->w, src.weights, nnz * 4);
  } else {
    PALLOC(op->row_ptr, (nrows + 1) * 4, false, "row_ptr");
    PALLOC(op->col, nnz * 4, false, "col");
    PALLOC(op->w, nnz * wbytes, false, "values");
  }
  PALLOC(op->rx, nc * 4, false, "x");
  PALLOC(op->rxs[0], words * 4, true, "x_spikes");
  PALLOC(op->rxs[1], words * 4, true, "x_spikes");
  PALLOC(op->ry, nrows * 4, true, "y");
  PALLOC(op->rv, nrows * 4, true, "v");
  PALLOC(op->rth, nrows * 4, true, "theta");
  PALLOC(op->rspk, nrows, true, "spikes");
  PALLOC(op->idx_list, nrows * 4, true, "spike index list");
  PALLOC(op->tile_flags, ((uint64_t)std::max(row_tiles(op->nrows), ell_tiles(op->nrows)) + 1) * 8, false,
         "tile flags");
  PALLOC(op->ticket, 64, false, "tile ticket");
  const cudaMemcpyKind in_kind = src.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (!borrow && cudaMemcpyAsync(op->row_ptr.p, src.d_row_ptr ? src.d_row_ptr : row_ptr, (nrows + 1) * 4, in_kind,
                                 op->stream) != cudaSuccess)
    return bail(fail_cuda("prepare", cudaGetLastError()));
  if (nnz && !borrow) {
    if (cudaMemcpyAsync(op->col.p, src.col, nnz * 4, in_kind, op->stream) != cudaSuccess)
      return bail(fail_cuda("prepare", cudaGetLastError()));
  }
  std::vector<uint16_t> narrow;
  if (nnz && !borrow) {
    if (precision == 0) {
      if (cudaMemcpyAsync(op->w.p, src.weights, nnz * 4, in_kind, op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
    } else if (src.device) {
      // The same encoder as the host's, run on the GPU (codec.cuh).
      if (launch_encode_narrow(precision, src.weights, op->w.as<uint16_t>(), nnz, op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
    } else {
      narrow.resize(nnz);
      encode_narrow(precision, src.weights, narrow.data(), nnz);
      if (cudaMemcpyAsync(op->w.p, narrow.data(), nnz * 2, cudaMemcpyHostToDevice, op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
    }
  }
  std::vector<uint64_t> sell_ptr_h;
  if (op->has_t) {
    // The stable reverse index, built on the GPU from the uploaded CSR
    // (csc.cu) into temporaries; the operator keeps the sliced-ELL form or,
    // for hub-column operators, the CSC itself.
    PALLOC(op->col_ptr, (nc + 1) * 4, false, "csc col_ptr");
    TmpBufs tmp;
    const uint64_t nslices = (nc + 31) / 32;
    if (dalloc(tmp.row, nnz * 4, false, op->stream) != cudaSuccess ||
        dalloc(tmp.eidx, nnz * 4, false, op->stream) != cudaSuccess ||
        dalloc(tmp.keys, nnz * 4, false, op->stream) != cudaSuccess ||
        dalloc(tmp.scratch, csc_scratch_bytes(nnz), false, op->stream) != cudaSuccess ||
        dalloc(tmp.depth, nslices * 4, false, op->stream) != cudaSuccess)
      return bail(fail(SPARSL_ERR_ALLOCATION, "reverse index", "device allocation failed for the reverse index"));
    if (csc_build(op->row_ptr.as<uint32_t>(), nrows, op->col.as<uint32_t>(), nnz, nc, op->col_ptr.as<uint32_t>(),
                  tmp.row.as<uint32_t>(), tmp.eidx.as<uint32_t>(), tmp.keys.as<uint32_t>(), tmp.scratch.p, op->err.d,
                  op->stream) != cudaSuccess ||
        launch_slice_depth(op->col_ptr.as<uint32_t>(), nc, tmp.depth.as<uint32_t>(), op->stream) != cudaSuccess)
      return bail(fail_cuda("prepare", cudaGetLastError()));
    // Sliced ELL: slices of 32 columns, each padded to its longest column,
    // entries column-major within the slice.  Kept only while the padding at
    // most doubles the entries (a hub column would blow it up).
    std::vector<uint32_t> depth(nslices);
    if (nslices) {
      if (cudaMemcpyAsync(depth.data(), tmp.depth.p, nslices * 4, cudaMemcpyDeviceToHost, op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
    }
    rc = wait_op(op, "prepare");  // also reports a reverse-index look-back that gave up
    if (rc != SPARSL_OK) return bail(rc);
    std::vector<uint64_t> sp(nslices + 1, 0);
    for (uint64_t sl = 0; sl < nslices; ++sl) sp[sl + 1] = sp[sl] + (uint64_t)depth[sl] * 32;
    if (nnz && sp[nslices] <= 2 * nnz + 32 * nslices && nslices <= 0xffffffffull) {
      sell_ptr_h.swap(sp);
      op->sell_total = sell_ptr_h[nslices];
      op->sell_slices = (uint32_t)nslices;
      PALLOC(op->sell_ptr, (nslices + 1) * 8, false, "sliced-ELL offsets");
      PALLOC(op->sell_row, op->sell_total * 4, false, "sliced-ELL rows");
      PALLOC(op->sell_eidx, op->sell_total * 4, false, "sliced-ELL edge index");
      PALLOC(op->w_sell, op->sell_total * wbytes, false, "sliced-ELL values");
      PALLOC(op->sell_ctr, 16, false, "sliced-ELL counter");
      cudaMemcpyAsync(op->sell_ptr.p, sell_ptr_h.data(), (nslices + 1) * 8, cudaMemcpyHostToDevice, op->stream);
      cudaMemsetAsync(op->sell_row.p, 0, op->sell_total * 4, op->stream);
      cudaMemsetAsync(op->sell_eidx.p, 0, op->sell_total * 4, op->stream);
      cudaMemsetAsync(op->sell_ctr.p, 0, op->sell_ctr.bytes, op->stream);
      if (launch_sell_fill(op->col_ptr.as<uint32_t>(), tmp.keys.as<uint32_t>(), tmp.row.as<uint32_t>(),
                           tmp.eidx.as<uint32_t>(), nnz, op->sell_ptr.as<unsigned long long>(),
                           op->sell_row.as<uint32_t>(), op->sell_eidx.as<uint32_t>(), op->stream) != cudaSuccess ||
          launch_gather_weights(op->w.p, op->sell_eidx.as<uint32_t>(), op->sell_total, (int)wbytes, op->w_sell.p,
                                op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
      op->sell_ok = true;
      // The transpose product with x in shared-memory panels: the reverse
      // index's slices are already tiles of 32 lines; each is padded to a
      // multiple of 8 positions.
      uint32_t twidth = 0, tnp = 0;
      uint32_t max_depth = 0;
      for (uint64_t sl = 0; sl < nslices; ++sl) max_depth = std::max(max_depth, depth[sl]);
      if (!borrow && nnz <= (1ull << 30) && max_depth <= kPanelMaxRowLen && panel_geometry(nrows, twidth, tnp)) {
        std::vector<uint64_t> to(nslices + 1, 0);
        for (uint64_t sl = 0; sl < nslices; ++sl) to[sl + 1] = to[sl] + (depth[sl] + 7) / 8;
        PALLOC(op->ttoff, (nslices + 1) * 8, false, "transpose panel offsets");
        PALLOC(op->tcol, to[nslices] * 256 * 2, false, "transpose panel rows");
        PALLOC(op->tw, to[nslices] * 256 * wbytes, false, "transpose panel values");
        PALLOC(op->tsplit, nslices * 32 * (tnp + 1) * 2, false, "transpose panel split points");
        if (cudaMemcpyAsync(op->ttoff.p, to.data(), (nslices + 1) * 8, cudaMemcpyHostToDevice, op->stream) !=
                cudaSuccess ||
            launch_panel_build_sell(op->sell_ptr.as<unsigned long long>(), op->col_ptr.as<uint32_t>(),
                                    op->sell_row.as<uint32_t>(), nc, (uint32_t)nslices, op->ttoff.as<uint64_t>(),
                                    twidth, tnp, op->tcol.as<uint16_t>(), op->tsplit.as<uint16_t>(),
                                    op->stream) != cudaSuccess ||
            launch_panel_weights_sell(op->sell_ptr.as<unsigned long long>(), op->col_ptr.as<uint32_t>(),
                                      op->w_sell.p, nc, (uint32_t)nslices, op->ttoff.as<uint64_t>(), (int)wbytes,
                                      op->tw.p, op->stream) != cudaSuccess)
          return bail(fail_cuda("prepare", cudaGetLastError()));
        // The host offsets must outlive the asynchronous copy.
        rc = wait_op(op, "prepare");
        if (rc != SPARSL_OK) return bail(rc);
        PanelOp& tp = op->tpanel;
        tp.col16 = op->tcol.as<uint16_t>();
        tp.w = op->tw.p;
        tp.split = op->tsplit.as<uint16_t>();
        tp.toff = op->ttoff.as<uint64_t>();
        tp.wkind = wkind_of(precision);
        tp.nrows = (uint32_t)nc;
        tp.L = 0;
        tp.ncols = (uint32_t)nrows;
        tp.width = twidth;
        tp.npanels = tnp;
        tp.ok = true;
      }
    } else {
      std::swap(op->csc_row, tmp.row);
      std::swap(op->csc_eidx, tmp.eidx);
      // The transpose product streams its weights in reverse-index order
      // instead of gathering them through edge_idx (same products, same order).
      PALLOC(op->w_csc, nnz * wbytes, false, "csc values");
      if (nnz &&
          launch_gather_weights(op->w.p, op->csc_eidx.as<uint32_t>(), nnz, (int)wbytes, op->w_csc.p, op->stream) !=
              cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
    }
    rc = wait_op(op, "prepare");  // the temporaries are freed on return
    if (rc != SPARSL_OK) return bail(rc);
  }
  cudaMemsetAsync(op->rx.p, 0, op->rx.bytes, op->stream);
  cudaMemsetAsync(op->rxs[0].p, 0, op->rxs[0].bytes, op->stream);
  cudaMemsetAsync(op->rxs[1].p, 0, op->rxs[1].bytes, op->stream);
  cudaMemsetAsync(op->ry.p, 0, op->ry.bytes, op->stream);
  cudaMemsetAsync(op->rv.p, 0, op->rv.bytes, op->stream);
  cudaMemsetAsync(op->rth.p, 0, op->rth.bytes, op->stream);
  cudaMemsetAsync(op->rspk.p, 0, op->rspk.bytes, op->stream);
  cudaMemsetAsync(op->tile_flags.p, 0, op->tile_flags.bytes, op->stream);
  cudaMemsetAsync(op->ticket.p, 0, op->ticket.bytes, op->stream);
  // Uniform row length (fixed fan-in / fixed degree): enable the TMA path.
  if (nrows && nnz && nnz % nrows == 0) {
    const uint64_t L = nnz / nrows;
    bool uniform = L <= 0xffffffffull;
    for (uint64_t r = 0; uniform && r <= nrows; ++r) uniform = (uint64_t)row_ptr[r] == r * L;
    if (uniform) ell_encode(op->ell, op->col.as<uint32_t>(), op->w.p, wkind_of(precision), nrows, (uint32_t)L);
    // Dense-x SpMV with x in shared memory: the operator's own (not a
    // borrowed) arrays, interleaved by tiles of 32 rows, up to 2^30 entries.
    uint32_t width = 0, npanels = 0;
    if (uniform && !borrow && nnz <= (1ull << 30) && L <= kPanelMaxRowLen &&
        panel_geometry(op->ncols, width, npanels)) {
      PALLOC(op->pcol, panel_col_elems(nrows, (uint32_t)L) * 2, false, "interleaved col");
      PALLOC(op->pw, panel_w_elems(nrows, (uint32_t)L) * wbytes, false, "interleaved values");
      PALLOC(op->psplit, panel_split_elems(nrows, npanels) * 2, false, "panel split points");
      if (launch_panel_build(op->col.as<uint32_t>(), nrows, (uint32_t)L, width, npanels, op->pcol.as<uint16_t>(),
                             op->psplit.as<uint16_t>(), op->stream) != cudaSuccess ||
          launch_panel_weights(op->w.p, nrows, (uint32_t)L, (int)wbytes, op->pw.p, op->stream) != cudaSuccess)
        return bail(fail_cuda("prepare", cudaGetLastError()));
      PanelOp& pn = op->panel;
      pn.col16 = op->pcol.as<uint16_t>();
      pn.w = op->pw.p;
      pn.split = op->psplit.as<uint16_t>();
      pn.wkind = wkind_of(precision);
      pn.nrows = (uint32_t)nrows;
      pn.L = (uint32_t)L;
      pn.ncols = op->ncols;
      pn.width = width;
      pn.npanels = npanels;
      pn.ok = true;
    }
  }
  // SpMM work units.  Equal rows: fixed runs of rows.  Otherwise rows by
  // descending length (ties by index), cut into units of >= kSpmmUnitNnz
  // entries or a single row, at most kSpmmUnitRows rows each.  Operators of
  // kSpmmRangeMinRows rows or more also get units per range of consecutive
  // rows (the host-buffer pipeline launches one range at a time); for equal
  // rows those are runs of the same units.
  std::vector<uint32_t> sp_order, sp_units, rg_order, rg_units;
  PALLOC(op->spmm_ctr, 16, false, "spmm counters");
  cudaMemsetAsync(op->spmm_ctr.p, 0, op->spmm_ctr.bytes, op->stream);
  if (nrows) {
    const uint32_t maxlen = (uint32_t)sh.max_row_nnz;
    uint32_t minlen = maxlen;
    for (uint64_t r = 0; r < nrows && minlen; ++r) minlen = std::min(minlen, row_ptr[r + 1] - row_ptr[r]);
    const bool ranged = nrows >= kSpmmRangeMinRows;
    if (minlen == maxlen) {
      const uint32_t R = std::max(1u, std::min(kSpmmUnitRows, kSpmmUnitNnz / std::max(maxlen, 1u)));
      op->spmm_rows_per_unit = R;
      op->spmm_nunits = (uint32_t)((nrows + R - 1) / R);
      if (ranged) {
        const uint64_t per = ((op->spmm_nunits + kSpmmRanges - 1) / kSpmmRanges);
        for (uint64_t k = 0; k <= kSpmmRanges; ++k) {
          const uint64_t u = std::min<uint64_t>(k * per, op->spmm_nunits);
          op->spmm_range_unit.push_back((uint32_t)u);
          op->spmm_range_row.push_back(std::min<uint64_t>(u * R, nrows));
        }
      }
    } else {
      auto len = [&](uint64_t r) { return row_ptr[r + 1] - row_ptr[r]; };
      // Rows [r0, r1) by descending length, appended to `order`, and their
      // units appended to `units` (positions in `order`).
      auto build = [&](uint64_t r0, uint64_t r1, std::vector<uint32_t>& order, std::vector<uint32_t>& units) {
        const size_t base = order.size();
        order.resize(base + (r1 - r0));
        uint32_t* o = order.data() + base;
        if ((uint64_t)maxlen <= 4 * (r1 - r0) + 4096) {
          // Counting sort by length (descending, stable).
          std::vector<uint32_t> start((size_t)maxlen + 2, 0);
          for (uint64_t r = r0; r < r1; ++r) ++start[maxlen - len(r) + 1];
          for (size_t k = 1; k < start.size(); ++k) start[k] += start[k - 1];
          for (uint64_t r = r0; r < r1; ++r) o[start[maxlen - len(r)]++] = (uint32_t)r;
        } else {
          for (uint64_t r = r0; r < r1; ++r) o[r - r0] = (uint32_t)r;
          std::stable_sort(o, o + (r1 - r0), [&](uint32_t a, uint32_t b) { return len(a) > len(b); });
        }
        if (units.empty()) units.push_back(0);
        uint64_t acc = 0, rows_in = 0;
        for (uint64_t i = base; i < order.size(); ++i) {
          acc += len(order[i]);
          ++rows_in;
          if (acc >= kSpmmUnitNnz || rows_in >= kSpmmUnitRows || i + 1 == order.size()) {
            units.push_back((uint32_t)(i + 1));
            acc = rows_in = 0;
          }
        }
      };
      build(0, nrows, sp_order, sp_units);
      op->spmm_nunits = (uint32_t)(sp_units.size() - 1);
      // Row folds take the descending-length order when a natural-order warp
      // would often idle behind one long row: the longest row exceeds both
      // one staging chunk and four times the mean (a function of the shape).
      op->row_ordered = maxlen > 32 && (uint64_t)maxlen * nrows > 4 * (uint64_t)nnz;
      if (op->row_ordered) {
        // Rows of a staging chunk or more (32 entries), longest first, then
        // the shorter rows in their natural order, so runs of consecutive
        // short rows keep coalesced loads and stores.
        std::vector<uint32_t> ro;
        ro.reserve(nrows);
        for (uint64_t i = 0; i < nrows && len(sp_order[i]) >= 32; ++i) ro.push_back(sp_order[i]);
        for (uint64_t r = 0; r < nrows; ++r)
          if (len(r) < 32) ro.push_back((uint32_t)r);
        PALLOC(op->row_order, nrows * 4, false, "row order");
        cudaMemcpyAsync(op->row_order.p, ro.data(), nrows * 4, cudaMemcpyHostToDevice, op->stream);
        cudaStreamSynchronize(op->stream);
      }
      PALLOC(op->spmm_order, nrows * 4, false, "spmm row order");
      PALLOC(op->spmm_units, sp_units.size() * 4, false, "spmm units");
      cudaMemcpyAsync(op->spmm_order.p, sp_order.data(), nrows * 4, cudaMemcpyHostToDevice, op->stream);
      cudaMemcpyAsync(op->spmm_units.p, sp_units.data(), sp_units.size() * 4, cudaMemcpyHostToDevice, op->stream);
      // Skewed rows, the operator's own arrays, up to 2^30 entries: the
      // ordered fold.  The rows of kOrderedLongRow entries or more (a prefix
      // of the descending order) are folded one warp each from the CSR
      // arrays; tile T of the copy holds rows sp_order[nlong + 32T ..], padded
      // to its first (longest) row, rounded up to 8.
      if (op->row_ordered && !borrow && nnz <= (1ull << 30)) {
        uint64_t nlong = 0;
        while (nlong < nrows && len(sp_order[nlong]) >= kOrderedLongRow) ++nlong;
        const uint64_t nshort = nrows - nlong, nt = (nshort + 31) / 32;
        std::vector<uint64_t> to(nt + 1, 0);
        for (uint64_t T = 0; T < nt; ++T) to[T + 1] = to[T] + (len(sp_order[nlong + T * 32]) + 7) / 8;
        PALLOC(op->otoff, (nt + 1) * 8, false, "ordered offsets");
        PALLOC(op->ocol, to[nt] * 256 * 4, false, "ordered col");
        PALLOC(op->ow, to[nt] * 256 * wbytes, false, "ordered values");
        PALLOC(op->olen, nt * 32 * 4, false, "ordered lengths");
        if (cudaMemcpyAsync(op->otoff.p, to.data(), (nt + 1) * 8, cudaMemcpyHostToDevice, op->stream) !=
                cudaSuccess ||
            launch_ordered_build(op->row_ptr.as<uint32_t>(), op->col.as<uint32_t>(), op->w.p, (int)wbytes,
                                 op->spmm_order.as<uint32_t>() + nlong, nshort, op->otoff.as<uint64_t>(),
                                 op->ocol.as<uint32_t>(), op->ow.p, op->olen.as<uint32_t>(), op->stream) !=
                cudaSuccess)
          return bail(fail_cuda("prepare", cudaGetLastError()));
        cudaStreamSynchronize(op->stream);  // the host offsets outlive the copy
        OrderedOp& od = op->ordered;
        od.col = op->ocol.as<uint32_t>();
        od.w = op->ow.p;
        od.len = op->olen.as<uint32_t>();
        od.toff = op->otoff.as<uint64_t>();
        od.order = op->spmm_order.as<uint32_t>();
        od.row_ptr = op->row_ptr.as<uint32_t>();
        od.csr_col = op->col.as<uint32_t>();
        od.csr_w = op->w.p;
        od.wkind = wkind_of(precision);
        od.nrows = (uint32_t)nrows;
        od.nlong = (uint32_t)nlong;
        od.ok = true;
      }
      if (ranged) {
        const uint64_t per = (nrows + kSpmmRanges - 1) / kSpmmRanges;
        op->spmm_range_unit.push_back(0);
        op->spmm_range_row.push_back(0);
        for (uint64_t k = 0; k < kSpmmRanges; ++k) {
          const uint64_t r0 = std::min(k * per, nrows), r1 = std::min((k + 1) * per, nrows);
          if (r1 > r0) build(r0, r1, rg_order, rg_units);
          op->spmm_range_unit.push_back(rg_units.empty() ? 0 : (uint32_t)(rg_units.size() - 1));
          op->spmm_range_row.push_back(r1);
        }
        PALLOC(op->spmm_rorder, nrows * 4, false, "spmm ranged row order");
        PALLOC(op->spmm_runits, rg_units.size() * 4, false, "spmm ranged units");
        cudaMemcpyAsync(op->spmm_rorder.p, rg_order.data(), nrows * 4, cudaMemcpyHostToDevice, op->stream);
        cudaMemcpyAsync(op->spmm_runits.p, rg_units.data(), rg_units.size() * 4, cudaMemcpyHostToDevice,
                        op->stream);
      }
    }
  }
  rc = wait_op(op, "prepare");  // host vectors above must outlive the copies
  if (rc != SPARSL_OK) return bail(rc);
#undef PALLOC
  *out = op;
  return SPARSL_OK;
}
}  // namespace

void sparsl_op_destroy(sparsl_op* op) {
  if (!op) return;
  cudaSetDevice(op->dev->ordinal);
  if (op->stream) cudaStreamSynchronize(op->stream);
  DBuf* bufs[] = {&op->row_ptr, &op->col,     &op->w,       &op->col_ptr, &op->csc_row, &op->csc_eidx, &op->w_csc,
                  &op->sell_ptr, &op->sell_row, &op->sell_eidx, &op->w_sell, &op->sell_ctr,
                  &op->rx,      &op->rxs[0],  &op->rxs[1],  &op->ry,      &op->rv,      &op->rth,
                  &op->rspk,    &op->idx_list, &op->tile_flags, &op->ticket, &op->trace, &op->sx,
                  &op->sbits,   &op->sy,      &op->sv,      &op->sth,     &op->sspk,
                  &op->spmm_order, &op->spmm_units, &op->spmm_ctr, &op->spmm_rorder, &op->spmm_runits,
                  &op->row_order, &op->pcol, &op->pw, &op->psplit, &op->tcol, &op->tw, &op->tsplit, &op->ttoff,
                  &op->ocol, &op->ow, &op->olen, &op->otoff};
  for (DBuf* b : bufs) dfree(*b);
  op->err.release();
  if (op->side) cudaStreamSynchronize(op->side);
  for (cudaEvent_t e : {op->tick_ev, op->done_ev[0], op->done_ev[1]})
    if (e) cudaEventDestroy(e);
  if (op->side) cudaStreamDestroy(op->side);
  for (cudaStream_t st : {op->up, op->down})
    if (st) {
      cudaStreamSynchronize(st);
      cudaStreamDestroy(st);
    }
  for (cudaEvent_t e : {op->up_ev, op->fold_ev, op->down_ev})
    if (e) cudaEventDestroy(e);
  if (op->ev) cudaEventDestroy(op->ev);
  if (op->stream) cudaStreamDestroy(op->stream);
  delete op;
}

int sparsl_op_shape(sparsl_op* op, sparsl_shape* out) {
  if (!op || !out) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_op_shape");
  *out = sparsl_shape{};
  out->nrows = op->nrows;
  out->ncols = op->ncols;
  out->nnz = op->nnz;
  out->max_row_nnz = op->max_row_nnz;
  return SPARSL_OK;
}

int sparsl_op_weight_precision(sparsl_op* op) { return op ? op->precision : -1; }
int sparsl_op_layouts(sparsl_op* op) {
  if (!op) return 0;
  return (op->ell.ok ? SPARSL_LAYOUT_ELL : 0) | (op->row_ordered ? SPARSL_LAYOUT_ROW_ORDER : 0) |
         (op->panel.ok ? SPARSL_LAYOUT_X_PANELS : 0) | (op->tpanel.ok ? SPARSL_LAYOUT_T_X_PANELS : 0) |
         (op->ordered.ok ? SPARSL_LAYOUT_ORDERED_COPY : 0) |
         (op->sell_ok ? SPARSL_LAYOUT_SLICED_REVERSE : 0) |
         (op->has_t && !op->sell_ok ? SPARSL_LAYOUT_CSC : 0);
}
int sparsl_op_has_transpose(sparsl_op* op) { return op && op->has_t ? 1 : 0; }

int sparsl_op_test_mark_canary(sparsl_op* op) {
  ADMIT();
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "test_mark_canary: null operator");
  std::lock_guard<std::mutex> lk(op->mu);
  CK("test_mark_canary", cudaSetDevice(op->dev->ordinal));
  // The host writes one word of y's canary tail (inside the allocation), as
  // an out-of-bounds kernel write within the tail would.
  static const uint32_t kMark = 0;
  CK("test_mark_canary", cudaMemcpyAsync(const_cast<uint32_t*>(op->ry.canary()), &kMark, sizeof kMark,
                                         cudaMemcpyHostToDevice, op->stream));
  return finish(op, "test_mark_canary");
}

int sparsl_op_force_plain_row_fold(sparsl_op* op) {
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_op_force_plain_row_fold: null operator");
  std::lock_guard<std::mutex> lk(op->mu);
  // The tensor maps are host-side descriptors over the operator's own col /
  // weight arrays; clearing the flags is all it takes to route every later
  // forward launch through the generic row fold in natural row order.
  op->ell.ok = false;
  op->row_ordered = false;
  op->panel.ok = false;
  op->tpanel.ok = false;
  op->ordered.ok = false;
  return SPARSL_OK;
}

int sparsl_op_set_weights(sparsl_op* op, const float* weights, uint64_t n) {
  ADMIT();
  TRY(check_len("weights", n, op->nnz));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("set_weights", cudaSetDevice(op->dev->ordinal));
  if (n == 0) return SPARSL_OK;
  std::vector<uint16_t> narrow;
  if (op->precision == 0) {
    CK("set_weights", cudaMemcpyAsync(op->w.p, weights, n * 4, cudaMemcpyHostToDevice, op->stream));
  } else {
    narrow.resize(n);
    encode_narrow(op->precision, weights, narrow.data(), n);
    CK("set_weights", cudaMemcpyAsync(op->w.p, narrow.data(), n * 2, cudaMemcpyHostToDevice, op->stream));
  }
  if (op->ordered.ok)
    CK("set_weights", launch_ordered_weights(op->row_ptr.as<uint32_t>(), op->w.p, op->precision == 0 ? 4 : 2,
                                             op->ordered.order + op->ordered.nlong,
                                             op->nrows - op->ordered.nlong, op->ordered.toff, op->ow.p,
                                             op->stream));
  if (op->panel.ok)
    CK("set_weights", launch_panel_weights(op->w.p, op->nrows, op->panel.L, op->precision == 0 ? 4 : 2, op->pw.p,
                                           op->stream));
  if (op->sell_ok)
    CK("set_weights", launch_gather_weights(op->w.p, op->sell_eidx.as<uint32_t>(), op->sell_total,
                                            op->precision == 0 ? 4 : 2, op->w_sell.p, op->stream));
  if (op->tpanel.ok)
    CK("set_weights", launch_panel_weights_sell(op->sell_ptr.as<unsigned long long>(), op->col_ptr.as<uint32_t>(),
                                                op->w_sell.p, op->ncols, op->sell_slices, op->tpanel.toff,
                                                op->precision == 0 ? 4 : 2, op->tw.p, op->stream));
  else if (op->has_t)
    CK("set_weights", launch_gather_weights(op->w.p, op->csc_eidx.as<uint32_t>(), n, op->precision == 0 ? 4 : 2,
                                            op->w_csc.p, op->stream));
  return wait_op(op, "set_weights");
}

// True when ptr is pinned host memory that the current device can address;
// *dptr is then that address.  Such memory can be read and written by
// kernels directly, over PCIe.
static bool host_mapped(const void* ptr, void** dptr) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();  // an unknown pointer is not an error here
    return false;
  }
  *dptr = a.devicePointer;
  return a.type == cudaMemoryTypeHost && a.devicePointer != nullptr;
}

int sparsl_op_spmv(sparsl_op* op, const float* x, uint64_t x_len, float* y, uint64_t y_len) {
  ADMIT();
  TRY(check_min("x", x_len, op->ncols));
  TRY(check_len("y", y_len, op->nrows));
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spmv", cudaSetDevice(op->dev->ordinal));
  // A bound x is read in place of the slice; a bound y is accumulated into
  // and then read back into the slice (metal.rs:2143-2170).
  RowLaunch p = fwd_launch(op);
  if (op->ext_x) {
    p.x = op->ext_x;
  } else {
    ALLOC(op->sx, (uint64_t)op->ncols * 4 + 16, false, "x staging");
    if (op->ncols)
      CK("spmv", cudaMemcpyAsync(op->sx.p, x, (uint64_t)op->ncols * 4, cudaMemcpyHostToDevice, op->stream));
    p.x = op->sx.as<float>();
  }
  // A pinned y (and no bound y) is accumulated into in place, over PCIe.
  void* dy = nullptr;
  const bool mapped = !op->ext_y && host_mapped(y, &dy);
  if (op->ext_y) {
    p.y = op->ext_y;
  } else if (mapped) {
    p.y = static_cast<float*>(dy);
  } else {
    ALLOC(op->sy, (uint64_t)op->nrows * 4 + 16, true, "y staging");
    CK("spmv", cudaMemcpyAsync(op->sy.p, y, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, op->stream));
    p.y = op->sy.as<float>();
  }
  CK("spmv", launch_fwd(op, p, op->stream));
  if (!mapped) CK("spmv", cudaMemcpyAsync(y, p.y, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "spmv");
}

int sparsl_op_spmv_spikes(sparsl_op* op, const uint32_t* spikes, uint64_t words, float* y, uint64_t y_len) {
  ADMIT();
  TRY(check_min("spikes", words, op->words()));
  TRY(check_len("y", y_len, op->nrows));
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spmv_spikes", cudaSetDevice(op->dev->ordinal));
  ALLOC(op->sbits, op->words() * 4 + 16, false, "spike staging");
  if (op->words())
    CK("spmv_spikes", cudaMemcpyAsync(op->sbits.p, spikes, op->words() * 4, cudaMemcpyHostToDevice, op->stream));
  RowLaunch p = fwd_launch(op);
  set_bits_mode(p, op->sbits.as<uint32_t>(), op->words());
  // A pinned y is accumulated into in place, over PCIe.
  void* dy = nullptr;
  const bool mapped = host_mapped(y, &dy);
  if (mapped) {
    p.y = static_cast<float*>(dy);
  } else {
    ALLOC(op->sy, (uint64_t)op->nrows * 4 + 16, true, "y staging");
    CK("spmv_spikes", cudaMemcpyAsync(op->sy.p, y, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, op->stream));
    p.y = op->sy.as<float>();
  }
  CK("spmv_spikes", launch_fwd(op, p, op->stream));
  if (!mapped)
    CK("spmv_spikes", cudaMemcpyAsync(y, op->sy.p, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "spmv_spikes");
}

// The transpose product: the sliced-ELL fold when the operator has it, the
// row-fold engine over the CSC lines otherwise.
static cudaError_t launch_transpose(sparsl_op* op, const float* x, float* y, cudaStream_t s) {
  if (op->tpanel.ok) return launch_panel_spmv(op->tpanel, x, y, s);
  if (op->sell_ok) {
    SellLaunch p;
    p.slice_ptr = op->sell_ptr.as<uint64_t>();
    p.line_ptr = op->col_ptr.as<uint32_t>();
    p.idx = op->sell_row.as<uint32_t>();
    p.w = op->w_sell.p;
    p.wkind = wkind_of(op->precision);
    p.x = x;
    p.y = y;
    p.nlines = op->ncols;
    p.nslices = op->sell_slices;
    p.ctr = op->sell_ctr.as<uint32_t>();
    return launch_sell(p, op->dev->sm_count, s);
  }
  RowLaunch p;
  p.ptr = op->col_ptr.as<uint32_t>();
  p.idx = op->csc_row.as<uint32_t>();
  p.w = op->w_csc.p;  // reverse-index order: a plain row fold over the CSC lines
  p.wkind = wkind_of(op->precision);
  p.nlines = op->ncols;
  p.x = x;
  p.y = y;
  p.err = op->err.d;
  return launch_rows(p, s);
}

int sparsl_op_spmv_t(sparsl_op* op, const float* x, uint64_t x_len, float* y, uint64_t y_len) {
  ADMIT();
  TRY(check_min("x", x_len, op->nrows));
  TRY(check_len("y", y_len, op->ncols));
  if (op->ncols == 0) return SPARSL_OK;
  if (!op->has_t)
    return fail(SPARSL_ERR_NO_TRANSPOSE, "transpose not prepared",
                "this operator has no reverse index; build it with prepare_with_transpose to use spmv_t");
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spmv_t", cudaSetDevice(op->dev->ordinal));
  ALLOC(op->sx, (uint64_t)std::max(op->nrows, op->ncols) * 4 + 16, false, "x staging");
  ALLOC(op->sy, (uint64_t)std::max(op->nrows, op->ncols) * 4 + 16, true, "y staging");
  if (op->nrows) CK("spmv_t", cudaMemcpyAsync(op->sx.p, x, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, op->stream));
  CK("spmv_t", cudaMemcpyAsync(op->sy.p, y, (uint64_t)op->ncols * 4, cudaMemcpyHostToDevice, op->stream));
  CK("spmv_t", launch_transpose(op, op->sx.as<float>(), op->sy.as<float>(), op->stream));
  CK("spmv_t", cudaMemcpyAsync(y, op->sy.p, (uint64_t)op->ncols * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "spmv_t");
}

static SpmmLaunch spmm_launch(sparsl_op* op, const float* x, float* y, uint32_t n_vec) {
  SpmmLaunch p;
  p.ptr = op->row_ptr.as<uint32_t>();
  p.idx = op->col.as<uint32_t>();
  p.w = op->w.p;
  p.wkind = wkind_of(op->precision);
  p.x = x;
  p.y = y;
  p.nrows = op->nrows;
  p.n_vec = n_vec;
  p.order = op->spmm_order.p ? op->spmm_order.as<uint32_t>() : nullptr;
  p.unit_start = op->spmm_units.p ? op->spmm_units.as<uint32_t>() : nullptr;
  p.nunits = op->spmm_nunits;
  p.rows_per_unit = op->spmm_rows_per_unit;
  p.ctr = op->spmm_ctr.as<uint32_t>();
  return p;
}

int sparsl_op_spmm(sparsl_op* op, const float* x, uint64_t x_len, uint64_t n_vec, float* y, uint64_t y_len) {
  ADMIT();
  if (n_vec == 0) return fail(SPARSL_ERR_LENGTH, "n_vec", "`n_vec` must have length 1, got 0");
  if (op->ncols && n_vec > UINT64_MAX / op->ncols)
    return fail(SPARSL_ERR_LENGTH, "SpMM input element count", "SpMM input element count overflowed");
  if (op->nrows && n_vec > UINT64_MAX / op->nrows)
    return fail(SPARSL_ERR_LENGTH, "SpMM output element count", "SpMM output element count overflowed");
  const uint64_t need_x = (uint64_t)op->ncols * n_vec, need_y = (uint64_t)op->nrows * n_vec;
  TRY(check_min("x", x_len, need_x));
  TRY(check_len("y", y_len, need_y));
  if (op->nrows == 0) return SPARSL_OK;
  if (n_vec == 1) return sparsl_op_spmv(op, x, x_len, y, y_len);  // mod.rs:2370-2373
  if (n_vec > 0xffffffffull) return fail(SPARSL_ERR_LENGTH, "n_vec", "n_vec exceeds the u32 kernel range");
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spmm", cudaSetDevice(op->dev->ordinal));
  ALLOC(op->sx, need_x * 4 + 16, false, "X staging");
  ALLOC(op->sy, need_y * 4 + 16, true, "Y staging");
  SpmmLaunch p = spmm_launch(op, op->sx.as<float>(), op->sy.as<float>(), (uint32_t)n_vec);
  if (op->spmm_range_unit.empty()) {
    if (need_x) CK("spmm", cudaMemcpyAsync(op->sx.p, x, need_x * 4, cudaMemcpyHostToDevice, op->stream));
    CK("spmm", cudaMemcpyAsync(op->sy.p, y, need_y * 4, cudaMemcpyHostToDevice, op->stream));
    CK("spmm", launch_spmm(p, op->dev->sm_count, op->stream));
    CK("spmm", cudaMemcpyAsync(y, op->sy.p, need_y * 4, cudaMemcpyDeviceToHost, op->stream));
    return finish(op, "spmm");
  }
  // Pipelined by row range: X, then each range's Y rows, go up on one copy
  // stream; range k is folded once its rows are in, and its rows go down on
  // another copy stream while later ranges go up.  Each range is one launch
  // over its own units, so every output is still its own left fold.
  if (!op->up) {
    CK("spmm", cudaStreamCreateWithFlags(&op->up, cudaStreamNonBlocking));
    CK("spmm", cudaStreamCreateWithFlags(&op->down, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&op->up_ev, &op->fold_ev, &op->down_ev})
      CK("spmm", cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  }
  if (op->spmm_rorder.p) {
    p.order = op->spmm_rorder.as<uint32_t>();
    p.unit_start = op->spmm_runits.as<uint32_t>();
  }
  CK("spmm", cudaEventRecord(op->fold_ev, op->stream));  // staging is free once earlier work is done
  CK("spmm", cudaStreamWaitEvent(op->up, op->fold_ev, 0));
  if (need_x) CK("spmm", cudaMemcpyAsync(op->sx.p, x, need_x * 4, cudaMemcpyHostToDevice, op->up));
  for (size_t k = 0; k + 1 < op->spmm_range_unit.size(); ++k) {
    const uint64_t r0 = op->spmm_range_row[k], r1 = op->spmm_range_row[k + 1];
    if (r1 == r0) continue;
    const uint64_t off = r0 * n_vec, cnt = (r1 - r0) * n_vec;
    CK("spmm", cudaMemcpyAsync(op->sy.as<float>() + off, y + off, cnt * 4, cudaMemcpyHostToDevice, op->up));
    CK("spmm", cudaEventRecord(op->up_ev, op->up));
    CK("spmm", cudaStreamWaitEvent(op->stream, op->up_ev, 0));
    p.unit_base = op->spmm_range_unit[k];
    p.nunits = op->spmm_range_unit[k + 1] - op->spmm_range_unit[k];
    CK("spmm", launch_spmm(p, op->dev->sm_count, op->stream));
    CK("spmm", cudaEventRecord(op->fold_ev, op->stream));
    CK("spmm", cudaStreamWaitEvent(op->down, op->fold_ev, 0));
    CK("spmm", cudaMemcpyAsync(y + off, op->sy.as<float>() + off, cnt * 4, cudaMemcpyDeviceToHost, op->down));
  }
  CK("spmm", cudaEventRecord(op->down_ev, op->down));
  CK("spmm", cudaStreamWaitEvent(op->stream, op->down_ev, 0));
  return finish(op, "spmm");
}

static int fused_common(sparsl_op* op, const float* x, const uint32_t* bits, float* v, float* theta, uint8_t* spk,
                        float decay, float v_reset, float dtheta, const char* name) {
  std::lock_guard<std::mutex> lk(op->mu);
  CK(name, cudaSetDevice(op->dev->ordinal));
  const uint64_t nr = op->nrows;
  // v, theta and the spike bytes in pinned host memory: the tick's epilogue
  // reads and writes them in place (a tile's state is loaded when its
  // stream starts), so only the operand is copied.
  void *dv = nullptr, *dth = nullptr, *dspk = nullptr;
  const bool mapped = host_mapped(v, &dv) && host_mapped(theta, &dth) && host_mapped(spk, &dspk);
  if (!mapped) {
    ALLOC(op->sv, nr * 4 + 16, true, "v staging");
    ALLOC(op->sth, nr * 4 + 16, true, "theta staging");
    ALLOC(op->sspk, nr + 16, true, "spike staging");
  }
  RowLaunch p = fwd_launch(op);
  if (x && op->ext_x) {
    p.x = op->ext_x;  // a bound x replaces the slice (metal.rs:2686-2688)
  } else if (x) {
    ALLOC(op->sx, (uint64_t)op->ncols * 4 + 16, false, "x staging");
    if (op->ncols) CK(name, cudaMemcpyAsync(op->sx.p, x, (uint64_t)op->ncols * 4, cudaMemcpyHostToDevice, op->stream));
    p.x = op->sx.as<float>();
  } else {
    ALLOC(op->sbits, op->words() * 4 + 16, false, "spike staging");
    if (op->words()) CK(name, cudaMemcpyAsync(op->sbits.p, bits, op->words() * 4, cudaMemcpyHostToDevice, op->stream));
    set_bits_mode(p, op->sbits.as<uint32_t>(), op->words());
  }
  p.epilogue = EPI_LIF;
  p.decay = decay;
  p.v_reset = v_reset;
  p.dtheta = dtheta;
  if (mapped) {
    p.v = static_cast<float*>(dv);
    p.theta = static_cast<float*>(dth);
    p.spikes = static_cast<uint8_t*>(dspk);
    CK(name, launch_fwd(op, p, op->stream));
    return finish(op, name);
  }
  CK(name, cudaMemcpyAsync(op->sv.p, v, nr * 4, cudaMemcpyHostToDevice, op->stream));
  CK(name, cudaMemcpyAsync(op->sth.p, theta, nr * 4, cudaMemcpyHostToDevice, op->stream));
  p.v = op->sv.as<float>();
  p.theta = op->sth.as<float>();
  p.spikes = op->sspk.as<uint8_t>();
  CK(name, launch_fwd(op, p, op->stream));
  CK(name, cudaMemcpyAsync(v, op->sv.p, nr * 4, cudaMemcpyDeviceToHost, op->stream));
  CK(name, cudaMemcpyAsync(theta, op->sth.p, nr * 4, cudaMemcpyDeviceToHost, op->stream));
  CK(name, cudaMemcpyAsync(spk, op->sspk.p, nr, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, name);
}

int sparsl_op_fused_lif(sparsl_op* op, const float* x, uint64_t x_len, float* v, float* theta, uint8_t* spikes,
                        uint64_t n, float decay, float v_reset, float dtheta) {
  ADMIT();
  TRY(check_min("x", x_len, op->ncols));
  TRY(check_len("v", n, op->nrows));
  if (op->nrows == 0) return SPARSL_OK;
  return fused_common(op, x, nullptr, v, theta, spikes, decay, v_reset, dtheta, "fused_spmv_lif");
}

int sparsl_op_fused_spikes_lif(sparsl_op* op, const uint32_t* s_in, uint64_t words, float* v, float* theta,
                               uint8_t* s_out, uint64_t n, float decay, float v_reset, float dtheta) {
  ADMIT();
  TRY(check_min("spikes_in", words, op->words()));
  TRY(check_len("v", n, op->nrows));
  if (op->nrows == 0) return SPARSL_OK;
  return fused_common(op, nullptr, s_in, v, theta, s_out, decay, v_reset, dtheta, "fused_spmv_spikes_lif");
}

// ---- resident ------------------------------------------------------------
int sparsl_op_write_x(sparsl_op* op, const float* x, uint64_t len) {
  ADMIT();
  TRY(check_min("x", len, op->ncols));
  std::lock_guard<std::mutex> lk(op->mu);
  if (op->ext_x)
    return fail(SPARSL_ERR_BACKEND, "write_x refused while an external buffer is bound as x; unbind first",
                "write_x refused while an external buffer is bound as x; unbind first");
  CK("write_x", cudaSetDevice(op->dev->ordinal));
  if (op->ncols) CK("write_x", cudaMemcpyAsync(op->rx.p, x, (uint64_t)op->ncols * 4, cudaMemcpyHostToDevice, op->stream));
  return wait_op(op, "write_x");
}

int sparsl_op_write_x_spikes(sparsl_op* op, const uint32_t* s, uint64_t words) {
  ADMIT();
  TRY(check_min("spikes", words, op->words()));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("write_x_spikes", cudaSetDevice(op->dev->ordinal));
  if (op->words())
    CK("write_x_spikes", cudaMemcpyAsync(op->rxs[op->cur].p, s, op->words() * 4, cudaMemcpyHostToDevice, op->stream));
  return wait_op(op, "write_x_spikes");
}

int sparsl_op_write_y(sparsl_op* op, const float* y, uint64_t len) {
  ADMIT();
  TRY(check_len("y", len, op->nrows));
  std::lock_guard<std::mutex> lk(op->mu);
  if (op->ext_y)
    return fail(SPARSL_ERR_BACKEND, "write_y refused while an external buffer is bound as y; unbind first",
                "write_y refused while an external buffer is bound as y; unbind first");
  CK("write_y", cudaSetDevice(op->dev->ordinal));
  if (op->nrows) CK("write_y", cudaMemcpyAsync(op->ry.p, y, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, op->stream));
  return wait_op(op, "write_y");
}

int sparsl_op_write_lif_state(sparsl_op* op, const float* v, const float* theta, uint64_t n) {
  ADMIT();
  TRY(check_len("v", n, op->nrows));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("write_lif_state", cudaSetDevice(op->dev->ordinal));
  if (n) {
    CK("write_lif_state", cudaMemcpyAsync(op->rv.p, v, n * 4, cudaMemcpyHostToDevice, op->stream));
    CK("write_lif_state", cudaMemcpyAsync(op->rth.p, theta, n * 4, cudaMemcpyHostToDevice, op->stream));
  }
  return wait_op(op, "write_lif_state");
}

int sparsl_op_spmv_resident(sparsl_op* op) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spmv_resident", cudaSetDevice(op->dev->ordinal));
  RowLaunch p = fwd_launch(op);
  p.x = op->x_active();
  p.y = op->y_active();
  CK("spmv_resident", launch_fwd(op, p, op->stream));
  return wait_op(op, "spmv_resident");
}

static void lif_resident_launch(sparsl_op* op, RowLaunch& p, float decay, float v_reset, float dtheta) {
  p.epilogue = EPI_LIF;
  p.v = op->rv.as<float>();
  p.theta = op->rth.as<float>();
  p.spikes = op->rspk.as<uint8_t>();
  p.decay = decay;
  p.v_reset = v_reset;
  p.dtheta = dtheta;
}

int sparsl_op_fused_lif_resident(sparsl_op* op, float decay, float v_reset, float dtheta) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("fused_spmv_lif_resident", cudaSetDevice(op->dev->ordinal));
  RowLaunch p = fwd_launch(op);
  p.x = op->x_active();
  lif_resident_launch(op, p, decay, v_reset, dtheta);
  CK("fused_spmv_lif_resident", launch_fwd(op, p, op->stream));
  return wait_op(op, "fused_spmv_lif_resident");
}

int sparsl_op_fused_spikes_lif_resident(sparsl_op* op, float decay, float v_reset, float dtheta) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("fused_spmv_spikes_lif_resident", cudaSetDevice(op->dev->ordinal));
  RowLaunch p = fwd_launch(op);
  set_bits_mode(p, op->rxs[op->cur].as<uint32_t>(), op->words());
  lif_resident_launch(op, p, decay, v_reset, dtheta);
  CK("fused_spmv_spikes_lif_resident", launch_fwd(op, p, op->stream));
  return wait_op(op, "fused_spmv_spikes_lif_resident");
}

int sparsl_op_pack_resident_spikes(sparsl_op* op) {
  ADMIT();
  TRY(check_len("recurrent nrows", op->nrows, op->ncols));
  if (op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("pack_resident_spikes_to_x_spikes", cudaSetDevice(op->dev->ordinal));
  CK("pack_resident_spikes_to_x_spikes",
     launch_pack(op->rspk.as<uint8_t>(), op->nrows, op->rxs[op->cur].as<uint32_t>(), op->words(), op->stream));
  return wait_op(op, "pack_resident_spikes_to_x_spikes");
}

// Uniform rows: each tick is the streaming kernel on the operator's stream,
// then the compaction of its packed spikes on the side stream, overlapping
// the next tick.  Tick t + 1 overwrites the buffer tick t - 1 wrote, so it
// first waits for the compaction that read it.
static int enqueue_recurrent_ell(sparsl_op* op, float decay, float v_reset, float dtheta, uint64_t steps) {
  const char* name = "fused_spmv_spikes_lif_recurrent_steps";
  if (!op->side) {
    CK(name, cudaStreamCreateWithFlags(&op->side, cudaStreamNonBlocking));
    CK(name, cudaEventCreateWithFlags(&op->tick_ev, cudaEventDisableTiming));
    CK(name, cudaEventCreateWithFlags(&op->done_ev[0], cudaEventDisableTiming));
    CK(name, cudaEventCreateWithFlags(&op->done_ev[1], cudaEventDisableTiming));
    CK(name, cudaEventRecord(op->done_ev[0], op->side));
    CK(name, cudaEventRecord(op->done_ev[1], op->side));
  }
  for (uint64_t t = 0; t < steps; ++t) {
    const int out = op->cur ^ 1;
    RowLaunch p = fwd_launch(op);
    set_bits_mode(p, op->rxs[op->cur].as<uint32_t>(), op->words());
    lif_resident_launch(op, p, decay, v_reset, dtheta);
    p.out_bits = op->rxs[out].as<uint32_t>();
    p.tile_flags = op->tile_flags.as<unsigned long long>();
    p.tile_ticket = op->ticket.as<uint32_t>();
    CK(name, cudaStreamWaitEvent(op->stream, op->done_ev[out], 0));
    CK(name, launch_ell(op->ell, p, op->stream));
    CK(name, cudaEventRecord(op->tick_ev, op->stream));
    CK(name, cudaStreamWaitEvent(op->side, op->tick_ev, 0));
    CK(name, launch_compact_bits(p.out_bits, op->words(), op->idx_list.as<uint32_t>(), op->trace.as<uint32_t>() + t,
                                 0, op->side));
    CK(name, cudaEventRecord(op->done_ev[out], op->side));
    op->cur = out;
  }
  // Everything after this call (waits, reads of the list and the trace)
  // follows the last compaction.
  CK(name, cudaStreamWaitEvent(op->stream, op->done_ev[op->cur], 0));
  op->last_steps = steps;
  return SPARSL_OK;
}

static int enqueue_recurrent(sparsl_op* op, float decay, float v_reset, float dtheta, uint64_t steps) {
  TRY(ensure_trace(op, steps));
  if (op->ell.ok) return enqueue_recurrent_ell(op, decay, v_reset, dtheta, steps);
  for (uint64_t t = 0; t < steps; ++t) {
    RowLaunch p = fwd_launch(op);
    set_bits_mode(p, op->rxs[op->cur].as<uint32_t>(), op->words());
    lif_resident_launch(op, p, decay, v_reset, dtheta);
    p.out_bits = op->rxs[op->cur ^ 1].as<uint32_t>();
    p.idx_list = op->idx_list.as<uint32_t>();
    p.idx_count = op->trace.as<uint32_t>() + t;
    p.tile_flags = op->tile_flags.as<unsigned long long>();
    p.tile_ticket = op->ticket.as<uint32_t>();
    CK("fused_spmv_spikes_lif_recurrent_steps", launch_fwd(op, p, op->stream));
    op->cur ^= 1;
  }
  op->last_steps = steps;
  return SPARSL_OK;
}

int sparsl_op_recurrent_steps(sparsl_op* op, float decay, float v_reset, float dtheta, uint64_t steps) {
  ADMIT();
  TRY(check_len("recurrent nrows", op->nrows, op->ncols));
  if (steps == 0 || op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("fused_spmv_spikes_lif_recurrent_steps", cudaSetDevice(op->dev->ordinal));
  TRY(enqueue_recurrent(op, decay, v_reset, dtheta, steps));
  return wait_op(op, "fused_spmv_spikes_lif_recurrent_steps");
}

int sparsl_op_recurrent_steps_async(sparsl_op* op, float decay, float v_reset, float dtheta, uint64_t steps) {
  ADMIT();
  TRY(check_len("recurrent nrows", op->nrows, op->ncols));
  if (steps == 0 || op->nrows == 0) return SPARSL_OK;
  std::lock_guard<std::mutex> lk(op->mu);
  CK("fused_spmv_spikes_lif_recurrent_steps", cudaSetDevice(op->dev->ordinal));
  return enqueue_recurrent(op, decay, v_reset, dtheta, steps);
}

int sparsl_op_sync_y(sparsl_op* op, float* y, uint64_t len) {
  ADMIT();
  TRY(check_len("y", len, op->nrows));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("sync_y", cudaSetDevice(op->dev->ordinal));
  if (op->nrows)
    CK("sync_y", cudaMemcpyAsync(y, op->y_active(), (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "sync_y");
}

int sparsl_op_sync_lif_state(sparsl_op* op, float* v, float* theta, uint8_t* spikes, uint64_t n) {
  ADMIT();
  TRY(check_len("v", n, op->nrows));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("sync_lif_state", cudaSetDevice(op->dev->ordinal));
  if (n) {
    CK("sync_lif_state", cudaMemcpyAsync(v, op->rv.p, n * 4, cudaMemcpyDeviceToHost, op->stream));
    CK("sync_lif_state", cudaMemcpyAsync(theta, op->rth.p, n * 4, cudaMemcpyDeviceToHost, op->stream));
    CK("sync_lif_state", cudaMemcpyAsync(spikes, op->rspk.p, n, cudaMemcpyDeviceToHost, op->stream));
  }
  return finish(op, "sync_lif_state");
}

// ---- zero-copy interop (mod.rs:1975-2098, metal.rs:1805-1955) -------------
namespace {

// validate_external_vec (metal.rs:1805-1832): the buffer must be device
// memory of the operator's GPU and hold `elems` f32 from `p` to the end of
// its allocation.
int check_external(sparsl_op* op, const void* p, uint64_t elems, const char* what) {
  cudaPointerAttributes at{};
  const bool ok = p && cudaPointerGetAttributes(&at, p) == cudaSuccess &&
                  ((at.type == cudaMemoryTypeDevice && at.device == op->dev->ordinal) ||
                   at.type == cudaMemoryTypeManaged);
  if (!ok) {
    cudaGetLastError();
    return fail(SPARSL_ERR_BACKEND, "external buffer is not device memory of this operator's GPU",
                std::string(what) + ": not device memory of GPU " + std::to_string(op->dev->ordinal));
  }
  AddrRangeFn fn = addr_range_fn();
  unsigned long long base = 0;
  size_t size = 0;
  const unsigned long long a = reinterpret_cast<unsigned long long>(p);
  if (!fn || fn(&base, &size, a) != 0)
    return fail(SPARSL_ERR_BACKEND, "external buffer is not device memory of this operator's GPU",
                std::string(what) + ": no allocation holds it");
  const uint64_t need = elems * 4, got = base + size - a;
  if (got < need)
    return fail(SPARSL_ERR_LENGTH, "external buffer too short",
                std::string(what) + ": needs " + std::to_string(need) + " bytes, its allocation holds " +
                    std::to_string(got) + " from this address");
  return SPARSL_OK;
}

}  // namespace

int sparsl_op_bind_x(sparsl_op* op, const float* d_x) {
  ADMIT();
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "bind_x: null operator");
  CK("bind_x", cudaSetDevice(op->dev->ordinal));
  TRY(check_external(op, d_x, op->ncols, "external x"));
  std::lock_guard<std::mutex> lk(op->mu);
  op->ext_x = d_x;
  return SPARSL_OK;
}

int sparsl_op_bind_y(sparsl_op* op, float* d_y) {
  ADMIT();
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "bind_y: null operator");
  CK("bind_y", cudaSetDevice(op->dev->ordinal));
  TRY(check_external(op, d_y, op->nrows, "external y"));
  std::lock_guard<std::mutex> lk(op->mu);
  op->ext_y = d_y;
  return SPARSL_OK;
}

int sparsl_op_unbind_x(sparsl_op* op) {
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "unbind_x: null operator");
  std::lock_guard<std::mutex> lk(op->mu);
  op->ext_x = nullptr;
  return SPARSL_OK;
}

int sparsl_op_unbind_y(sparsl_op* op) {
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "unbind_y: null operator");
  std::lock_guard<std::mutex> lk(op->mu);
  op->ext_y = nullptr;
  return SPARSL_OK;
}

int sparsl_op_x_address(sparsl_op* op, uint64_t* out) {
  if (!op || !out) return fail(SPARSL_ERR_INVALID, "null argument", "x_address: null argument");
  std::lock_guard<std::mutex> lk(op->mu);
  *out = reinterpret_cast<uint64_t>(op->x_active());
  return SPARSL_OK;
}

int sparsl_op_y_address(sparsl_op* op, uint64_t* out) {
  if (!op || !out) return fail(SPARSL_ERR_INVALID, "null argument", "y_address: null argument");
  std::lock_guard<std::mutex> lk(op->mu);
  *out = reinterpret_cast<uint64_t>(op->y_active());
  return SPARSL_OK;
}

int sparsl_op_alloc_f32(sparsl_op* op, const float* data, uint64_t n, float** out) {
  ADMIT();
  if (!op || !out) return fail(SPARSL_ERR_INVALID, "null argument", "alloc_f32: null argument");
  *out = nullptr;
  CK("alloc_f32", cudaSetDevice(op->dev->ordinal));
  void* p = sparsl_device_alloc(op->dev, n * 4);
  if (!p)
    return fail(SPARSL_ERR_BACKEND, "could not allocate an external buffer on the operator's GPU",
                "alloc_f32: device allocation failed");
  if (n && data && cudaMemcpy(p, data, n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    sparsl_device_free(p);
    return fail_cuda("alloc_f32", cudaGetLastError());
  }
  *out = static_cast<float*>(p);
  return SPARSL_OK;
}

int sparsl_op_wait_event(sparsl_op* op, void* event, uint64_t timeout_ms) {
  ADMIT();
  if (!op) return fail(SPARSL_ERR_INVALID, "null argument", "wait_event: null operator");
  if (!event) return SPARSL_OK;  // like a shared-event value of 0: nothing to wait for
  CK("wait_event", cudaSetDevice(op->dev->ordinal));
  cudaEvent_t ev = static_cast<cudaEvent_t>(event);
  // Device order first: the operator's later work follows the peer's even if
  // the host stops waiting.
  CK("wait_event", cudaStreamWaitEvent(op->stream, ev, 0));
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return SPARSL_OK;
    if (q != cudaErrorNotReady) return fail_cuda("wait_event", q);
    if (std::chrono::steady_clock::now() >= deadline)
      return fail(SPARSL_ERR_EXECUTION, "wait_event timed out",
                  "wait_event: the peer event did not complete within " + std::to_string(timeout_ms) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int sparsl_op_signal_event(sparsl_op* op, void* event) {
  ADMIT();
  if (!op || !event) return fail(SPARSL_ERR_INVALID, "null argument", "signal_event: null argument");
  CK("signal_event", cudaSetDevice(op->dev->ordinal));
  // Completes once every call enqueued on the operator before it has finished.
  CK("signal_event", cudaEventRecord(static_cast<cudaEvent_t>(event), op->stream));
  return SPARSL_OK;
}

int sparsl_op_sync_x_spikes(sparsl_op* op, uint32_t* s, uint64_t words) {
  ADMIT();
  TRY(check_min("spikes", words, op->words()));
  std::lock_guard<std::mutex> lk(op->mu);
  CK("sync_x_spikes", cudaSetDevice(op->dev->ordinal));
  if (op->words())
    CK("sync_x_spikes", cudaMemcpyAsync(s, op->rxs[op->cur].p, op->words() * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "sync_x_spikes");
}

int sparsl_op_spike_trace(sparsl_op* op, uint32_t* out, uint64_t cap, uint64_t* n_out) {
  ADMIT();
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spike_trace", cudaSetDevice(op->dev->ordinal));
  const uint64_t n = std::min<uint64_t>(cap, op->last_steps);
  if (n_out) *n_out = op->last_steps;
  if (n) CK("spike_trace", cudaMemcpyAsync(out, op->trace.p, n * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "spike_trace");
}

int sparsl_op_spike_indices(sparsl_op* op, uint32_t* out, uint64_t cap, uint64_t* count) {
  ADMIT();
  std::lock_guard<std::mutex> lk(op->mu);
  CK("spike_indices", cudaSetDevice(op->dev->ordinal));
  if (op->last_steps == 0) {
    if (count) *count = 0;
    return SPARSL_OK;
  }
  uint32_t c = 0;
  CK("spike_indices", cudaMemcpyAsync(&c, op->trace.as<uint32_t>() + (op->last_steps - 1), 4, cudaMemcpyDeviceToHost,
                                      op->stream));
  CK("spike_indices", cudaStreamSynchronize(op->stream));
  if (count) *count = c;
  const uint64_t n = std::min<uint64_t>(cap, c);
  if (n) CK("spike_indices", cudaMemcpyAsync(out, op->idx_list.p, n * 4, cudaMemcpyDeviceToHost, op->stream));
  return finish(op, "spike_indices");
}

// ---- device-pointer entry points ------------------------------------------
static cudaStream_t pick(sparsl_op* op, void* stream) {
  return stream ? static_cast<cudaStream_t>(stream) : op->stream;
}

int sparsl_op_spmv_device(sparsl_op* op, const float* d_x, float* d_y, void* stream) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  CK("spmv", cudaSetDevice(op->dev->ordinal));
  RowLaunch p = fwd_launch(op);
  p.x = d_x;
  p.y = d_y;
  CK("spmv", launch_fwd(op, p, pick(op, stream)));
  return SPARSL_OK;
}

int sparsl_op_spmv_spikes_device(sparsl_op* op, const uint32_t* d_spikes, float* d_y, void* stream) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  CK("spmv_spikes", cudaSetDevice(op->dev->ordinal));
  RowLaunch p = fwd_launch(op);
  set_bits_mode(p, d_spikes, op->words());
  p.y = d_y;
  CK("spmv_spikes", launch_fwd(op, p, pick(op, stream)));
  return SPARSL_OK;
}

int sparsl_op_spmv_t_device(sparsl_op* op, const float* d_x, float* d_y, void* stream) {
  ADMIT();
  if (op->ncols == 0) return SPARSL_OK;
  if (!op->has_t) return fail(SPARSL_ERR_NO_TRANSPOSE, "transpose not prepared", "no reverse index");
  CK("spmv_t", cudaSetDevice(op->dev->ordinal));
  CK("spmv_t", launch_transpose(op, d_x, d_y, pick(op, stream)));
  return SPARSL_OK;
}

int sparsl_op_spmm_device(sparsl_op* op, const float* d_x, uint64_t n_vec, float* d_y, void* stream) {
  ADMIT();
  if (op->nrows == 0) return SPARSL_OK;
  if (n_vec == 0 || n_vec > 0xffffffffull) return fail(SPARSL_ERR_LENGTH, "n_vec", "n_vec out of range");
  CK("spmm", cudaSetDevice(op->dev->ordinal));
  if (n_vec == 1) return sparsl_op_spmv_device(op, d_x, d_y, stream);
  CK("spmm", launch_spmm(spmm_launch(op, d_x, d_y, (uint32_t)n_vec), op->dev->sm_count, pick(op, stream)));
  return SPARSL_OK;
}

void* sparsl_op_stream(sparsl_op* op) { return op ? op->stream : nullptr; }
int sparsl_op_wait(sparsl_op* op) {
  if (!op) return fail(SPARSL_ERR_INVALID, "null operator", "null operator");
  cudaSetDevice(op->dev->ordinal);
  return wait_op(op, "wait");
}

// ---- memory helpers --------------------------------------------------------
void* sparsl_host_alloc(uint64_t bytes) {
  void* p = nullptr;
  if (cudaHostAlloc(&p, std::max<uint64_t>(bytes, 16), cudaHostAllocDefault) != cudaSuccess) return nullptr;
  return p;
}
void sparsl_host_free(void* p) {
  if (p) cudaFreeHost(p);
}
void* sparsl_device_alloc(sparsl_dev* d, uint64_t bytes) {
  if (!d) return nullptr;
  cudaSetDevice(d->ordinal);
  void* p = nullptr;
  if (cudaMalloc(&p, round_up(std::max<uint64_t>(bytes, 16), kAlign) + kAlign) != cudaSuccess) return nullptr;
  return p;
}
void sparsl_device_free(void* p) {
  if (p) cudaFree(p);
}
int sparsl_memcpy(void* dst, const void* src, uint64_t bytes) {
  CK("memcpy", cudaMemcpy(dst, src, bytes, cudaMemcpyDefault));
  return SPARSL_OK;
}

// ==========================================================================
// Multi-GPU network tick
// ==========================================================================
}  // extern "C"

struct sparsl_net {
  sparsl_dev* dev = nullptr;
  std::vector<sparsl_op*> blocks;
  std::vector<uint64_t> block_off;  // local row offset of each block
  uint64_t row_offset = 0, n_global = 0, local_rows = 0, words = 0;
  int rank = 0, nranks = 1;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev = nullptr;
  // Blocks alternate between `stream` and `side` within a tick, so one
  // block's persistent kernel starts on the SMs the other's tail frees.
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  ErrWord err;
  DBuf xs[2], trace;
  int cur = 0;
  uint64_t trace_cap = 0, last_steps = 0;
  ncclComm_t comm = nullptr;
  // Optional per-tick timing of the fused tick kernels (events bracket the
  // block kernels of each tick, excluding the exchange).
  bool timing = false;
  std::vector<cudaEvent_t> ev_a, ev_b;
  uint64_t timed_ticks = 0;
  // Exchange of the spike vector between ranks: SPARSL_NET_EXCHANGE_PEER
  // (peer stores over NVLink and one small flag kernel per tick) or
  // SPARSL_NET_EXCHANGE_NCCL (an in-place ncclAllGather, then a count).
  int exchange = SPARSL_NET_EXCHANGE_PEER;
  DBuf box;         // this rank's NetMailbox, written by the peers
  DBuf tick_count;  // this rank's spike count of the current tick
  // Peers' memory mapped into this process (cudaIpcOpenMemHandle), to close.
  std::vector<void*> opened;
  // Device pointer tables: [parity][block][rank] peer words at each block's
  // offset, [parity][rank] peer words at this rank's slice, [rank] mailboxes.
  DBuf peer_out, peer_slice, peer_box;
  uint32_t tick = 0;  // ticks run so far (the same on every rank)
  // sparsl_net_steps_host: copy streams and per-block events, made at its
  // first call.  Block b's state arrives on copy_in (ev_in[b]); its first
  // tick waits for that alone, and its copy back starts on copy_out when its
  // last tick kernel ends (ev_out[b]), under the other blocks' kernels.
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  std::vector<cudaEvent_t> ev_in, ev_out;
  cudaEvent_t ev_copied = nullptr;
};

namespace {
// Maps every peer's spike vectors and mailbox into this process: each rank
// exports cudaIpc handles of its two spike-vector copies and its mailbox,
// one ncclAllGather hands them to every rank, and each rank opens the
// others'.  All of it happens once, at create; the tick path uses only the
// resulting device pointers.
int net_map_peers(sparsl_net* net) {
  const uint32_t R = (uint32_t)net->nranks, me = (uint32_t)net->rank;
  if (R > kNetMaxRanks) return fail(SPARSL_ERR_INVALID, "nranks", "at most 32 ranks per network");
  cudaStream_t s = net->stream;
  if (dalloc(net->box, sizeof(NetMailbox), false, s) != cudaSuccess ||
      dalloc(net->tick_count, 16, false, s) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "exchange area", "device allocation failed for the exchange area");
  CK("net_create", cudaMemsetAsync(net->box.p, 0, sizeof(NetMailbox), s));
  CK("net_create", cudaMemsetAsync(net->tick_count.p, 0, 16, s));
  constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
  std::vector<unsigned char> mine(3 * kH), all(3 * kH * R);
  void* bases[3] = {net->xs[0].p, net->xs[1].p, net->box.p};
  for (int i = 0; i < 3; ++i) {
    cudaIpcMemHandle_t h;
    CK("net_create", cudaIpcGetMemHandle(&h, bases[i]));
    std::memcpy(mine.data() + i * kH, &h, kH);
  }
  DBuf xfer;
  if (dalloc(xfer, all.size(), false, s) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "exchange setup", "device allocation failed for the handle exchange");
  unsigned char* d = xfer.as<unsigned char>();
  int rc = SPARSL_OK;
  do {
    if (cudaMemcpyAsync(d + me * mine.size(), mine.data(), mine.size(), cudaMemcpyHostToDevice, s) != cudaSuccess) {
      rc = fail_cuda("net_create", cudaGetLastError());
      break;
    }
    ncclResult_t r = nccl_settle(net->comm, g_nccl.AllGather(d + me * mine.size(), d, mine.size(), ncclUint8,
                                                            net->comm, s));
    if (r != ncclSuccess) {
      rc = fail(SPARSL_ERR_EXECUTION, "ncclAllGather failed", "handle exchange: ncclAllGather failed");
      break;
    }
    if (cudaMemcpyAsync(all.data(), d, all.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
      rc = fail_cuda("net_create", cudaGetLastError());
      break;
    }
    rc = wait_bounded(s, net->ev, net->err.d, net->err.h, "net_create");
  } while (false);
  dfree(xfer);
  if (rc != SPARSL_OK) return rc;
  std::vector<uint32_t*> px[2] = {std::vector<uint32_t*>(R, nullptr), std::vector<uint32_t*>(R, nullptr)};
  std::vector<NetMailbox*> pbox(R, nullptr);
  for (uint32_t r = 0; r < R; ++r) {
    if (r == me) continue;
    void* ptrs[3] = {};
    for (int i = 0; i < 3; ++i) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, all.data() + (r * 3 + i) * kH, kH);
      const cudaError_t e = cudaIpcOpenMemHandle(&ptrs[i], h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess)
        return fail(SPARSL_ERR_BACKEND, "peer memory unavailable",
                    std::string("net_create: cannot map rank ") + std::to_string(r) +
                        "'s memory (cudaIpcOpenMemHandle: " + cudaGetErrorString(e) + ")");
      net->opened.push_back(ptrs[i]);
    }
    px[0][r] = static_cast<uint32_t*>(ptrs[0]);
    px[1][r] = static_cast<uint32_t*>(ptrs[1]);
    pbox[r] = static_cast<NetMailbox*>(ptrs[2]);
  }
  const size_t nb = net->blocks.size();
  std::vector<uint32_t*> out(2 * nb * R, nullptr), slice(2 * R, nullptr);
  for (int q = 0; q < 2; ++q)
    for (uint32_t r = 0; r < R; ++r) {
      if (!px[q][r]) continue;
      slice[q * R + r] = px[q][r] + net->row_offset / 32;
      for (size_t b = 0; b < nb; ++b) out[(q * nb + b) * R + r] = px[q][r] + (net->row_offset + net->block_off[b]) / 32;
    }
  if (dalloc(net->peer_out, out.size() * sizeof(void*), false, s) != cudaSuccess ||
      dalloc(net->peer_slice, slice.size() * sizeof(void*), false, s) != cudaSuccess ||
      dalloc(net->peer_box, R * sizeof(void*), false, s) != cudaSuccess)
    return fail(SPARSL_ERR_ALLOCATION, "exchange tables", "device allocation failed for the peer tables");
  CK("net_create", cudaMemcpyAsync(net->peer_out.p, out.data(), out.size() * sizeof(void*), cudaMemcpyHostToDevice, s));
  CK("net_create", cudaMemcpyAsync(net->peer_slice.p, slice.data(), slice.size() * sizeof(void*), cudaMemcpyHostToDevice, s));
  CK("net_create", cudaMemcpyAsync(net->peer_box.p, pbox.data(), R * sizeof(void*), cudaMemcpyHostToDevice, s));
  return wait_bounded(s, net->ev, net->err.d, net->err.h, "net_create");
}
}  // namespace

extern "C" {

int sparsl_nccl_unique_id(uint8_t out[128]) {
  if (const char* why = nccl_load()) return fail(SPARSL_ERR_BACKEND, why, why);
  ncclUniqueId id;
  ncclResult_t r = g_nccl.GetUniqueId(&id);
  if (r != ncclSuccess) return fail(SPARSL_ERR_BACKEND, "ncclGetUniqueId failed", g_nccl.GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out, &id, 128);
  return SPARSL_OK;
}

int sparsl_net_create(sparsl_dev* d, sparsl_op* const* blocks, uint32_t n_blocks, uint64_t row_offset,
                      uint64_t n_global, int rank, int nranks, const uint8_t* nccl_id, sparsl_net** out) {
  ADMIT();
  if (!d || !out || (n_blocks && !blocks)) return fail(SPARSL_ERR_INVALID, "null argument", "sparsl_net_create");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(SPARSL_ERR_INVALID, "rank", "rank out of range");
  if (row_offset % 32) return fail(SPARSL_ERR_INVALID, "row_offset", "row_offset must be a multiple of 32");
  if (n_global % 32 || (n_global / 32) % nranks)
    return fail(SPARSL_ERR_INVALID, "n_global", "n_global must split into equal 32-aligned rank slices");
  uint64_t local = 0;
  std::vector<uint64_t> offs;
  for (uint32_t b = 0; b < n_blocks; ++b) {
    sparsl_op* op = blocks[b];
    if (op->dev != d) return fail(SPARSL_ERR_INVALID, "block device", "all blocks must live on the net's device");
    if (op->ncols != n_global) return fail(SPARSL_ERR_INVALID, "block ncols", "every block must have ncols == n_global");
    if (local % 32) return fail(SPARSL_ERR_INVALID, "block rows", "every block but the last must hold a multiple of 32 rows");
    offs.push_back(local);
    local += op->nrows;
  }
  if (nranks > 1 && local != n_global / nranks)
    return fail(SPARSL_ERR_INVALID, "local rows", "each rank must hold n_global / nranks rows");
  if (row_offset + local > n_global) return fail(SPARSL_ERR_INVALID, "local rows", "rows exceed n_global");
  CK("net_create", cudaSetDevice(d->ordinal));
  auto* net = new sparsl_net();
  net->dev = d;
  net->blocks.assign(blocks, blocks + n_blocks);
  net->block_off = offs;
  net->row_offset = row_offset;
  net->n_global = n_global;
  net->local_rows = local;
  net->words = n_global / 32;
  net->rank = rank;
  net->nranks = nranks;
  auto bail = [&](int code) {
    sparsl_net_destroy(net);
    return code;
  };
  if (cudaStreamCreateWithFlags(&net->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&net->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&net->ev, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&net->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&net->ev_join, cudaEventDisableTiming) != cudaSuccess || net->err.init() != cudaSuccess)
    return bail(fail(SPARSL_ERR_BACKEND, "stream creation failed", "could not create net stream"));
  for (int i = 0; i < 2; ++i) {
    if (dalloc(net->xs[i], net->words * 4 + 16, true, net->stream) != cudaSuccess)
      return bail(fail(SPARSL_ERR_ALLOCATION, "x_spikes", "device allocation failed for x_spikes"));
    cudaMemsetAsync(net->xs[i].p, 0, net->xs[i].bytes, net->stream);
  }
  if (nranks > 1) {
    if (!nccl_id) return bail(fail(SPARSL_ERR_INVALID, "nccl id", "nccl_id is required when nranks > 1"));
    if (const char* why = nccl_load()) return bail(fail(SPARSL_ERR_BACKEND, why, why));
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = g_nccl.CommInitRankConfig(&net->comm, nranks, id, rank, &cfg);
    if (r == ncclSuccess || r == ncclInProgress) {
      if (r == ncclSuccess) g_nccl.CommGetAsyncError(net->comm, &r);
      r = nccl_settle(net->comm, r);
      if (r == ncclInProgress) {
        g_nccl.CommAbort(net->comm);
        net->comm = nullptr;
        return bail(fail(SPARSL_ERR_EXECUTION, "NCCL init timed out", "ncclCommInitRank did not complete in time"));
      }
    }
    if (r != ncclSuccess) {
      if (net->comm) g_nccl.CommAbort(net->comm);
      net->comm = nullptr;
      return bail(fail(SPARSL_ERR_BACKEND, "NCCL init failed", g_nccl.GetErrorString(r)));
    }
  }
  int rc = wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_create");
  if (rc != SPARSL_OK) return bail(rc);
  if (nranks > 1) {
    rc = net_map_peers(net);
    if (rc != SPARSL_OK) return bail(rc);
  }
  *out = net;
  return SPARSL_OK;
}

void sparsl_net_destroy(sparsl_net* net) {
  if (!net) return;
  cudaSetDevice(net->dev->ordinal);
  if (net->stream) cudaStreamSynchronize(net->stream);
  if (net->comm) {
    // Finalize flushes the communicator's outstanding work (polled, bounded);
    // a quarantined process or a finalize that does not settle aborts instead.
    if (!g_quarantine.load() && nccl_settle(net->comm, g_nccl.CommFinalize(net->comm)) == ncclSuccess)
      g_nccl.CommDestroy(net->comm);
    else
      g_nccl.CommAbort(net->comm);
  }
  for (cudaEvent_t e : net->ev_a) cudaEventDestroy(e);
  for (cudaEvent_t e : net->ev_b) cudaEventDestroy(e);
  for (void* p : net->opened) cudaIpcCloseMemHandle(p);
  for (DBuf* b : {&net->box, &net->tick_count, &net->peer_out, &net->peer_slice, &net->peer_box}) dfree(*b);
  dfree(net->xs[0]);
  dfree(net->xs[1]);
  dfree(net->trace);
  net->err.release();
  if (net->side) cudaStreamSynchronize(net->side);
  for (cudaStream_t c : {net->copy_in, net->copy_out})
    if (c) {
      cudaStreamSynchronize(c);
      cudaStreamDestroy(c);
    }
  for (cudaEvent_t e : net->ev_in) cudaEventDestroy(e);
  for (cudaEvent_t e : net->ev_out) cudaEventDestroy(e);
  if (net->ev_copied) cudaEventDestroy(net->ev_copied);
  if (net->ev) cudaEventDestroy(net->ev);
  if (net->ev_fork) cudaEventDestroy(net->ev_fork);
  if (net->ev_join) cudaEventDestroy(net->ev_join);
  if (net->side) cudaStreamDestroy(net->side);
  if (net->stream) cudaStreamDestroy(net->stream);
  delete net;
}

void* sparsl_net_stream(sparsl_net* net) { return net ? net->stream : nullptr; }

int sparsl_net_write_state(sparsl_net* net, const uint32_t* xs, uint64_t words, const float* v, const float* theta,
                           uint64_t local_rows) {
  ADMIT();
  TRY(check_min("x_spikes", words, net->words));
  TRY(check_len("v", local_rows, net->local_rows));
  CK("net_write_state", cudaSetDevice(net->dev->ordinal));
  CK("net_write_state", cudaMemcpyAsync(net->xs[net->cur].p, xs, net->words * 4, cudaMemcpyHostToDevice, net->stream));
  for (size_t b = 0; b < net->blocks.size(); ++b) {
    sparsl_op* op = net->blocks[b];
    const uint64_t o = net->block_off[b];
    if (!op->nrows) continue;
    CK("net_write_state", cudaMemcpyAsync(op->rv.p, v + o, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, net->stream));
    CK("net_write_state", cudaMemcpyAsync(op->rth.p, theta + o, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, net->stream));
  }
  return wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_write_state");
}

// in_ev / out_ev (one per block, or null): block b's first tick kernel
// waits for in_ev[b], and out_ev[b] is recorded when its last one ends.
// hv / hth (device-usable pointers to pinned host arrays of local_rows
// floats, or null): the first tick reads v / theta from them and the last
// tick writes the new state to them as well as to the device.
static int net_enqueue(sparsl_net* net, float decay, float v_reset, float dtheta, uint64_t steps,
                       const cudaEvent_t* in_ev = nullptr, const cudaEvent_t* out_ev = nullptr, float* hv = nullptr,
                       float* hth = nullptr) {
  if (!net->trace.p || net->trace_cap < steps) {
    const uint64_t cap = std::max<uint64_t>(steps, 1024);
    if (ensure(net->trace, cap * 4, true, net->stream) != cudaSuccess)
      return fail(SPARSL_ERR_ALLOCATION, "trace", "device allocation failed for the spike trace");
    net->trace_cap = cap;
  }
  const uint64_t slice = net->words / net->nranks;
  for (uint64_t t = 0; t < steps; ++t) {
    uint32_t* src = net->xs[net->cur].as<uint32_t>();
    uint32_t* dst = net->xs[net->cur ^ 1].as<uint32_t>();
    const bool tm = net->timing && t < net->ev_a.size();
    if (tm) CK("net_steps", cudaEventRecord(net->ev_a[t], net->stream));
    const bool fork = net->blocks.size() > 1;
    if (fork) {
      CK("net_steps", cudaEventRecord(net->ev_fork, net->stream));
      CK("net_steps", cudaStreamWaitEvent(net->side, net->ev_fork, 0));
    }
    const bool peer = net->nranks > 1 && net->exchange == SPARSL_NET_EXCHANGE_PEER;
    const int q = net->cur ^ 1;  // parity of the destination copy
    const size_t nb = net->blocks.size();
    bool all_pushed = true;
    for (size_t b = 0; b < nb; ++b) {
      sparsl_op* op = net->blocks[b];
      if (!op->nrows) continue;
      RowLaunch p = fwd_launch(op);
      set_bits_mode(p, src, net->words);
      lif_resident_launch(op, p, decay, v_reset, dtheta);
      p.out_bits = dst + (net->row_offset + net->block_off[b]) / 32;
      p.err = net->err.d;
      if (hv && t == 0) {
        p.v_src = hv + net->block_off[b];
        p.theta_src = hth + net->block_off[b];
      }
      if (hv && t + 1 == steps) {
        p.v_mirror = hv + net->block_off[b];
        p.theta_mirror = hth + net->block_off[b];
      }
      // The TMA tick stores its words into the peers' copies itself.
      if (peer && op->ell.ok) {
        p.peer_out = net->peer_out.as<uint32_t*>() + (q * nb + b) * net->nranks;
        p.npeers = (uint32_t)net->nranks;
        p.tick_count = net->tick_count.as<uint32_t>();
      } else {
        all_pushed = false;
      }
      cudaStream_t bs = (b & 1) ? net->side : net->stream;
      if (in_ev && t == 0) CK("net_steps", cudaStreamWaitEvent(bs, in_ev[b], 0));
      CK("net_steps", launch_fwd(op, p, bs));
      if (out_ev && t + 1 == steps) CK("net_steps", cudaEventRecord(out_ev[b], bs));
    }
    if (fork) {
      CK("net_steps", cudaEventRecord(net->ev_join, net->side));
      CK("net_steps", cudaStreamWaitEvent(net->stream, net->ev_join, 0));
    }
    if (tm) CK("net_steps", cudaEventRecord(net->ev_b[t], net->stream));
    if (peer) {
      NetExchange x;
      x.self = (uint32_t)net->rank;
      x.nranks = (uint32_t)net->nranks;
      x.local_words = dst + net->row_offset / 32;
      x.nwords = (uint32_t)(net->local_rows / 32);
      x.peer_words = net->peer_slice.as<uint32_t*>() + q * net->nranks;
      x.push = !all_pushed;
      x.count = all_pushed ? net->tick_count.as<uint32_t>() : nullptr;
      x.peer_box = net->peer_box.as<NetMailbox*>();
      x.my_box = net->box.as<NetMailbox>();
      x.tick = net->tick++;
      // Half the host's deadline (at most 30 s): an expired wait is reported
      // through the error word before the host would give up on the stream.
      x.wait_ns = std::min<uint64_t>(g_timeout_ms.load() / 2, 30000) * 1000000ull;
      x.trace_slot = net->trace.as<uint32_t>() + t;
      x.err = net->err.d;
      CK("net_steps", launch_net_exchange(x, net->stream));
      net->cur ^= 1;
      continue;
    }
    if (net->nranks > 1) {
      ncclResult_t r = nccl_settle(
          net->comm, g_nccl.AllGather(dst + (uint64_t)net->rank * slice, dst, slice, ncclUint32, net->comm, net->stream));
      if (r == ncclInProgress) return fail(SPARSL_ERR_EXECUTION, "ncclAllGather", "ncclAllGather was not enqueued in time");
      if (r != ncclSuccess) return fail(SPARSL_ERR_EXECUTION, "ncclAllGather failed", g_nccl.GetErrorString(r));
    }
    CK("net_steps", launch_popcount(dst, net->words, net->trace.as<uint32_t>() + t, net->stream));
    net->cur ^= 1;
  }
  net->last_steps = steps;
  net->timed_ticks = net->timing ? std::min<uint64_t>(steps, net->ev_a.size()) : 0;
  return SPARSL_OK;
}

int sparsl_net_steps_async(sparsl_net* net, float decay, float v_reset, float dtheta, uint64_t steps) {
  ADMIT();
  if (steps == 0) return SPARSL_OK;
  CK("net_steps", cudaSetDevice(net->dev->ordinal));
  return net_enqueue(net, decay, v_reset, dtheta, steps);
}

int sparsl_net_wait(sparsl_net* net) {
  ADMIT();
  CK("net_wait", cudaSetDevice(net->dev->ordinal));
  int rc = wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_steps");
  if (rc != SPARSL_OK && net->comm && g_quarantine.load()) {
    g_nccl.CommAbort(net->comm);
    net->comm = nullptr;
  }
  return rc;
}

int sparsl_net_steps(sparsl_net* net, float decay, float v_reset, float dtheta, uint64_t steps) {
  TRY(sparsl_net_steps_async(net, decay, v_reset, dtheta, steps));
  return sparsl_net_wait(net);
}

int sparsl_net_read_state(sparsl_net* net, uint32_t* xs, uint64_t words, float* v, float* theta, uint64_t local_rows) {
  ADMIT();
  TRY(check_min("x_spikes", words, net->words));
  TRY(check_len("v", local_rows, net->local_rows));
  CK("net_read_state", cudaSetDevice(net->dev->ordinal));
  CK("net_read_state", cudaMemcpyAsync(xs, net->xs[net->cur].p, net->words * 4, cudaMemcpyDeviceToHost, net->stream));
  CanarySet set;
  set.ptr[set.count++] = net->xs[0].canary();
  set.ptr[set.count++] = net->xs[1].canary();
  for (size_t b = 0; b < net->blocks.size(); ++b) {
    sparsl_op* op = net->blocks[b];
    const uint64_t o = net->block_off[b];
    if (!op->nrows) continue;
    CK("net_read_state", cudaMemcpyAsync(v + o, op->rv.p, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, net->stream));
    CK("net_read_state", cudaMemcpyAsync(theta + o, op->rth.p, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, net->stream));
    if (set.count + 2 <= CanarySet::kMax) {
      set.ptr[set.count++] = op->rv.canary();
      set.ptr[set.count++] = op->rth.canary();
    }
  }
  CK("net_read_state", launch_canary_check(set, net->err.d, net->stream));
  return wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_read_state");
}

int sparsl_net_steps_host(sparsl_net* net, uint32_t* xs, uint64_t words, float* v, float* theta, uint64_t local_rows,
                          float decay, float v_reset, float dtheta, uint64_t steps) {
  ADMIT();
  TRY(check_min("x_spikes", words, net->words));
  TRY(check_len("v", local_rows, net->local_rows));
  if (steps == 0) return SPARSL_OK;
  CK("net_steps_host", cudaSetDevice(net->dev->ordinal));
  const size_t nb = net->blocks.size();
  // Pinned host arrays that this device can address: the first tick reads
  // the state from them and the last one writes it back, over PCIe, from
  // inside the tick kernels (a tile's state is loaded when its stream
  // starts).  Only the spike vector is copied.
  void *dv = nullptr, *dth = nullptr;
  if (host_mapped(v, &dv) && host_mapped(theta, &dth)) {
    CK("net_steps_host", cudaMemcpyAsync(net->xs[net->cur].p, xs, net->words * 4, cudaMemcpyHostToDevice, net->stream));
    TRY(net_enqueue(net, decay, v_reset, dtheta, steps, nullptr, nullptr, static_cast<float*>(dv),
                    static_cast<float*>(dth)));
    CK("net_steps_host", cudaMemcpyAsync(xs, net->xs[net->cur].p, net->words * 4, cudaMemcpyDeviceToHost, net->stream));
    CanarySet set;
    set.ptr[set.count++] = net->xs[0].canary();
    set.ptr[set.count++] = net->xs[1].canary();
    for (size_t b = 0; b < nb && set.count + 2 <= CanarySet::kMax; ++b) {
      if (!net->blocks[b]->nrows) continue;
      set.ptr[set.count++] = net->blocks[b]->rv.canary();
      set.ptr[set.count++] = net->blocks[b]->rth.canary();
    }
    CK("net_steps_host", launch_canary_check(set, net->err.d, net->stream));
    int rc = wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_steps_host");
    if (rc != SPARSL_OK && net->comm && g_quarantine.load()) {
      g_nccl.CommAbort(net->comm);
      net->comm = nullptr;
    }
    return rc;
  }
  if (!net->copy_in) {
    // All or nothing: the net keeps the streams and events only when every
    // one of them was made.
    cudaStream_t ci = nullptr, co = nullptr;
    cudaEvent_t cp = nullptr;
    std::vector<cudaEvent_t> ei(nb, nullptr), eo(nb, nullptr);
    bool ok = cudaStreamCreateWithFlags(&ci, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&co, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&cp, cudaEventDisableTiming) == cudaSuccess;
    for (size_t b = 0; ok && b < nb; ++b)
      ok = cudaEventCreateWithFlags(&ei[b], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&eo[b], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
      const cudaError_t e = cudaGetLastError();
      for (cudaEvent_t x : ei)
        if (x) cudaEventDestroy(x);
      for (cudaEvent_t x : eo)
        if (x) cudaEventDestroy(x);
      if (cp) cudaEventDestroy(cp);
      if (co) cudaStreamDestroy(co);
      if (ci) cudaStreamDestroy(ci);
      return fail(SPARSL_ERR_BACKEND, "copy stream creation failed", cudaGetErrorString(e));
    }
    net->copy_in = ci;
    net->copy_out = co;
    net->ev_copied = cp;
    net->ev_in = std::move(ei);
    net->ev_out = std::move(eo);
  }
  // Work already on the net's stream (an earlier sparsl_net_steps_async)
  // ends before copy_in overwrites any state.
  CK("net_steps_host", cudaEventRecord(net->ev_copied, net->stream));
  CK("net_steps_host", cudaStreamWaitEvent(net->copy_in, net->ev_copied, 0));
  // The spike vector first, on the net's stream (every block's first tick
  // reads all of it), then each block's v and theta on copy_in.
  CK("net_steps_host", cudaMemcpyAsync(net->xs[net->cur].p, xs, net->words * 4, cudaMemcpyHostToDevice, net->stream));
  for (size_t b = 0; b < nb; ++b) {
    sparsl_op* op = net->blocks[b];
    const uint64_t o = net->block_off[b];
    if (op->nrows) {
      CK("net_steps_host", cudaMemcpyAsync(op->rv.p, v + o, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, net->copy_in));
      CK("net_steps_host",
         cudaMemcpyAsync(op->rth.p, theta + o, (uint64_t)op->nrows * 4, cudaMemcpyHostToDevice, net->copy_in));
    }
    CK("net_steps_host", cudaEventRecord(net->ev_in[b], net->copy_in));
  }
  TRY(net_enqueue(net, decay, v_reset, dtheta, steps, net->ev_in.data(), net->ev_out.data()));
  CanarySet set;
  set.ptr[set.count++] = net->xs[0].canary();
  set.ptr[set.count++] = net->xs[1].canary();
  for (size_t b = 0; b < nb; ++b) {
    sparsl_op* op = net->blocks[b];
    const uint64_t o = net->block_off[b];
    if (!op->nrows) continue;
    CK("net_steps_host", cudaStreamWaitEvent(net->copy_out, net->ev_out[b], 0));
    CK("net_steps_host", cudaMemcpyAsync(v + o, op->rv.p, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, net->copy_out));
    CK("net_steps_host",
       cudaMemcpyAsync(theta + o, op->rth.p, (uint64_t)op->nrows * 4, cudaMemcpyDeviceToHost, net->copy_out));
    if (set.count + 2 <= CanarySet::kMax) {
      set.ptr[set.count++] = op->rv.canary();
      set.ptr[set.count++] = op->rth.canary();
    }
  }
  // The spike vector after the last tick (and its exchange), then join.
  CK("net_steps_host", cudaMemcpyAsync(xs, net->xs[net->cur].p, net->words * 4, cudaMemcpyDeviceToHost, net->stream));
  CK("net_steps_host", cudaEventRecord(net->ev_copied, net->copy_out));
  CK("net_steps_host", cudaStreamWaitEvent(net->stream, net->ev_copied, 0));
  CK("net_steps_host", launch_canary_check(set, net->err.d, net->stream));
  int rc = wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_steps_host");
  if (rc != SPARSL_OK && net->comm && g_quarantine.load()) {
    g_nccl.CommAbort(net->comm);
    net->comm = nullptr;
  }
  return rc;
}

int sparsl_net_set_timing(sparsl_net* net, uint64_t max_ticks) {
  if (!net) return fail(SPARSL_ERR_INVALID, "null net", "null net");
  CK("net_set_timing", cudaSetDevice(net->dev->ordinal));
  CK("net_set_timing", cudaStreamSynchronize(net->stream));
  for (cudaEvent_t e : net->ev_a) cudaEventDestroy(e);
  for (cudaEvent_t e : net->ev_b) cudaEventDestroy(e);
  net->ev_a.clear();
  net->ev_b.clear();
  net->timing = max_ticks > 0;
  for (uint64_t i = 0; i < max_ticks; ++i) {
    cudaEvent_t a, b;
    CK("net_set_timing", cudaEventCreate(&a));
    CK("net_set_timing", cudaEventCreate(&b));
    net->ev_a.push_back(a);
    net->ev_b.push_back(b);
  }
  return SPARSL_OK;
}

int sparsl_net_kernel_ms(sparsl_net* net, double* total_ms, uint64_t* ticks) {
  if (!net) return fail(SPARSL_ERR_INVALID, "null net", "null net");
  CK("net_kernel_ms", cudaSetDevice(net->dev->ordinal));
  CK("net_kernel_ms", cudaStreamSynchronize(net->stream));
  double sum = 0.0;
  for (uint64_t t = 0; t < net->timed_ticks; ++t) {
    float ms = 0.f;
    CK("net_kernel_ms", cudaEventElapsedTime(&ms, net->ev_a[t], net->ev_b[t]));
    sum += ms;
  }
  if (total_ms) *total_ms = sum;
  if (ticks) *ticks = net->timed_ticks;
  return SPARSL_OK;
}

int sparsl_net_set_exchange(sparsl_net* net, int mode) {
  if (!net) return fail(SPARSL_ERR_INVALID, "null net", "null net");
  if (mode != SPARSL_NET_EXCHANGE_PEER && mode != SPARSL_NET_EXCHANGE_NCCL)
    return fail(SPARSL_ERR_INVALID, "exchange mode", "unknown exchange mode");
  CK("net_set_exchange", cudaSetDevice(net->dev->ordinal));
  CK("net_set_exchange", cudaStreamSynchronize(net->stream));
  net->exchange = mode;
  return SPARSL_OK;
}

int sparsl_net_tick_ms(sparsl_net* net, float* out, uint64_t cap, uint64_t* n_out) {
  if (!net) return fail(SPARSL_ERR_INVALID, "null net", "null net");
  CK("net_tick_ms", cudaSetDevice(net->dev->ordinal));
  CK("net_tick_ms", cudaStreamSynchronize(net->stream));
  if (n_out) *n_out = net->timed_ticks;
  const uint64_t n = std::min<uint64_t>(cap, net->timed_ticks);
  for (uint64_t t = 0; t < n; ++t) CK("net_tick_ms", cudaEventElapsedTime(&out[t], net->ev_a[t], net->ev_b[t]));
  return SPARSL_OK;
}

int sparsl_net_trace(sparsl_net* net, uint32_t* out, uint64_t cap, uint64_t* n_out) {
  ADMIT();
  CK("net_trace", cudaSetDevice(net->dev->ordinal));
  const uint64_t n = std::min<uint64_t>(cap, net->last_steps);
  if (n_out) *n_out = net->last_steps;
  if (n) CK("net_trace", cudaMemcpyAsync(out, net->trace.p, n * 4, cudaMemcpyDeviceToHost, net->stream));
  return wait_bounded(net->stream, net->ev, net->err.d, net->err.h, "net_trace");
}

}  // extern "C"
