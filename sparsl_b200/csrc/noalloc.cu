// Allocation-free entry point for the exact affine-map scan.
//
// Some callers cannot allocate device memory at all: a host whose allocator
// owns every byte of HBM up front (a framework memory pool, or a Rust host
// that hands this library only the buffers it already holds), or code running
// where a cudaMalloc would be refused or would stall the device.  For them the
// scan's scratch -- look-back records, boundary counters, mismatch bitmaps and
// the device error word -- lives in a file-scope __device__ array instead of
// an allocation.  Every GPU that loads this library keeps that array resident
// until the process exits.
//
// The call follows the library's admission and quarantine rules: it is
// refused while the backend is quarantined, it counts as work in flight for
// sparsl_device_reset, and a timeout, a device fault or a set device error
// word quarantines the backend.  After a timeout the scan may still be
// running on the shared array; the quarantine keeps every later call (this
// one included) from clearing the array under it until the caller has let the
// stream drain and called sparsl_device_reset.
#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "../../include/sparsl_cuda.h"
#include "scan.cuh"

namespace sparsl {
// capi.cu
int record_error(int code, const char* message);
int record_error_detail(int code, const char* reason, const std::string& detail);
bool admission_enter();
void admission_leave();
void quarantine_backend();
uint64_t timeout_ms_setting();
int check_device_array(const void* p, uint64_t bytes, int ordinal, const char* what);
std::string describe_device_error(uint32_t bits);
}  // namespace sparsl

namespace {

// Largest scan this entry point accepts, and the static scratch it needs.
constexpr uint64_t kNoAllocMaxMaps = 1ull << 22;  // 4,194,304 maps
constexpr size_t kNoAllocBytes = 256 * 1024;      // covers scan_scratch_bytes(kNoAllocMaxMaps) + error word

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device

// Failures are reported through sparsl_last_error / sparsl_last_reason.
int set_msg(int code, const char* m) { return sparsl::record_error(code, m); }

// Counts the call as admitted work for as long as it runs.
struct Admitted {
  bool ok = sparsl::admission_enter();
  ~Admitted() { sparsl::admission_leave(); }
};

}  // namespace

extern "C" int sparsl_dev_assoc_scan_noalloc(int ordinal, const float* d_in, uint64_t n, float* d_out,
                                             void* stream, uint64_t timeout_ms) {
  Admitted adm;
  if (!adm.ok)
    return set_msg(SPARSL_ERR_BACKEND,
                   "assoc_scan_noalloc: CUDA backend is quarantined; call sparsl_device_reset once no work is in "
                   "flight");
  if (n > kNoAllocMaxMaps)
    return set_msg(SPARSL_ERR_LENGTH, "assoc_scan_noalloc: n exceeds the allocation-free maximum of 4194304 maps");
  if (n == 0) return SPARSL_OK;
  if (!d_in || !d_out) return set_msg(SPARSL_ERR_INVALID, "assoc_scan_noalloc: null buffer");
  if (ordinal < 0 || ordinal >= kMaxDevices) return set_msg(SPARSL_ERR_BACKEND, "assoc_scan_noalloc: bad device");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int prev = -1;
  cudaGetDevice(&prev);
  if (cudaSetDevice(ordinal) != cudaSuccess) return set_msg(SPARSL_ERR_BACKEND, "assoc_scan_noalloc: cudaSetDevice failed");
  int rc = SPARSL_OK;
  do {
    // The call polls the stream and reads the error word back, neither of
    // which a stream capture allows: refuse instead of breaking the capture.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
      cudaGetLastError();
      rc = set_msg(SPARSL_ERR_INVALID, "assoc_scan_noalloc: the stream is being captured; this call cannot be captured");
      break;
    }
    // Caller buffers: device memory of this GPU, each inside one allocation.
    if ((rc = sparsl::check_device_array(d_in, n * 8, ordinal, "assoc_scan_noalloc input")) != SPARSL_OK) break;
    if ((rc = sparsl::check_device_array(d_out, n * 8, ordinal, "assoc_scan_noalloc output")) != SPARSL_OK) break;
    // Set-up, once per device with that device current: the host-side name of
    // the array is only a stand-in, so fetch its device address.
    void* base = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      if (!g_addr[ordinal]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
          cudaGetLastError();
          rc = set_msg(SPARSL_ERR_BACKEND, "assoc_scan_noalloc: cudaGetSymbolAddress failed");
          break;
        }
        g_addr[ordinal] = p;
      }
      base = g_addr[ordinal];
    }
    const size_t need = sparsl::scan_scratch_bytes(kNoAllocMaxMaps);
    if (need + 256 > kNoAllocBytes) {
      rc = set_msg(SPARSL_ERR_BACKEND, "assoc_scan_noalloc: static scratch too small");
      break;
    }
    uint32_t* err = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(base) + kNoAllocBytes - 256);
    // The array keeps the last call's contents; clear everything that must
    // start at zero (look-back records, tickets, counters, error word).
    if (cudaMemsetAsync(base, 0, kNoAllocBytes, s) != cudaSuccess) {
      rc = set_msg(SPARSL_ERR_EXECUTION, "assoc_scan_noalloc: clearing the scratch failed");
      break;
    }
    const sparsl::ScanScratch sc = sparsl::scan_scratch_carve(base, kNoAllocMaxMaps);
    if (sparsl::launch_scan(d_in, d_out, n, sc, err, s) != cudaSuccess) {
      rc = set_msg(SPARSL_ERR_EXECUTION, "assoc_scan_noalloc: launch failed");
      break;
    }
    // Bounded wait on the caller's stream (the process-wide timeout unless
    // the caller gives one), then the device error word.
    const uint64_t limit_ms = timeout_ms ? timeout_ms : sparsl::timeout_ms_setting();
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t q;
    uint64_t polls = 0;
    while ((q = cudaStreamQuery(s)) == cudaErrorNotReady) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(limit_ms)) {
        sparsl::quarantine_backend();
        rc = sparsl::record_error_detail(
            SPARSL_ERR_EXECUTION, "assoc_scan_noalloc timed out",
            "assoc_scan_noalloc: did not complete within " + std::to_string(limit_ms) +
                " ms; backend quarantined (the scan may still be running on the shared scratch: let the stream "
                "drain, then call sparsl_device_reset)");
        break;
      }
      if (++polls > 200) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    if (rc != SPARSL_OK) break;
    if (q != cudaSuccess) {
      sparsl::quarantine_backend();
      rc = sparsl::record_error_detail(SPARSL_ERR_EXECUTION, "assoc_scan_noalloc device failure",
                                       std::string("assoc_scan_noalloc: device execution failed: ") +
                                           cudaGetErrorString(q) + "; backend quarantined");
      break;
    }
    // The stream was just seen idle, so this copy on it completes at once
    // (it does not queue behind work on other streams).
    uint32_t word = 0;
    const cudaError_t ce = cudaMemcpyAsync(&word, err, sizeof word, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess && cudaStreamSynchronize(s) == cudaSuccess && word == 0) break;
    sparsl::quarantine_backend();
    rc = sparsl::record_error_detail(SPARSL_ERR_EXECUTION, "assoc_scan_noalloc device error",
                                     "assoc_scan_noalloc: " +
                                         (ce != cudaSuccess ? std::string(cudaGetErrorString(ce))
                                                            : sparsl::describe_device_error(word)) +
                                         "; backend quarantined");
  } while (false);
  if (prev >= 0) cudaSetDevice(prev);
  return rc;
}
