// gemm_launch_noalloc: the kernel bank's launch for callers that must not
// allocate device memory.
//
// Who needs it: a GEMM called from code that is handed only input/output
// pointers and a stream -- for example a custom operator inside a runtime
// that plans every device buffer ahead of time, or a plugin living beside a
// framework whose caching allocator has already reserved almost all of the
// GPU's memory.  Such callers cannot cudaMalloc a workspace (it may fail, it
// fragments the other allocator's pool, and cudaMalloc/cudaFree can
// synchronise the device), yet split-K and the repacking of unaligned
// operands need scratch memory.
//
// How: the scratch lives in one file-scope __device__ array of
// GEMM_NOALLOC_SCRATCH_BYTES (32 MiB), which every GPU that loads this
// library holds until the process exits.  Host code cannot use the array's
// name as a device address, so the first call on each device looks the
// address up with cudaGetSymbolAddress (with that device current) and caches
// it; make that first call before any stream capture.  Each call then clears
// the split-K ticket region (cudaMemsetAsync on the caller's stream) and
// hands the array to gemm_launch as its workspace -- the kernels and the
// launch path are exactly those of gemm_launch.
//
// Limits: a problem whose workspace (gemm_workspace_bytes) exceeds the
// array is rejected with GEMM_ERR_WORKSPACE before anything is launched.
// All calls on a device share the one array and it keeps the last call's
// contents, so calls whose kernels overlap on the GPU (different streams,
// or different host threads) race on it; serialise them.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/gemm_sm100.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[GEMM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
cudaError_t g_scratch_status[kMaxDevices] = {};
std::once_flag g_scratch_once[kMaxDevices];

}  // namespace

namespace idb {
// Records the message gemm_last_error() returns (defined with it in gemm_capi.cu).
void record_last_error(const std::string& msg);
}  // namespace idb

extern "C" int gemm_launch_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                   int64_t lda, int64_t ldb, int64_t ldc, int cfg_id, void* stream) {
  const size_t need = gemm_workspace_bytes(A, B, M, N, K, lda, ldb, cfg_id);
  if (need > GEMM_NOALLOC_SCRATCH_BYTES) {
    idb::record_last_error("gemm_launch_noalloc: this problem needs " + std::to_string(need) +
                           " bytes of scratch, more than the fixed " +
                           std::to_string(static_cast<size_t>(GEMM_NOALLOC_SCRATCH_BYTES)) +
                           "-byte static buffer; use gemm_launch with a workspace or a smaller split_k");
    return GEMM_ERR_WORKSPACE;
  }
  if (need == 0) {
    // No scratch needed (or invalid arguments, which gemm_launch reports).
    return gemm_launch(A, B, C, M, N, K, lda, ldb, ldc, cfg_id, nullptr, 0, stream);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    idb::record_last_error(std::string("gemm_launch_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    return GEMM_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    idb::record_last_error("gemm_launch_noalloc: device index " + std::to_string(dev) + " out of range [0, " +
                           std::to_string(kMaxDevices) + ")");
    return GEMM_ERR_UNSUPPORTED;
  }
  // Set-up, once per device, with that device current.
  std::call_once(g_scratch_once[dev], [dev] {
    void* p = nullptr;
    g_scratch_status[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_scratch_ptr[dev] = (g_scratch_status[dev] == cudaSuccess) ? p : nullptr;
  });
  if (g_scratch_status[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr) {
    idb::record_last_error(std::string("gemm_launch_noalloc: cudaGetSymbolAddress: ") +
                           cudaGetErrorString(g_scratch_status[dev]));
    return GEMM_ERR_CUDA;
  }
  // The ticket region must start at zero; the array keeps the previous
  // call's contents (and an aborted launch could leave tickets set).
  const size_t tickets = gemm_workspace_counter_bytes();
  e = cudaMemsetAsync(g_scratch_ptr[dev], 0, tickets < need ? tickets : need, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    idb::record_last_error(std::string("gemm_launch_noalloc: cudaMemsetAsync: ") + cudaGetErrorString(e));
    return GEMM_ERR_CUDA;
  }
  return gemm_launch(A, B, C, M, N, K, lda, ldb, ldc, cfg_id, g_scratch_ptr[dev], GEMM_NOALLOC_SCRATCH_BYTES,
                     stream);
}
