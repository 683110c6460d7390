// Shared by the generated bank files (csrc/generated/gemm_bank_bn*.cu): one
// host launcher per compiled (tile_n, stages) instantiation of the kernel.
// Plays the role of the reference's TRY_CFG launch macro
// (src/gemm_kernels.cuh:87-96), but is reached through a table lookup by
// cfg_id instead of a linear chain of 5-tuple compares.
#pragma once
#include <atomic>
#include <cuda_runtime.h>

#include "gemm_sm100_kernel.cuh"

namespace idb {

using LaunchFn = cudaError_t (*)(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c,
                                 const GemmParams& p, int grid, cudaStream_t stream);

template <int BN, int STAGES>
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, const GemmParams& p,
                        int grid, cudaStream_t stream) {
  using Plan = SmemPlan<BN, STAGES>;
  // The opt-in shared-memory size is a per-device function attribute.
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(gemm_f16_sm100<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Plan::kDynamicBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  gemm_f16_sm100<BN, STAGES><<<grid, kNumThreads, Plan::kDynamicBytes, stream>>>(a, b, c, p);
  return cudaGetLastError();
}

}  // namespace idb

#define IDB_DEFINE_VARIANT(BN, ST)                                                                        \
  cudaError_t launch_bn##BN##_s##ST(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c,   \
                                    const GemmParams& p, int grid, cudaStream_t stream) {               \
    return launch_gemm<BN, ST>(a, b, c, p, grid, stream);                                               \
  }
