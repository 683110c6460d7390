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

template <int BN, int STAGES, int CG>
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, const GemmParams& p,
                        int grid, cudaStream_t stream) {
  using Plan = SmemPlan<BN, STAGES, CG>;
  auto kernel = gemm_f16_sm100<BN, STAGES, CG>;
  // The opt-in shared-memory size is a per-device function attribute.
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Plan::kDynamicBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  // Programmatic dependent launch: the kernel's set-up may overlap the end
  // of the previous grid in the stream (it waits with griddepcontrol.wait
  // before touching global memory).  CTA pairs: a cluster of 2 along x.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = Plan::kDynamicBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = CG == 2 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, a, b, c, p);
}

}  // namespace idb

#define IDB_DEFINE_VARIANT(BN, ST, CG)                                                                    \
  cudaError_t launch_bn##BN##_s##ST##_cg##CG(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, \
                                             const GemmParams& p, int grid, cudaStream_t stream) {        \
    return launch_gemm<BN, ST, CG>(a, b, c, p, grid, stream);                                            \
  }
