// Streaming probe for the skinny kernel's access patterns: TMA reads of an
// fp16 B [K x N] (N contiguous) with the kernel's boxes ([64 K x 64 n],
// 128-byte swizzle) and ring depths, but no MMA and no epilogue.  Each
// stage is released as soon as it lands, so the time is what streaming B
// alone costs in that pattern.  It is a measurement tool, not part of the
// library, and build.py does not compile it.
//
// Patterns (one line each on stdout):
//   * W columns per CTA, K split into S ranges, free-running CTAs;
//   * clusters of G adjacent column blocks held in step: every CTA's stage
//     s is released only after all G CTAs consumed their stage s, by a
//     remote mbarrier arrive (lock 1: .release.cluster, lock 2:
//     .relaxed.cluster) or a multicast tcgen05.commit (lock 3);
//   * a stream-K walk of (column block, K block) iterations over 148 CTAs.
//
// Build and run on a B200:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -I infinite-dreams_b200/csrc -o tma_stream_probe \
//        infinite-dreams_b200/probes/tma_stream_probe.cu -lcuda
//   ./tma_stream_probe
// Every wait is bounded (1 s); a timeout sets a bit in the printed error word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "sm100_ptx.cuh"

using namespace idb;

namespace {

constexpr uint64_t kProbeWaitNs = 1000000000ull;

__device__ __forceinline__ bool wait_full(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_limit(bar, parity, abort_flag, kProbeWaitNs);
}

template <int BOXES, int STAGES>
__global__ void __launch_bounds__(128, 1)
    stream_probe(const __grid_constant__ CUtensorMap tm, int ncb, int kb_total, int S, int lock, int sk_ctas,
                 int* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStage = BOXES * 64 * 64 * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStage);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int G = static_cast<int>(cluster_nctarank());
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], lock ? G : 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  cluster_sync();  // peers' barriers are initialised before any remote arrive
  // this CTA's iterations, (column block, K block) linearised column-block-major
  long long it0, it1;
  const int b = static_cast<int>(blockIdx.x);
  if (sk_ctas > 0) {
    const long long total = static_cast<long long>(ncb) * kb_total;
    it0 = total * b / sk_ctas;
    it1 = total * (b + 1) / sk_ctas;
  } else {
    const int ks = b / ncb, c = b % ncb;
    it0 = static_cast<long long>(c) * kb_total + static_cast<long long>(ks) * kb_total / S;
    it1 = static_cast<long long>(c) * kb_total + static_cast<long long>(ks + 1) * kb_total / S;
  }
  if (warp == 0 && lane == 0) {
    int stage = 0, issued = 0;
    uint32_t phase = 0;
    for (long long it = it0; it < it1; ++it) {
      if (issued >= STAGES && !wait_full(&empty[stage], phase ^ 1u, abort_flag)) {
        atomicOr(err, 1);
        *abort_flag = 1;
        break;
      }
      const int c = static_cast<int>(it / kb_total), kb = static_cast<int>(it % kb_total);
      mbar_arrive_expect_tx(&full[stage], kStage);
      for (int h = 0; h < BOXES; ++h) {
        tma_load_2d(smem + stage * kStage + h * 8192, &tm, &full[stage], c * BOXES * 64 + h * 64, kb * 64);
      }
      ++issued;
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // every issued fill lands before the CTA exits
    const int outstanding = issued < STAGES ? issued : STAGES;
    for (int i = 0; i < outstanding; ++i) {
      stage = (stage == 0) ? STAGES - 1 : stage - 1;
      if (stage == STAGES - 1) phase ^= 1u;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[stage], phase)) {
        if (globaltimer_ns() - t0 > kProbeWaitNs) {
          atomicOr(err, 2);
          break;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (long long it = it0; it < it1; ++it) {
      if (!wait_full(&full[stage], phase, abort_flag)) {
        atomicOr(err, 4);
        *abort_flag = 1;
        break;
      }
      if (lock == 1) {
        for (int q = 0; q < G; ++q) mbar_arrive_cluster(mapa_shared(smem_u32(&empty[stage]), q));
      } else if (lock == 2) {
        for (int q = 0; q < G; ++q) {
          asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                           mapa_shared(smem_u32(&empty[stage]), q))
                       : "memory");
        }
      } else if (lock == 3) {
        const uint16_t mask = static_cast<uint16_t>((1u << G) - 1u);
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                smem_u32(&empty[stage])),
            "h"(mask)
            : "memory");
      } else {
        mbar_arrive(&empty[stage]);
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  __syncwarp();
  cluster_sync();  // no CTA leaves while a peer may still arrive on its barriers
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

void check(cudaError_t e, int line) {
  if (e != cudaSuccess) {
    std::printf("CUDA error %s at line %d\n", cudaGetErrorString(e), line);
    std::exit(1);
  }
}
#define CHECK(x) check((x), __LINE__)

// Median time in ms of `reps` launches, each after a 512 MiB memset that
// flushes L2; every grid is checked against its cluster size first.
template <int BOXES, int STAGES>
float run(const CUtensorMap& tm, int N, int K, int S, int G, int lock, int sk, int* err, void* flush,
          size_t flush_bytes, int reps) {
  auto kern = stream_probe<BOXES, STAGES>;
  const int smem = STAGES * BOXES * 8192 + 2 * STAGES * 8 + 16 + 1024;
  CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int ncb = N / (BOXES * 64), kbt = K / 64;
  const int grid = sk ? sk : ncb * S;
  if (grid % G != 0 || N % (BOXES * 64) != 0 || K % 64 != 0) return -1.0f;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(G);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaEvent_t a, b;
  CHECK(cudaEventCreate(&a));
  CHECK(cudaEventCreate(&b));
  std::vector<float> ts;
  for (int r = 0; r < reps + 2; ++r) {
    CHECK(cudaMemsetAsync(flush, r & 0xff, flush_bytes));
    CHECK(cudaEventRecord(a));
    CHECK(cudaLaunchKernelEx(&cfg, kern, tm, ncb, kbt, S, lock, sk, err));
    CHECK(cudaEventRecord(b));
    CHECK(cudaEventSynchronize(b));
    float ms = 0.0f;
    CHECK(cudaEventElapsedTime(&ms, a, b));
    if (r >= 2) ts.push_back(ms);
  }
  CHECK(cudaEventDestroy(a));
  CHECK(cudaEventDestroy(b));
  std::sort(ts.begin(), ts.end());
  return ts[ts.size() / 2];
}

}  // namespace

int main() {
  void* fnp = nullptr;
  cudaDriverEntryPointQueryResult q;
  CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fnp, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess) return 1;
  EncodeFn enc = reinterpret_cast<EncodeFn>(fnp);
  int* err = nullptr;
  CHECK(cudaMalloc(&err, sizeof(int)));
  CHECK(cudaMemset(err, 0, sizeof(int)));
  const size_t flush_bytes = 512ull << 20;
  void* flush = nullptr;
  CHECK(cudaMalloc(&flush, flush_bytes));
  const int shapes[2][2] = {{14336, 4096}, {4096, 4096}};
  for (const auto& sh : shapes) {
    const int N = sh[0], K = sh[1];
    void* B = nullptr;
    CHECK(cudaMalloc(&B, static_cast<size_t>(N) * K * 2));
    CHECK(cudaMemset(B, 0, static_cast<size_t>(N) * K * 2));
    CUtensorMap tm;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
    const cuuint32_t box[2] = {64, 64}, es[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      std::printf("tensor map encode failed\n");
      return 1;
    }
    const double bytes = static_cast<double>(N) * K * 2;
    auto line = [&](const char* name, float ms) {
      std::printf("N=%5d K=%d %-34s %8.2f us %7.0f GB/s\n", N, K, name, ms * 1e3, bytes / (ms * 1e-3) / 1e9);
      std::fflush(stdout);
    };
    const int S = (N == 4096) ? 4 : 1;
    char name[96];
    for (int G : {1, 2, 4}) {
      for (int lock : {0, 1, 2, 3}) {
        if (G == 1 && lock != 0) continue;
        std::snprintf(name, sizeof name, "W128 st12 S%d G%d lock%d", S, G, lock);
        line(name, run<2, 12>(tm, N, K, S, G, lock, 0, err, flush, flush_bytes, 9));
      }
    }
    if (N == 14336) line("W256 st6 S2 G1", run<4, 6>(tm, N, K, 2, 1, 0, 0, err, flush, flush_bytes, 9));
    line("W256 st6 streamK 148", run<4, 6>(tm, N, K, 1, 1, 0, 148, err, flush, flush_bytes, 9));
    line("W512 st3 streamK 148", run<8, 3>(tm, N, K, 1, 1, 0, 148, err, flush, flush_bytes, 9));
    CHECK(cudaFree(B));
  }
  int herr = 0;
  CHECK(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost));
  std::printf("device error word: %d\n", herr);
  CHECK(cudaFree(flush));
  CHECK(cudaFree(err));
  return herr != 0;
}
