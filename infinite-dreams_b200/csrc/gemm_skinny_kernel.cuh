// Skinny FP16 GEMM (few rows of A) for sm_100a:  C[M,N] = A[M,K] * B[K,N].
//
// Same arithmetic as the reference kernel (src/gemm_kernels.cuh:6-83): fp16
// operands, fp32 accumulation, one rounding to fp16 (plus the optional fused
// epilogue of gemm_launch_ex).  Built for M <= 64, where a 128-row MMA tile
// would be mostly zero fill and the cost is streaming B from HBM:
//
//  * operands swapped: the MMA computes C^T = B^T A^T, so 128 columns of C
//    fill the 128 TMEM lanes (MMA M = 128) and the few rows of A are the MMA
//    N (TM = 16, 32 or 64).  A cluster owns TN = 128, 256 or 512 columns of
//    C (one, two or four MMAs per K step).  Per pipeline stage a CTA loads a
//    [64 K x TN] tile of B (16, 32 or 64 KiB, all useful) and a [TM x 64 K]
//    tile of A (2-8 KiB), so the ring holds ~200 KiB of B in flight;
//  * split-K inside a thread-block cluster: the S CTAs of a cluster own the
//    same TN columns and S consecutive K ranges.  CTA r owns columns
//    [r*TN/S, (r+1)*TN/S) of the block.  After a cluster barrier (every
//    accumulator complete), each CTA stores its fp32 accumulator values
//    straight from TMEM into the owner's idle pipeline buffers through
//    distributed shared memory (posted stores, one slot per sender); after a
//    second barrier each owner sums its S slots in rank order
//    (deterministic) from its own shared memory and stores C.  No workspace,
//    no atomics, no second pass over global memory, no remote loads;
//  * the finished block is staged as fp16 and written by TMA stores when C
//    is TMA-addressable.  A cluster of one stages straight from TMEM, with no
//    cluster barrier, through code that its epilogue warps run once "dry"
//    during the mainloop (skinny_stage_c).
//
// Roles as in gemm_sm100_kernel.cuh: warp 0 TMA producer, warp 1 TMEM owner
// and MMA issuer, warps 2..5 read the accumulator.  Every mbarrier wait is
// bounded; on the cluster path both cluster barriers are reached by every
// thread on every path, the abort path included.
#pragma once
#include <atomic>
#include <cuda_runtime.h>

#include "gemm_sm100_kernel.cuh"

namespace idb {

constexpr int kSkinnyN = 128;  // columns of C per MMA: the 128 TMEM lanes

// TN = columns of C per cluster: one, two or four MMAs of M = 128 per K step
// (128, 256 or 512 columns); a wider block reads more contiguous bytes of
// every row of B per stage (256 B, 512 B, 1 KiB).
template <int TM, int TN, int STAGES>
struct SkinnyPlan {
  static constexpr int kNB = TN / kSkinnyN;           // MMAs (accumulators) per K step
  static constexpr int kNBytes = kBK * TN * 2;        // B tile: 16 or 32 KiB
  static constexpr int kMBytes = TM * kBK * 2;        // A tile: TM rows of 128 B
  static constexpr int kStageBytes = kNBytes + kMBytes;
  static constexpr int kOffN = 0;
  static constexpr int kOffM = STAGES * kNBytes;
  static constexpr int kOffBar = kOffM + STAGES * kMBytes;
  static constexpr int kNumBars = 2 * STAGES + 1;  // full, empty, tmem_full
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kUsed = kOffMisc + 16;
  static constexpr int kDynamicBytes = kUsed + 1024;
  static constexpr uint32_t kTmemCols =
      kNB * TM <= 32 ? 32 : (kNB * TM <= 64 ? 64 : (kNB * TM <= 128 ? 128 : 256));
  static constexpr int kPartialBytes = TM * TN * 4;  // receive buffer fp32 [S][TM][TN / S]
  static_assert(TM == 16 || TM == 32 || TM == 64, "MMA N of the swapped tile");
  static_assert(TN == 128 || TN == 256 || TN == 512, "one, two or four 128-row MMAs");
  static_assert(kMBytes % 1024 == 0, "swizzled A tiles need 1024-byte alignment");
  static_assert(kPartialBytes <= kOffBar, "the receive buffer reuses the pipeline buffers");
  // fp16 staging of the finished C block for its TMA store: [TM][TN] at
  // offset 0 for a cluster of one; [TM][TN / S] after the receive buffer
  // otherwise (S >= 2)
  static constexpr int kStageCOff = kPartialBytes;
  static_assert(TM * TN * 2 <= kOffBar, "C staging of a cluster of one reuses the pipeline buffers");
  static_assert(kStageCOff + TM * (TN / 2) * 2 <= kOffBar, "C staging after the receive buffer");
};

// Width of one TMA store box of C (columns): a block of `ns` columns is
// stored as ns / box boxes of [TM rows x box columns], staged one after the
// other, each row-major.  The tensor map's box is [min(ns, 256) x TM].
__host__ __device__ constexpr int skinny_c_box(int ns) { return ns < 256 ? ns : 256; }

// Copies a cluster-of-one accumulator to the fp16 staging tile of its TMA
// store ([TM][TN] in boxes of skinny_c_box(TN) columns, each row-major),
// applying the fused epilogue when `epi`.  One thread's TMEM lane holds
// column n_local of every 128-column MMA block.
//
// Not inlined, so that both calls run the same instructions.  The epilogue
// warps first call it "dry" while the mainloop runs: keep = 0 sends every
// store to a 2-byte sink and no TMEM is read.  That brings this code into
// the instruction cache.  Fetched cold at the very end of a launch, while
// the memory system is still saturated, the unrolled copy of 64 rows took
// ~3 us.  The second call (keep = ~0) stages the real values.  Both calls
// take run-time arguments, so the compiler has no constant to specialise a
// copy of the function on.
template <int TM, int TN>
__device__ __noinline__ void skinny_stage_c(uint32_t taddr, int n_local, uint32_t dst, uint32_t keep, int m0,
                                            int n0, int M, int N, int epi, int act, float alpha, float beta,
                                            const __half* D, long long ldd, const __half* bias) {
  constexpr int kNB = TN / kSkinnyN;
  constexpr int kBox = skinny_c_box(TN);
#pragma unroll
  for (int c32 = 0; c32 < (kNB * TM + 31) / 32; ++c32) {
    uint32_t v[32];
    if (keep) {
      tmem_ld_32x32b_x32(taddr + c32 * 32, v);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0u;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int col = c32 * 32 + i;
      if (col < kNB * TM) {
        // accumulator h holds TMEM columns [h*TM, (h+1)*TM): row m of C for
        // column h*128 + n_local of the block
        const int h = col / TM, m = col - h * TM;
        const int bcol = h * kSkinnyN + n_local;
        float x = __uint_as_float(v[i]);
        if (epi) {
          const int gm = m0 + m, gn = n0 + bcol;
          float d = 0.0f, b = 0.0f;
          if (gm < M && gn < N) {
            if (beta != 0.0f) d = __half2float(D[static_cast<long long>(gm) * ldd + gn]);
            if (bias != nullptr) b = __half2float(bias[gn]);
          }
          float y = alpha * x;
          if (beta != 0.0f) y = fmaf(beta, d, y);
          x = apply_act(y + b, act);
        }
        const uint32_t off = static_cast<uint32_t>(((bcol / kBox) * (TM * kBox) + m * kBox + bcol % kBox) * 2);
        st_shared_u16(dst + (off & keep), __half_as_ushort(__float2half_rn(x)));
      }
    }
  }
}

template <int TM, int TN, int STAGES>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_skinny_f16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using Plan = SkinnyPlan<TM, TN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sN = smem + Plan::kOffN;
  uint8_t* sM = smem + Plan::kOffM;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Plan::kOffBar);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Plan::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* recv = reinterpret_cast<float*>(smem);  // after the mainloop: fp32 [S][TM][TN / S]

  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int S = static_cast<int>(cluster_nctarank());
  const int rank = static_cast<int>(cluster_ctarank());
  const int cid = static_cast<int>(cluster_id_x());
  const int n0 = (cid % p.tiles_n) * TN;
  const int m0 = (cid / p.tiles_n) * TM;
  const int kb0 = static_cast<int>(static_cast<long long>(rank) * p.kb_total / S);
  const int kb1 = static_cast<int>(static_cast<long long>(rank + 1) * p.kb_total / S);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.c_tma) prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc<1>(tmem_slot, Plan::kTmemCols);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // global memory only after the previous grid in the stream has completed
  bool acc_ok = true;  // epilogue warps: the accumulator barrier completed in time
  // producer: ring position after its last load, for the drain at the end
  int drain_stage = 0, drain_issued = 0;
  uint32_t drain_phase = 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (issued >= STAGES && !mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int k0 = kb * kBK;
        uint8_t* n_dst = sN + stage * Plan::kNBytes;
        mbar_arrive_expect_tx(&full_bar[stage], Plan::kStageBytes);
#pragma unroll
        for (int h = 0; h < Plan::kNB; ++h) {
          uint8_t* dst = n_dst + h * (kBK * kSkinnyN * 2);
          const int n = n0 + h * kSkinnyN;
          if (p.b_kmaj) {
            // B stored N x K: one [128 n x 64 K] box per MMA, K-major rows
            tma_load_2d(dst, &tmB, &full_bar[stage], k0, n);
          } else {
            // B stored K x N: two [64 K x 64 n] atoms per MMA, n-major
            tma_load_2d(dst, &tmB, &full_bar[stage], n, k0);
            tma_load_2d(dst + kBK * 128, &tmB, &full_bar[stage], n + 64, k0);
          }
        }
        tma_load_2d(sM + stage * Plan::kMBytes, &tmA, &full_bar[stage], k0, m0);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      griddep_launch_dependents();  // every load of this CTA is issued
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, kDevErrTimeoutProducer);
      }
      // The last fills are drained only after an abort, at the very end of
      // the kernel.  In a normal run the MMA thread waited for every fill
      // issued here before its MMAs retired and the accumulator completed, so
      // none is in flight once the buffers are reused.  After an abort the
      // drain keeps the CTA, and its shared memory, alive until every fill
      // has landed.  Draining here, every time, put this thread last at the
      // first barrier after the mainloop: it saw the final fill ~0.8 us after
      // the MMA thread had consumed it.
      drain_stage = stage;
      drain_phase = phase;
      drain_issued = issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // A operand = the B tile (128 n rows), B operand = the A tile (TM rows, K-major)
      const uint32_t idesc = idesc_f16_f32(kSkinnyN, TM, p.b_kmaj == 0, false);
      const uint32_t n_lbo = p.b_kmaj ? 16 : kBK * 128, n_kstep = p.b_kmaj ? kUmmaK * 2 : kUmmaK * 128;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t nb = smem_u32(sN + stage * Plan::kNBytes);
        const uint32_t mb = smem_u32(sM + stage * Plan::kMBytes);
#pragma unroll
        for (int j = 0; j < kBK / kUmmaK; ++j) {
#pragma unroll
          for (int h = 0; h < Plan::kNB; ++h) {
            mma_f16_ss<1>(tmem_base + static_cast<uint32_t>(h * TM),
                          smem_desc_sw128(nb + h * (kBK * kSkinnyN * 2) + j * n_kstep, n_lbo, 1024),
                          smem_desc_sw128(mb + j * (kUmmaK * 2), 16, 1024), idesc, (kb > kb0 || j > 0) ? 1u : 0u);
          }
        }
        mma_commit<1>(&empty_bar[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, kDevErrTimeoutMma);
      }
      // tfull completes when every MMA above has retired (also what makes
      // the pipeline buffers free to receive partial tiles and TMEM safe to free)
      mma_commit<1>(tfull_bar);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(tfull_bar, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kDevErrTimeoutTeardown);
          break;
        }
      }
    }
  } else {
    if (S == 1 && p.c_tma) {
      // dry staging pass while the mainloop runs (see skinny_stage_c);
      // p.M < 0 never holds, it only keeps the arguments run-time values
      const uint32_t sink = smem_u32(smem + Plan::kOffMisc + 8);
      const bool never = p.M < 0;
      skinny_stage_c<TM, TN>(tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16), (warp & 3) * 32 + lane,
                             sink, never ? ~0u : 0u, m0, n0, p.M, p.N, never ? p.epi : 0, p.act, p.alpha, p.beta,
                             p.D, p.ldd, p.bias);
    }
    // ------------------------------------------------------------ wait for the accumulator
    // One lane per warp polls the barrier through the whole mainloop; the
    // others wait at the shuffle instead of competing for issue slots with
    // the producer and MMA threads.
    bool got = true;
    if (lane == 0) got = mbar_wait(tfull_bar, 0, abort_flag);
    got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
    acc_ok = named_bar_and(1, 32 * kEpiWarps, got);
    if (!acc_ok && threadIdx.x == 64) {
      *abort_flag = 1;
      atomicOr(p.err, kDevErrTimeoutEpilogue);
    }
  }

  // Per-thread global stores issued at the very end of a launch are slow
  // (each waits behind the memory traffic of the CTAs still streaming), so
  // when C is TMA-addressable the finished block is staged in shared memory
  // as fp16 and written by one TMA store per box.
  if (S == 1 && p.c_tma) {
    // ------------------------------------------------------------ one CTA owns the block
    // No partial tiles to combine and no peer: the pipeline buffers are free
    // once this CTA's accumulator is complete (every fill was consumed by an
    // MMA that has retired), so the epilogue warps stage C there directly.
    constexpr int kBox = skinny_c_box(TN);
    __half* stage = reinterpret_cast<__half*>(smem);
    if (warp >= 2 && acc_ok) {
      skinny_stage_c<TM, TN>(tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16), (warp & 3) * 32 + lane,
                             smem_u32(stage), ~0u, m0, n0, p.M, p.N, p.epi, p.act, p.alpha, p.beta, p.D, p.ldd,
                             p.bias);
      fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncwarp();
    __syncthreads();  // staging complete; every tcgen05.ld has completed
    if (threadIdx.x == 64 && acc_ok) {
#pragma unroll
      for (int b = 0; b < TN / kBox; ++b) {
        // TMA clips the rows and columns past M and N; a box that starts
        // past the last column has nothing to write
        if (n0 + b * kBox < p.N) tma_store_2d(&tmC, stage + b * (TM * kBox), n0 + b * kBox, m0);
      }
      bulk_commit_group();
      bulk_wait_group_read<0>();  // shared memory stays valid until the TMA has read it
    }
  } else {
    // ------------------------------------------------------------ cluster reduction
    // Barrier 1: every CTA of the cluster has completed its accumulator (all
    // MMAs retired, so every fill they consumed has landed), so its buffers
    // may now receive partial tiles.
    tc_fence_before();
    __syncwarp();
    cluster_sync();
    tc_fence_after();
    const int ns = TN / S;  // columns of the block this CTA reduces and stores
    if (warp >= 2 && acc_ok) {
      // Push: each accumulator value goes straight from TMEM to the CTA that
      // owns its column, into slot `rank` of that CTA's receive buffer
      // fp32 [S][TM][ns].  The stores are posted (no round trip), and each
      // warp instruction writes 128 contiguous bytes.
      const int ew = warp & 3;
      const int n_local = ew * 32 + lane;
      const uint32_t base = smem_u32(recv);
  #pragma unroll
      for (int c32 = 0; c32 < (Plan::kNB * TM + 31) / 32; ++c32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + c32 * 32, v);
        tmem_ld_wait();
  #pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int col = c32 * 32 + i;
          if (col < Plan::kNB * TM) {
            // accumulator h holds TMEM columns [h*TM, (h+1)*TM): rows m of C
            // for column h*128 + n_local of the block
            const int h = col / TM, m = col - h * TM;
            const int bcol = h * kSkinnyN + n_local;
            const int owner = bcol / ns;
            const uint32_t off = static_cast<uint32_t>(((rank * TM + m) * ns + bcol - owner * ns) * 4);
            st_dsmem_f32(mapa_shared(base + off, static_cast<uint32_t>(owner)), __uint_as_float(v[i]));
          }
        }
      }
    }
    // Barrier 2: every partial has reached its owner (release/acquire at
    // cluster scope); from here each CTA reads only its own shared memory, so
    // no CTA waits for another one before leaving.
    tc_fence_before();
    __syncwarp();
    cluster_sync();
    {
      const int g_per_row = ns / 4;  // 4-column groups per row
      const int groups = TM * g_per_row;
      const bool vec = ((reinterpret_cast<uintptr_t>(p.C) | static_cast<uintptr_t>(p.ldc * 2)) & 7u) == 0;
      __half* stage_c = reinterpret_cast<__half*>(smem + Plan::kStageCOff);  // [TM][ns] when C takes TMA stores
      for (int g = static_cast<int>(threadIdx.x); g < groups; g += kNumThreads) {
        const int m = g / g_per_row;
        const int n = (g - m * g_per_row) * 4;
        const int gm = m0 + m, gn = n0 + rank * ns + n;
        if (gm >= p.M || gn >= p.N) continue;
        // sum the S slots in rank order: the same result whatever the timing
        float4 acc = *reinterpret_cast<const float4*>(recv + m * ns + n);
        for (int q = 1; q < S; ++q) {
          const float4 x = *reinterpret_cast<const float4*>(recv + (q * TM + m) * ns + n);
          acc.x += x.x;
          acc.y += x.y;
          acc.z += x.z;
          acc.w += x.w;
        }
        float* v = &acc.x;
        if (p.epi) {
          for (int c = 0; c < 4 && gn + c < p.N; ++c) {
            const float d = (p.beta != 0.0f) ? __half2float(p.D[static_cast<long long>(gm) * p.ldd + gn + c]) : 0.0f;
            const float b = (p.bias != nullptr) ? __half2float(p.bias[gn + c]) : 0.0f;
            v[c] = epilogue_value(p, v[c], d, b);
          }
        }
        if (p.c_tma) {
          uint2 hv;
          hv.x = pack_half2(v[0], v[1]);
          hv.y = pack_half2(v[2], v[3]);
          *reinterpret_cast<uint2*>(stage_c + m * ns + n) = hv;
          continue;
        }
        __half* dst = p.C + static_cast<long long>(gm) * p.ldc + gn;
        if (vec && gn + 3 < p.N) {
          uint2 hv;
          hv.x = pack_half2(v[0], v[1]);
          hv.y = pack_half2(v[2], v[3]);
          *reinterpret_cast<uint2*>(dst) = hv;
        } else {
          for (int c = 0; c < 4 && gn + c < p.N; ++c) dst[c] = __float2half_rn(v[c]);
        }
      }
      if (p.c_tma) {
        // one box of [TM rows x ns columns]; TMA clips the rows and columns
        // past M and N, and a box that starts past the last column is skipped
        fence_proxy_async_smem();
        __syncwarp();
        __syncthreads();
        if (threadIdx.x == 64 && n0 + rank * ns < p.N) {
          tma_store_2d(&tmC, stage_c, n0 + rank * ns, m0);
          bulk_commit_group();
          bulk_wait_group_read<0>();  // shared memory stays valid until the TMA has read it
        }
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, Plan::kTmemCols);
  }
  if (warp == 0 && lane == 0 && *abort_flag) {
    // after an abort: the last min(issued, STAGES) fills land before this CTA
    // exits (every role raises the flag before the barriers above, so the
    // producer reads its final value here)
    const int outstanding = drain_issued < STAGES ? drain_issued : STAGES;
    for (int i = 0; i < outstanding; ++i) {
      drain_stage = (drain_stage == 0) ? STAGES - 1 : drain_stage - 1;
      if (drain_stage == STAGES - 1) drain_phase ^= 1u;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full_bar[drain_stage], drain_phase)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kDevErrTimeoutTeardown);
          break;
        }
      }
    }
  }
}

template <int TM, int TN, int STAGES>
cudaError_t launch_skinny(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, const GemmParams& p,
                          int grid, int cluster, cudaStream_t stream) {
  using Plan = SkinnyPlan<TM, TN, STAGES>;
  auto kernel = gemm_skinny_f16<TM, TN, STAGES>;
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = Plan::kDynamicBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, a, b, c, p);
}

using SkinnyLaunchFn = cudaError_t (*)(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c,
                                       const GemmParams& p, int grid, int cluster, cudaStream_t stream);

}  // namespace idb

#define IDB_DEFINE_SKINNY(TM, TN, ST)                                                                     \
  cudaError_t launch_skinny_tm##TM##_tn##TN##_s##ST(const CUtensorMap& a, const CUtensorMap& b,            \
                                                    const CUtensorMap& c, const GemmParams& p, int grid,   \
                                                    int cluster, cudaStream_t stream) {                    \
    return launch_skinny<TM, TN, ST>(a, b, c, p, grid, cluster, stream);                                  \
  }
