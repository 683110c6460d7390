// FP16-in / FP32-accumulate / FP16-out GEMM  C[M,N] = A[M,K] * B[K,N]  for sm_100a.
//
// Replaces the reference's SIMT kernel `gemm_tiled_reg<TILE_M,TILE_N,TILE_K,TM,TN>`
// (src/gemm_kernels.cuh:6-83): same operand layout (all row-major, fp16 in,
// fp32 accumulate, fp16 out rounded to nearest as __float2half does, zero
// contribution from rows/columns outside M/N/K), built the Blackwell way:
//
//   warp 0      TMA producer: per pipeline stage one A tile [128 rows x 64 K]
//               and one B tile [64 K x BN/CG columns], 128B-swizzled, in
//               whichever major order the operand is stored (row-major A is
//               K-major, a stored-transposed A is M-major; row-major B is
//               N-major, a stored-transposed B is K-major), completing on a
//               `full` mbarrier.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (K=16 per instruction), frees smem stages with
//               tcgen05.commit -> `empty` mbarrier, hands finished accumulators
//               to the epilogue with tcgen05.commit -> `tmem_full`.
//   warps 2..5  epilogue: tcgen05.ld (32 lanes x 32 columns per warp), the
//               optional fused alpha / beta*D / bias / activation step in
//               fp32, fp16 conversion, 128B-swizzled smem staging, TMA store (or a
//               coalesced st.global path when C's row pitch is not 16-byte
//               aligned).  Split-K / stream-K partials go to an fp32
//               workspace; the last CTA of a tile (atomic ticket, no
//               spinning) sums the partials in K order and writes C.
//
// CG (CTA group) = 1: one CTA owns a 128 x BN tile (MMA M=128).
// CG = 2: a cluster of two CTAs owns a 256 x BN tile (tcgen05 cta_group::2,
// MMA M=256).  Each CTA loads its own 128 rows of A and its own BN/2 columns
// of B (no multicast); the even CTA issues the MMAs, which read both CTAs'
// shared memory and write each CTA's 128 accumulator rows into its own TMEM;
// commits are multicast to both CTAs' barriers.  Per CTA this halves the B
// bytes moved from L2 for the same MMA work.
//
// The kernel is persistent (grid <= #SMs, static round-robin over work units)
// and double-buffers the TMEM accumulator (2 x BN columns), so the epilogue of
// one tile overlaps the mainloop of the next.  Every mbarrier wait is bounded
// (see sm100_ptx.cuh); a timeout raises a CTA abort flag and an error bit in
// the library's device error word, and every role drains what it started
// before the CTA frees TMEM and exits.
#pragma once
#include "sm100_ptx.cuh"

namespace idb {

constexpr int kBM = 128;          // rows per CTA: one TMEM lane per row
constexpr int kBK = 64;           // K per pipeline stage: one 128-byte fp16 swizzle row
constexpr int kUmmaK = 16;        // K per tcgen05.mma.kind::f16
constexpr int kEpiWarps = 4;      // one warpgroup covers the 128 TMEM lanes
constexpr int kNumThreads = 64 + 32 * kEpiWarps;
constexpr int kStoreRows = 32;    // rows per epilogue store box (one warp's TMEM lanes)
constexpr int kStoreCols = 64;    // columns per epilogue store box (128 bytes)
constexpr int kCounterSlots = 65536;  // split-K tile tickets at the head of the workspace
constexpr int kMaxPeers = 7;          // peer copies of C (fused all-gather over 8 GPUs)

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n;   // tiles of (128 * CG) x BN
  int num_tiles;
  int split_k;    // >= 1, <= kb_total (1 when CG = 2); 1 in stream-K mode
  int kb_total;   // ceil(K / kBK)
  int streamk;    // 1: stream-K: tiles [0, dp_tiles) data-parallel, the rest split evenly by iterations
  int dp_tiles;   // stream-K: whole tiles walked data-parallel before the stream-K region
  int max_parts;  // partial slots per tile in the workspace (split_k, or the most stream-K pieces of any tile)
  long long total_iters;  // stream-K: (num_tiles - dp_tiles) * kb_total iterations of the stream-K region
  int sk_workers; // stream-K: workers [0, sk_workers) share the stream-K region (<= the grid's workers)
  int raster;     // 0: groups of `group` tile-rows, M fastest; 1: groups of tile-columns, N fastest
  int group;      // >= 1
  int c_tma;      // 1: TMA-store epilogue; 0: coalesced st.global epilogue (any pitch)
  __half* C;
  long long ldc;
  float* partials;          // fp32 partial tiles (tile, part, 128 x BN) of split-K / stream-K
  unsigned int* counters;   // split-K tickets, zero on entry and on exit
  int* err;                 // device error word
  // Operand layouts.  a_mn = 1: A is stored K x M (the GEMM uses its
  // transpose), its tiles are loaded M-major; b_kmaj = 1: B is stored N x K,
  // its tiles are loaded K-major.  tcgen05 reads either major order from
  // shared memory, so no operand is ever transposed in memory.
  int a_mn, b_kmaj;
  // Fused epilogue (epi = 1):  C = act(alpha * acc + beta * D + bias[col]),
  // evaluated in fp32 and rounded once to fp16.  D is read only when
  // beta != 0 and may be C itself; bias (fp16[N]) may be null.
  // act: 0 none, 1 ReLU, 2 GELU (erf form).  epi = 0: C = fp16(acc).
  int epi, act;
  float alpha, beta;
  const __half* D;
  long long ldd;
  const __half* bias;
  // Fused all-gather: each finished box of C is also stored into the C of
  // every peer GPU (peer_C[i]: that GPU's copy at this rank's offset, same
  // pitch ldc), over NVLink, right after it is staged.  Non-split configs.
  // peer_tma = 1 (C TMA-addressable): the staged box goes to each peer by a
  // TMA store through peer_map[i] (peer_C[i] with C's extents, pitch and
  // box), issued next to the local store; the TMA unit moves the bytes and
  // the epilogue warp only waits for its staging buffer to be read.
  // peer_tma = 0: the warp copies the box with 16-byte stores.
  int n_peers;
  int peer_tma;
  __half* peer_C[kMaxPeers];
  CUtensorMap peer_map[kMaxPeers];
  // Multicast all-gather: mc_C is this rank's rows of C at an NVLink
  // multicast address (same pitch ldc) of a C that every rank holds.  Each
  // staged box is stored once, with multimem.st, and NVSwitch writes it into
  // every rank's copy, this rank's included; C itself is then not written
  // separately.  Non-split configs, N and ldc multiples of 8, c_tma = 0,
  // n_peers = 0.
  __half* mc_C;
};

template <int BN, int STAGES, int CG>
struct SmemPlan {
  static constexpr int kBNc = BN / CG;                          // B columns held by this CTA
  static constexpr int kABytes = kBM * kBK * 2;                 // 16 KiB
  static constexpr int kBBytes = kBK * kBNc * 2;                // kBNc x 128 B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kCBufBytes = kStoreRows * kStoreCols * 2;  // 4 KiB
  static constexpr int kCBytes = kEpiWarps * 2 * kCBufBytes;      // double-buffered per warp
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + STAGES * kABytes;
  static constexpr int kOffC = kOffB + STAGES * kBBytes;
  static constexpr int kOffBar = kOffC + kCBytes;
  static constexpr int kNumBars = 2 * STAGES + 4 + 1;           // full, empty, tmem_full[2], tmem_empty[2], done
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kUsed = kOffMisc + 16;
  static constexpr int kDynamicBytes = kUsed + 1024;            // slack for 1024-byte alignment
  // One tcgen05.mma covers at most 256 columns; a 512-column pair tile is two
  // MMAs per K step, and each CTA holds its half of both MMAs' B columns.
  static constexpr int kMmaN = BN < 256 ? BN : 256;   // columns per MMA
  static constexpr int kNumMma = BN / kMmaN;          // MMAs per K step
  static constexpr int kMmaNc = kMmaN / CG;           // B columns per MMA held by this CTA
  // Accumulators in TMEM: two (the epilogue of one unit overlaps the next
  // unit's mainloop) when 2 * BN columns fit in the 512, else one.
  static constexpr int kNumAcc = (2 * BN <= 512) ? 2 : 1;
  static constexpr uint32_t kTmemCols = (kNumAcc * BN <= 32)    ? 32
                                        : (kNumAcc * BN <= 64)  ? 64
                                        : (kNumAcc * BN <= 128) ? 128
                                        : (kNumAcc * BN <= 256) ? 256
                                                                : 512;
  static_assert(CG == 1 || CG == 2, "CTA group of 1 or 2");
  static_assert(kBNc % 64 == 0 && kBNc >= 64 && kMmaNc % 64 == 0, "B columns per CTA and MMA: multiples of 64");
  static_assert(BN <= 256 || (CG == 2 && BN == 512), "a 512-column tile needs a CTA pair");
  static_assert(kNumAcc * BN <= 512, "TMEM holds 512 fp32 columns");
  static_assert(kOffB % 1024 == 0 && kOffC % 1024 == 0, "swizzled buffers need 1024-byte alignment");
};

// Tile index -> (tile row, tile column) in grouped raster order.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& tm, int& tn) {
  if (p.raster == 0) {
    const int per_group = p.group * p.tiles_n;
    const int g = t / per_group;
    const int first = g * p.group;
    const int gs = min(p.tiles_m - first, p.group);
    const int r = t - g * per_group;
    tm = first + r % gs;
    tn = r / gs;
  } else {
    const int per_group = p.group * p.tiles_m;
    const int g = t / per_group;
    const int first = g * p.group;
    const int gs = min(p.tiles_n - first, p.group);
    const int r = t - g * per_group;
    tn = first + r % gs;
    tm = r / gs;
  }
}

// One piece of work: tile (tm, tn), K blocks [kb0, kb1), and which of the
// tile's `nparts` K pieces it is (nparts = 1: the whole K range, written
// straight to C; otherwise a partial tile reduced by the last arriving CTA).
struct Unit {
  int tile, tm, tn, kb0, kb1, part, nparts;
  bool down;  // walk K from the end
};

// This worker's position in its list of units.
//  * data-parallel / split-K: units u = worker, worker + workers, ...;
//    u -> (tile u / split_k, K slice u % split_k).  The persistent workers
//    advance through their units in lock-step waves, and every other wave
//    walks K from the end (serpentine order): consecutive waves share operand
//    blocks, and the K slices a wave touched last are the ones still in L2.
//  * stream-K (hybrid): the first dp_tiles tiles are walked data-parallel as
//    above, whole tiles in waves; the remaining tiles (a last wave at most
//    half full, or else the last one to two waves' worth) form the stream-K
//    region, whose T = (num_tiles - dp_tiles) * kb_total (tile, K-block)
//    iterations are split evenly over the first W' = sk_workers workers,
//    worker w owning [w*T/W', (w+1)*T/W') cut at tile boundaries.  A half
//    empty last wave of R tiles takes W' = 2R: every tile in two K halves.
//    No SM idles in a partial last wave, and the concurrent tiles stay
//    neighbours in the raster order (an all-stream-K walk spreads the
//    workers over the whole tile range at once and loses L2 reuse).
struct WorkIter {
  long long cur, end;  // stream-K region / data-parallel unit index and limit
  int dp;              // stream-K mode: next data-parallel tile of this worker
  int count;
};

__device__ __forceinline__ WorkIter work_begin(const GemmParams& p, int worker, int workers) {
  WorkIter w;
  if (p.streamk) {
    const long long base = static_cast<long long>(p.dp_tiles) * p.kb_total;
    w.dp = worker;
    const int sw = p.sk_workers;
    w.cur = worker < sw ? base + static_cast<long long>(worker) * p.total_iters / sw : base;
    w.end = worker < sw ? base + static_cast<long long>(worker + 1) * p.total_iters / sw : base;
  } else {
    w.dp = 0;
    w.cur = worker;
    w.end = static_cast<long long>(p.num_tiles) * p.split_k;
  }
  w.count = 0;
  return w;
}

// Worker that owns iteration x of the stream-K region (x counted from the
// region's start).
__device__ __forceinline__ int sk_owner(const GemmParams& p, long long x) {
  return static_cast<int>(((x + 1) * p.sk_workers - 1) / p.total_iters);
}

__device__ __forceinline__ bool work_next(const GemmParams& p, int worker, int workers, WorkIter& it, Unit& w) {
  const int kbt = p.kb_total;
  if (p.streamk && it.dp < p.dp_tiles) {
    // data-parallel part of a stream-K walk: one whole tile per unit
    w.tile = it.dp;
    w.kb0 = 0;
    w.kb1 = kbt;
    w.part = 0;
    w.nparts = 1;
    w.down = (it.count & 1) != 0;
    it.dp += workers;
  } else if (it.cur >= it.end) {
    return false;
  } else if (p.streamk) {
    w.tile = static_cast<int>(it.cur / kbt);
    w.kb0 = static_cast<int>(it.cur - static_cast<long long>(w.tile) * kbt);
    const long long left = it.end - it.cur;
    w.kb1 = (left < kbt - w.kb0) ? w.kb0 + static_cast<int>(left) : kbt;
    it.cur += w.kb1 - w.kb0;
    const long long t0 = static_cast<long long>(w.tile - p.dp_tiles) * kbt;
    const int first = sk_owner(p, t0);
    w.part = worker - first;
    w.nparts = sk_owner(p, t0 + kbt - 1) - first + 1;
    w.down = false;
  } else {
    const int u = static_cast<int>(it.cur);
    w.tile = u / p.split_k;
    w.part = u - w.tile * p.split_k;
    w.nparts = p.split_k;
    // part * kb_total < 16 * 2^25 fits 32 bits (K < 2^31, split_k <= 16)
    w.kb0 = static_cast<int>(static_cast<unsigned>(w.part * kbt) / static_cast<unsigned>(p.split_k));
    w.kb1 = static_cast<int>(static_cast<unsigned>((w.part + 1) * kbt) / static_cast<unsigned>(p.split_k));
    w.down = (it.count & 1) != 0;
    it.cur += workers;
  }
  tile_coords(p, w.tile, w.tm, w.tn);
  ++it.count;
  return true;
}

__device__ __forceinline__ float apply_act(float x, int act) {
  if (act == 1) return fmaxf(x, 0.0f);
  if (act == 2) return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));  // x * Phi(x)
  return x;
}

// One element of the fused epilogue; d and b are the D and bias values.
__device__ __forceinline__ float epilogue_value(const GemmParams& p, float acc, float d, float b) {
  float v = p.alpha * acc;
  if (p.beta != 0.0f) v = fmaf(p.beta, d, v);
  return apply_act(v + b, p.act);
}

// 64 consecutive fp16 values src[0..63] as 8 x 16 bytes; positions at or
// past `valid` read as 0.  `vec`: src is 16-byte aligned.  Plain (coherent)
// loads, because D may be the C that this kernel writes.
__device__ __forceinline__ void load_chunk64(const __half* src, int valid, bool vec, uint4 (&out)[8]) {
  if (vec && valid >= 64) {
#pragma unroll
    for (int q = 0; q < 8; ++q) out[q] = __ldcg(reinterpret_cast<const uint4*>(src) + q);
  } else {
    const unsigned short* s = reinterpret_cast<const unsigned short*>(src);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      unsigned short h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = (8 * q + e < valid) ? s[8 * q + e] : static_cast<unsigned short>(0);
      out[q] = make_uint4(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16),
                          h[4] | (static_cast<uint32_t>(h[5]) << 16), h[6] | (static_cast<uint32_t>(h[7]) << 16));
    }
  }
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __low2float(*reinterpret_cast<const __half2*>(&w)); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __high2float(*reinterpret_cast<const __half2*>(&w)); }

// Applies the fused epilogue to the 64 values of one row chunk (columns
// col0 .. col0 + 63 of C); dv holds the row's D values (unused when beta = 0).
__device__ __forceinline__ void apply_epilogue64(const GemmParams& p, float (&f)[64], const uint4 (&dv)[8], int col0) {
  uint4 bv[8];
  if (p.bias != nullptr) {
    const bool vec = (reinterpret_cast<uintptr_t>(p.bias) & 15u) == 0;
    load_chunk64(p.bias + col0, p.N - col0, vec, bv);
  } else {
#pragma unroll
    for (int q = 0; q < 8; ++q) bv[q] = make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t dw[4] = {dv[q].x, dv[q].y, dv[q].z, dv[q].w};
    const uint32_t bw[4] = {bv[q].x, bv[q].y, bv[q].z, bv[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[8 * q + 2 * e] = epilogue_value(p, f[8 * q + 2 * e], half_lo(dw[e]), half_lo(bw[e]));
      f[8 * q + 2 * e + 1] = epilogue_value(p, f[8 * q + 2 * e + 1], half_hi(dw[e]), half_hi(bw[e]));
    }
  }
}

// Loads D[row0 .. row0+31][col0 .. col0+63] (one epilogue warp's box) with
// coalesced 16-byte reads: in step i lane l reads row 4i + l/8, segment l%8,
// so each instruction covers four whole 128-byte rows.  Out-of-range
// elements read 0.  The box is handed to the owning threads through shared
// memory (transpose_d_box).
__device__ __forceinline__ void load_d_box(const GemmParams& p, int row0, int col0, int lane, uint4 (&draw)[8]) {
  const int seg = lane & 7;
  const int c = col0 + seg * 8;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.D) | static_cast<uintptr_t>(p.ldd * 2)) & 15u) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = row0 + 4 * i + (lane >> 3);
    draw[i] = make_uint4(0u, 0u, 0u, 0u);
    if (r >= p.M || c >= p.N) continue;
    const __half* src = p.D + static_cast<long long>(r) * p.ldd + c;
    if (vec && c + 8 <= p.N) {
      draw[i] = __ldcg(reinterpret_cast<const uint4*>(src));
    } else {
      const unsigned short* s = reinterpret_cast<const unsigned short*>(src);
      unsigned short h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = (c + e < p.N) ? s[e] : static_cast<unsigned short>(0);
      draw[i] = make_uint4(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16),
                           h[4] | (static_cast<uint32_t>(h[5]) << 16), h[6] | (static_cast<uint32_t>(h[7]) << 16));
    }
  }
}

// Writes a box loaded by load_d_box into a [32 x 128 B] staging buffer (the
// 128-byte swizzle of the C staging layout, conflict-free both ways) and
// returns this lane's own row in dv.  The buffer must be free; the caller
// overwrites only its own row afterwards, so no further sync is needed.
__device__ __forceinline__ void transpose_d_box(uint8_t* buf, int lane, const uint4 (&draw)[8], uint4 (&dv)[8]) {
  const int seg = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    *reinterpret_cast<uint4*>(buf + r * 128 + ((seg ^ (r & 7)) << 4)) = draw[i];
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 8; ++q) dv[q] = *reinterpret_cast<const uint4*>(buf + lane * 128 + ((q ^ (lane & 7)) << 4));
}

// Reduction of a split tile by the 128 epilogue threads of the CTA that
// brought its last K piece: C[row0 + r][col0 + c] = sum over parts (in K
// order) of the fp32 partial slots, for the tile's valid rows/columns.  The
// work is spread over (row, 4-column group) pairs, rows fastest so that
// partial reads coalesce, with the loads of two parts x 8 elements in flight
// per thread.  The sum order is fixed, so the result does not depend on which
// CTA finishes last.
template <int BN>
__device__ __forceinline__ void reduce_partials(const GemmParams& p, const float* slots, int nparts, int row0,
                                                int col0, int et) {
  const int R = min(kBM, p.M - row0);
  const int cols = min(BN, p.N - col0);
  const int C4 = (cols + 3) >> 2;
  const int E = R * C4;
  const bool vec = (((reinterpret_cast<uintptr_t>(p.C) | static_cast<uintptr_t>(p.ldc * 2)) & 7u) == 0);
  constexpr int kB = 8;
  for (int e0 = et; e0 < E; e0 += kEpiWarps * 32 * kB) {
    float4 acc[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) acc[b] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < nparts; s += 2) {
      const float4* sa = reinterpret_cast<const float4*>(slots + static_cast<size_t>(s) * (kBM * BN));
      const float4* sb = reinterpret_cast<const float4*>(slots + static_cast<size_t>(s + 1) * (kBM * BN));
      const bool two = (s + 1 < nparts);
      float4 xa[kB], xb[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int e = e0 + b * kEpiWarps * 32;
        xa[b] = make_float4(0.f, 0.f, 0.f, 0.f);
        xb[b] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < E) {
          const int r = e % R, j4 = e / R;
          xa[b] = __ldcg(&sa[j4 * kBM + r]);
          if (two) xb[b] = __ldcg(&sb[j4 * kBM + r]);
        }
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        acc[b].x += xa[b].x; acc[b].y += xa[b].y; acc[b].z += xa[b].z; acc[b].w += xa[b].w;
        if (two) {
          acc[b].x += xb[b].x; acc[b].y += xb[b].y; acc[b].z += xb[b].z; acc[b].w += xb[b].w;
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int e = e0 + b * kEpiWarps * 32;
      if (e >= E) continue;
      const int r = e % R, j4 = e / R;
      const int gc = col0 + 4 * j4;
      if (p.epi) {
        float* v = &acc[b].x;
        for (int c = 0; c < 4 && gc + c < p.N; ++c) {
          const float d = (p.beta != 0.0f) ? __half2float(p.D[static_cast<long long>(row0 + r) * p.ldd + gc + c]) : 0.0f;
          const float bb = (p.bias != nullptr) ? __half2float(p.bias[gc + c]) : 0.0f;
          v[c] = epilogue_value(p, v[c], d, bb);
        }
      }
      __half* dst = p.C + static_cast<long long>(row0 + r) * p.ldc + gc;
      if (vec && gc + 3 < p.N) {
        uint2 hv;
        hv.x = pack_half2(acc[b].x, acc[b].y);
        hv.y = pack_half2(acc[b].z, acc[b].w);
        *reinterpret_cast<uint2*>(dst) = hv;
      } else {
        const float vals[4] = {acc[b].x, acc[b].y, acc[b].z, acc[b].w};
        for (int c = 0; c < 4 && gc + c < p.N; ++c) dst[c] = __float2half_rn(vals[c]);
      }
    }
  }
}

// Copies one staged [32 x 64] box (128-byte swizzled, as stage_row_sw128
// left it) to the same place in every peer's C: in step i lane l moves the
// 16 bytes of row 4i + l/8, segment l%8, so each store instruction writes
// four whole 128-byte rows of every peer.
__device__ __forceinline__ void copy_box_to_peers(const GemmParams& p, const uint8_t* buf, int row0, int col0,
                                                  int lane) {
  const int seg = lane & 7;
  const int c = col0 + seg * 8;
  const bool vec = (static_cast<uintptr_t>(p.ldc * 2) & 15u) == 0;
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const int gr = row0 + r;
    if (gr >= p.M || c >= p.N) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 128 + ((seg ^ (r & 7)) << 4));
    const long long off = static_cast<long long>(gr) * p.ldc + c;
    for (int q = 0; q < p.n_peers; ++q) {
      __half* dst = p.peer_C[q] + off;
      if (vec && c + 8 <= p.N && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const __half* h = reinterpret_cast<const __half*>(&v);
        for (int e = 0; e < 8 && c + e < p.N; ++e) dst[e] = h[e];
      }
    }
  }
}

// Stores one staged [32 x 64] box through the multicast address of C (every
// rank's copy at once), with the same lane layout as copy_box_to_peers.  N
// is a multiple of 8, so a lane's 8-column segment is wholly inside or
// wholly outside C.
__device__ __forceinline__ void store_box_multicast(const GemmParams& p, const uint8_t* buf, int row0, int col0,
                                                    int lane) {
  const int seg = lane & 7;
  const int c = col0 + seg * 8;
  if (c >= p.N) return;
#pragma unroll 4
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const int gr = row0 + r;
    if (gr >= p.M) break;
    const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 128 + ((seg ^ (r & 7)) << 4));
    multimem_st_v4(p.mc_C + static_cast<long long>(gr) * p.ldc + c, v);
  }
}

// Column offset (relative to this CTA's first B column of MMA 0) of the j-th
// 64-column B atom this CTA holds: atoms are grouped per MMA.
template <class Plan>
__device__ __forceinline__ int b_atom_col(int j) {
  constexpr int kAtomsPerMma = Plan::kMmaNc / 64;
  return (j / kAtomsPerMma) * Plan::kMmaN + (j % kAtomsPerMma) * 64;
}

// Converts 64 fp32 values of one row to fp16 and writes them as row `lane`
// of a [32 x 64] fp16 staging box in the TMA 128-byte swizzle layout.
__device__ __forceinline__ void stage_row_sw128(uint8_t* buf, int lane, const float (&f)[64]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 w;
    w.x = pack_half2(f[8 * c + 0], f[8 * c + 1]);
    w.y = pack_half2(f[8 * c + 2], f[8 * c + 3]);
    w.z = pack_half2(f[8 * c + 4], f[8 * c + 5]);
    w.w = pack_half2(f[8 * c + 6], f[8 * c + 7]);
    const int phys = c ^ (lane & 7);
    *reinterpret_cast<uint4*>(buf + lane * 128 + phys * 16) = w;
  }
}

template <int BN, int STAGES, int CG>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_f16_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ GemmParams p) {
  using Plan = SmemPlan<BN, STAGES, CG>;
  constexpr int kBNc = Plan::kBNc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + Plan::kOffA;
  uint8_t* sB = smem + Plan::kOffB;
  uint8_t* sC = smem + Plan::kOffC;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Plan::kOffBar);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Plan::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;   // position in the CTA pair
  const bool leader = (rank == 0);
  const int cluster_id = static_cast<int>(blockIdx.x) / CG;
  const int num_clusters = static_cast<int>(gridDim.x) / CG;

  // Barriers are set up by the first epilogue thread, so that the producer
  // thread can work out its first unit meanwhile (below).
  if (threadIdx.x == 64) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar[0], 1);
    mbar_init(&tfull_bar[1], 1);
    // every epilogue warp of every CTA in the group releases the accumulator
    mbar_init(&tempty_bar[0], kEpiWarps * CG);
    mbar_init(&tempty_bar[1], kEpiWarps * CG);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  // The first work unit of the producer and MMA threads is computed while
  // the barriers and TMEM are being set up, so the first TMA load and the
  // first MMA follow the sync without delay.
  WorkIter first_wi = work_begin(p, cluster_id, num_clusters);
  Unit first_w;
  bool first_have = false;
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.c_tma) prefetch_tmap(&tmC);
    if (p.peer_tma) {
      for (int q = 0; q < p.n_peers; ++q) prefetch_tmap(&p.peer_map[q]);
    }
  }
  if (warp < 2 && lane == 0) first_have = work_next(p, cluster_id, num_clusters, first_wi, first_w);
  if (warp == 1) {
    __syncwarp();  // tcgen05.alloc is warp-wide (.sync.aligned)
    tmem_alloc<CG>(tmem_slot, Plan::kTmemCols);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();   // the peer's barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The set-up above touches no global memory, so it may overlap the tail of
  // the previous grid in the stream (programmatic dependent launch); every
  // global access below comes after that grid has completed.
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      WorkIter& wi = first_wi;
      Unit& w = first_w;
      for (bool have = first_have; ok && have; have = work_next(p, cluster_id, num_clusters, wi, w)) {
        const int arow = w.tm * (kBM * CG) + static_cast<int>(rank) * kBM;
        // this CTA's B columns: its share of every MMA's N range
        const int bcol = w.tn * BN + static_cast<int>(rank) * Plan::kMmaNc;
        for (int it = w.kb0; it < w.kb1; ++it) {
          const int kb = w.down ? w.kb1 - 1 - (it - w.kb0) : it;
          // the first STAGES fills go to slots that have never been used
          if (issued >= STAGES && !mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * Plan::kABytes;
          uint8_t* b_dst = sB + stage * Plan::kBBytes;
          // Tiles land in the canonical 128-byte-swizzled layouts: K-major A
          // is one [128 rows x 64 K] box; M-major A is two [64 K x 64 M]
          // atoms; B is kBNc/64 atoms of 64 columns, [64 K x 64 N] boxes when
          // N-major, [64 N x 64 K] boxes when K-major.  (x, y) = (inner, outer)
          // coordinates of the operand as stored.
          const int k0 = kb * kBK;
          if constexpr (CG == 1) {
            mbar_arrive_expect_tx(&full_bar[stage], Plan::kStageBytes);
            if (!p.a_mn) {
              tma_load_2d(a_dst, &tmA, &full_bar[stage], k0, arow);
            } else {
              tma_load_2d(a_dst, &tmA, &full_bar[stage], arow, k0);
              tma_load_2d(a_dst + kBK * 128, &tmA, &full_bar[stage], arow + 64, k0);
            }
#pragma unroll
            for (int j = 0; j < kBNc / 64; ++j) {
              const int n = bcol + b_atom_col<Plan>(j);
              tma_load_2d(b_dst + j * (kBK * 128), &tmB, &full_bar[stage], p.b_kmaj ? k0 : n, p.b_kmaj ? n : k0);
            }
          } else {
            // Both CTAs' bytes complete on the even CTA's `full` barrier.
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Plan::kStageBytes);
            const uint32_t bar = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (!p.a_mn) {
              tma_load_2d_pair(a_dst, &tmA, bar, k0, arow);
            } else {
              tma_load_2d_pair(a_dst, &tmA, bar, arow, k0);
              tma_load_2d_pair(a_dst + kBK * 128, &tmA, bar, arow + 64, k0);
            }
#pragma unroll
            for (int j = 0; j < kBNc / 64; ++j) {
              const int n = bcol + b_atom_col<Plan>(j);
              tma_load_2d_pair(b_dst + j * (kBK * 128), &tmB, bar, p.b_kmaj ? k0 : n, p.b_kmaj ? n : k0);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every load of this CTA is issued: the next grid may begin its set-up
      griddep_launch_dependents();
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, kDevErrTimeoutProducer);
      }
      // Drain: the last min(issued, STAGES) fills must have landed before the
      // CTA may exit (an in-flight TMA write into a retired CTA is undefined).
      // With a CTA pair the fills complete on the even CTA's barriers, which
      // only that CTA can poll; the odd CTA is covered by the cluster barrier
      // at teardown, which the even CTA reaches after consuming every fill.
      if (leader) {
        const int outstanding = issued < STAGES ? issued : STAGES;
        for (int i = 0; i < outstanding; ++i) {
          stage = (stage == 0) ? STAGES - 1 : stage - 1;
          if (stage == STAGES - 1) phase ^= 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[stage], phase)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              atomicOr(p.err, kDevErrTimeoutTeardown);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_f16_f32(kBM * CG, Plan::kMmaN, p.a_mn != 0, p.b_kmaj == 0);
      // Descriptor strides of the two major orders (128-byte swizzle):
      //  K-major:  rows of 128 B, 8-row groups 1024 B apart, a K step of 16
      //            elements advances 32 B inside the swizzled row;
      //  MN-major: 64-element atoms kBK*128 B apart (LBO), 8-row K groups
      //            1024 B apart (SBO), a K step advances 16 rows = 2 KiB.
      const uint32_t a_lbo = p.a_mn ? kBK * 128 : 16, a_kstep = p.a_mn ? kUmmaK * 128 : kUmmaK * 2;
      const uint32_t b_lbo = p.b_kmaj ? 16 : kBK * 128, b_kstep = p.b_kmaj ? kUmmaK * 2 : kUmmaK * 128;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      WorkIter& wi = first_wi;
      Unit& w = first_w;
      for (bool have = first_have; ok && have; have = work_next(p, cluster_id, num_clusters, wi, w)) {
        const int kb0 = w.kb0, kb1 = w.kb1;
        // the first kNumAcc units use accumulators that have never been used
        // A single accumulator made of two MMA halves (512-column tiles) is
        // released half by half by the epilogue (tempty_bar[0] / [1]); the
        // first K block of a unit runs on half 0 before waiting for half 1.
        constexpr bool kHalves = (Plan::kNumAcc == 1 && Plan::kNumMma == 2);
        const bool wait_acc = wi.count > Plan::kNumAcc;
        if (wait_acc && !mbar_wait(&tempty_bar[kHalves ? 0 : acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        // (the K order of this unit only matters to the producer; the MMA
        //  consumes stages in arrival order and starts a fresh accumulator
        //  on the unit's first stage)
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Plan::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * Plan::kBBytes);
          // MMA i reads this CTA's atoms [i*kMmaNc/64, (i+1)*kMmaNc/64) and
          // writes accumulator columns [i*kMmaN, (i+1)*kMmaN).
          auto issue = [&](int i, int j) {
            const uint64_t ad = smem_desc_sw128(a0 + j * a_kstep, a_lbo, 1024);
            const uint64_t bd =
                smem_desc_sw128(b0 + i * (Plan::kMmaNc / 64) * (kBK * 128) + j * b_kstep, b_lbo, 1024);
            mma_f16_ss<CG>(d_tmem + static_cast<uint32_t>(i * Plan::kMmaN), ad, bd, idesc,
                           (kb > kb0 || j > 0) ? 1u : 0u);
          };
          if (kHalves && kb == kb0) {
#pragma unroll
            for (int j = 0; j < kBK / kUmmaK; ++j) issue(0, j);
            if (wait_acc && !mbar_wait(&tempty_bar[1], acc_phase ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < kBK / kUmmaK; ++j) issue(1, j);
          } else {
#pragma unroll
            for (int j = 0; j < kBK / kUmmaK; ++j) {
#pragma unroll
              for (int i = 0; i < Plan::kNumMma; ++i) issue(i, j);
            }
          }
          mma_commit<CG>(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit<CG>(&tfull_bar[acc]);
        if (++acc == Plan::kNumAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, kDevErrTimeoutMma);
      }
      // Every MMA this thread issued must retire before TMEM is freed.
      mma_commit<CG>(done_bar);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(done_bar, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kDevErrTimeoutTeardown);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;               // TMEM lane quarter this warp may access
    const int row = ew * 32 + lane;        // row inside this CTA's 128 rows
    const bool ticket_thread = (threadIdx.x == 64);
    uint8_t* cbufs = sC + ew * 2 * Plan::kCBufBytes;
    // the accumulator is released on the even CTA's barrier
    const uint32_t tempty_remote0 = (CG == 2) ? mapa_shared(smem_u32(&tempty_bar[0]), 0) : 0u;
    // one accumulator in two MMA halves: released half by half (see MMA issuer)
    constexpr bool kHalvesEpi = (Plan::kNumAcc == 1 && Plan::kNumMma == 2);
    auto release_acc = [&](int b) {
      if constexpr (CG == 1) {
        mbar_arrive(&tempty_bar[b]);
      } else {
        mbar_arrive_cluster(tempty_remote0 + static_cast<uint32_t>(b * 8));
      }
    };
    int cb = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    WorkIter wi = work_begin(p, cluster_id, num_clusters);
    Unit w;
    while (work_next(p, cluster_id, num_clusters, wi, w)) {
      const int tm = w.tm, tn = w.tn;
      // D of the tile's first chunk is requested before the accumulator is
      // ready, so its latency hides under the mainloop.
      const bool use_d = p.epi && p.beta != 0.0f;
      uint4 draw[8];
      if (use_d) load_d_box(p, tm * (kBM * CG) + static_cast<int>(rank) * kBM + ew * 32, tn * BN, lane, draw);
      // One lane per warp waits for the accumulator (the others wait at the
      // shuffle); all four warps then take the same decision, so none is
      // left waiting at a later named barrier if another gave up.
      bool got = true;
      if (lane == 0) got = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag);
      got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
      ok = named_bar_and(1, 32 * kEpiWarps, got);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int cta_row0 = tm * (kBM * CG) + static_cast<int>(rank) * kBM;
      const int grow = cta_row0 + row;
      const bool row_ok = grow < p.M;
      const int tile = w.tile;
      // Split tiles (split-K / stream-K): 1-CTA tiles, and CTA-pair tiles
      // with two accumulators.  Each CTA of a pair owns the slots and ticket
      // of its own 128 rows (slot tile = tile * CG + rank).
      constexpr bool kSplitOK = (CG == 1) || (Plan::kNumAcc == 2);
      const bool partial = kSplitOK && (w.nparts > 1);
      const int slot_tile = tile * CG + static_cast<int>(rank);
      float* slots = nullptr;
      if (partial) {
        // 1. this CTA's K piece of the tile -> its partial slot (valid rows only)
        slots = p.partials + static_cast<size_t>(slot_tile) * p.max_parts * (kBM * BN);
        float4* mine = reinterpret_cast<float4*>(slots + static_cast<size_t>(w.part) * (kBM * BN));
#pragma unroll 1
        for (int c32 = 0; c32 < BN / 32; ++c32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + c32 * 32, v);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              mine[(c32 * 8 + q) * kBM + row] =
                  make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                              __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
            }
          }
        }
        // 2. ticket: the CTA that brings the tile's last piece reduces it
        __threadfence();
        named_bar_sync(1, 32 * kEpiWarps);
        if (ticket_thread) {
          const unsigned old = atomicAdd(&p.counters[slot_tile], 1u);
          *last_flag = (old == static_cast<unsigned>(w.nparts - 1)) ? 1 : 0;
        }
        named_bar_sync(1, 32 * kEpiWarps);
        const bool last = (*last_flag != 0);
        // Few valid rows (skinny M): all 128 threads reduce from the slots and
        // the accumulator is released at once.  Many rows: the per-row path
        // below keeps this CTA's piece in TMEM and stores through TMA.
        const bool coop = (p.M - cta_row0) <= 32;
        if (!last || coop) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
          if (last) {
            __threadfence();
            reduce_partials<BN>(p, slots, w.nparts, cta_row0, tn * BN, static_cast<int>(threadIdx.x) - 64);
            if (ticket_thread) p.counters[slot_tile] = 0u;  // ticket zero for the next launch
          }
          if (++acc == Plan::kNumAcc) {
            acc = 0;
            acc_phase ^= 1u;
          }
          continue;
        }
        __threadfence();
      }
      {
#pragma unroll 1
        for (int c64 = 0; c64 < BN / 64; ++c64) {
          const int col0 = tn * BN + c64 * 64;
          const int row0 = cta_row0 + ew * 32;
          // D of this chunk (the first was requested before the wait): issued
          // before the TMEM reads so that its latency overlaps them
          if (use_d && c64 > 0) load_d_box(p, row0, col0, lane, draw);
          float f[64];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tbase + c64 * 64 + h * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) f[h * 32 + i] = __uint_as_float(v[i]);
          }
          if (partial) {
            // Sum the pieces in K order (deterministic whichever CTA is last);
            // this CTA's own piece comes from TMEM.
            float s[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) s[i] = 0.0f;
            for (int s2 = 0; s2 < w.nparts; ++s2) {
              if (s2 == w.part) {
#pragma unroll
                for (int i = 0; i < 64; ++i) s[i] += f[i];
              } else if (row_ok) {
                const float4* src = reinterpret_cast<const float4*>(slots + static_cast<size_t>(s2) * (kBM * BN));
                float4 x[16];
#pragma unroll
                for (int q = 0; q < 16; ++q) x[q] = __ldcg(&src[(c64 * 16 + q) * kBM + row]);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  s[4 * q] += x[q].x;
                  s[4 * q + 1] += x[q].y;
                  s[4 * q + 2] += x[q].z;
                  s[4 * q + 3] += x[q].w;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 64; ++i) f[i] = s[i];
          }
          uint8_t* buf = cbufs + cb * Plan::kCBufBytes;
          if (p.c_tma) {
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
          }
          if (p.epi && col0 < p.N) {
            uint4 dv[8];
            if (use_d) {
              transpose_d_box(buf, lane, draw, dv);
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q) dv[q] = make_uint4(0u, 0u, 0u, 0u);
            }
            apply_epilogue64(p, f, dv, col0);
          }
          stage_row_sw128(buf, lane, f);
          if (p.c_tma) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              // A box that starts past the edge has nothing to write; skip it
              // but still close a (possibly empty) bulk group so that the
              // wait_group.read<1> accounting above stays per buffer.
              if (row0 < p.M && col0 < p.N) {
                tma_store_2d(&tmC, buf, col0, row0);
                if (p.peer_tma) {
                  for (int q = 0; q < p.n_peers; ++q) tma_store_2d(&p.peer_map[q], buf, col0, row0);
                }
              }
              bulk_commit_group();
            }
          } else if (p.mc_C) {
            __syncwarp();  // every lane's row is staged
            store_box_multicast(p, buf, row0, col0, lane);
            __syncwarp();
          } else {
            __syncwarp();
            for (int r = 0; r < kStoreRows; ++r) {
              const int gr = row0 + r;
              if (gr >= p.M) break;
              __half* crow = p.C + static_cast<long long>(gr) * p.ldc;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int col = h * 32 + lane;
                const int gc = col0 + col;
                if (gc < p.N) {
                  const uint8_t* src = buf + r * 128 + (((col >> 3) ^ (r & 7)) << 4) + (col & 7) * 2;
                  crow[gc] = *reinterpret_cast<const __half*>(src);
                }
              }
            }
            __syncwarp();
          }
          if (p.n_peers > 0 && !p.peer_tma) {
            __syncwarp();  // every lane's row is staged
            copy_box_to_peers(p, buf, row0, col0, lane);
            __syncwarp();
          }
          cb ^= 1;
          if (kHalvesEpi && c64 == (BN / 64) / 2 - 1) {
            // first MMA half read out: the next unit's MMAs may start on it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(0);
          }
        }
        if (partial && ticket_thread) p.counters[slot_tile] = 0u;  // ticket zero for the next launch
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release_acc(kHalvesEpi ? 1 : acc);
      if (++acc == Plan::kNumAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicOr(p.err, kDevErrTimeoutEpilogue);
    }
    // The staging smem must stay valid until the last TMA stores have read it;
    // their global writes complete with the grid.
    if (p.c_tma && lane == 0) {
      // With peers, wait for the stores themselves (not only their reads of
      // shared memory): every byte has reached its GPU before the fence below.
      if (p.n_peers > 0) {
        bulk_wait_group<0>();
      } else {
        bulk_wait_group_read<0>();
      }
    }
    // Peer and multicast stores are ordered before anything this thread does
    // later (the grid's completion, which the ranks then agree on through NCCL).
    if (p.n_peers > 0 || p.mc_C) {
      __syncwarp();
      __threadfence_system();
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  // A CTA of a pair may not leave while its peer can still touch its shared
  // memory (remote arrives, MMA operand reads) or TMEM.
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, Plan::kTmemCols);
  }
}

}  // namespace idb
