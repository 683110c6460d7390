// C ABI of the kernel bank (declared in include/gemm_sm100.h).
//
// Host side of the path the reference implements in src/gemm_ext.cpp:22-132
// (validation, allocation, stream selection, config lookup) and
// src/gemm_cuda.cu:5-15 (dispatch).  Differences, all deliberate:
//  * the caller owns C and the workspace (no allocation in here);
//  * a configuration is found by table lookup, and a miss is an error;
//  * TMA descriptors are built per call from plain pointers and pitches;
//  * operands whose base or pitch TMA cannot address are first repacked into
//    the workspace by a copy kernel (pack_rows_f16).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/gemm_sm100.h"
#include "gemm_bank_common.cuh"
#include "gemm_skinny_kernel.cuh"
#include "generated/gemm_cfg_menu.inc"

namespace idb {

#define IDB_VARIANT(BN, ST, CG)                                                                           \
  cudaError_t launch_bn##BN##_s##ST##_cg##CG(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, \
                                             const GemmParams& p, int grid, cudaStream_t stream);
#include "generated/gemm_variants.inc"
#undef IDB_VARIANT

struct Variant {
  int bn;
  int stages;
  int cg;
  LaunchFn fn;
};

static const Variant kVariants[] = {
#define IDB_VARIANT(BN, ST, CG) {BN, ST, CG, &launch_bn##BN##_s##ST##_cg##CG},
#include "generated/gemm_variants.inc"
#undef IDB_VARIANT
};

#define IDB_SKINNY(TM, TN, ST)                                                                           \
  cudaError_t launch_skinny_tm##TM##_tn##TN##_s##ST(const CUtensorMap& a, const CUtensorMap& b,           \
                                                    const CUtensorMap& c, const GemmParams& p, int grid,  \
                                                    int cluster, cudaStream_t stream);
#include "generated/gemm_skinny_variants.inc"
#undef IDB_SKINNY

struct SkinnyVariant {
  int tm;
  int tn;
  int stages;
  SkinnyLaunchFn fn;
};

static const SkinnyVariant kSkinnyVariants[] = {
#define IDB_SKINNY(TM, TN, ST) {TM, TN, ST, &launch_skinny_tm##TM##_tn##TN##_s##ST},
#include "generated/gemm_skinny_variants.inc"
#undef IDB_SKINNY
};

// Copies a row-major fp16 matrix into a buffer whose row pitch is a multiple
// of 64 elements (128 bytes) so that TMA can address it.  Used only when a
// caller's A or B pitch / base address is not 16-byte aligned.
//
// One thread writes one 16-byte chunk (8 elements) of the packed copy.  Its
// source starts at a 2-byte aligned address, so it reads the one or two
// aligned 16-byte chunks that cover it with vector loads and shifts the bytes
// into place in registers (2-, 4- and 8-byte steps); neighbouring threads
// read the same chunks, which the cache serves.  A chunk that would reach
// outside the matrix's first and last bytes (its first or last 16 bytes, or
// a row's ragged end) is read element by element instead, so no load leaves
// the caller's memory.  Elements past `cols` in the last chunk of a row are
// written as zero (the tensor map's extent excludes them anyway).
__device__ __forceinline__ uint4 shift_chunks(uint4 c0, uint4 c1, int o) {
  uint32_t w0 = c0.x, w1 = c0.y, w2 = c0.z, w3 = c0.w, w4 = c1.x, w5 = c1.y, w6 = c1.z, w7 = c1.w;
  if (o & 8) {
    w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
  }
  if (o & 4) {
    w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
  }
  if (o & 2) {  // bytes 2..3 of one word, then bytes 0..1 of the next
    w0 = __byte_perm(w0, w1, 0x5432);
    w1 = __byte_perm(w1, w2, 0x5432);
    w2 = __byte_perm(w2, w3, 0x5432);
    w3 = __byte_perm(w3, w4, 0x5432);
  }
  return make_uint4(w0, w1, w2, w3);
}

__global__ void pack_rows_f16(const __half* __restrict__ src, long long lds, __half* __restrict__ dst,
                              long long ldd, int rows, int cols) {
  // The GEMM that reads the packed copy is launched as a programmatic
  // dependent: let it start its set-up now (it waits for this grid's
  // completion before it reads anything).
  griddep_launch_dependents();
  const long long chunks = (cols + 7) / 8;
  const long long total = static_cast<long long>(rows) * chunks;
  const uintptr_t begin = reinterpret_cast<uintptr_t>(src);
  const uintptr_t end = begin + (static_cast<uintptr_t>(rows - 1) * static_cast<uintptr_t>(lds) + cols) * 2u;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = idx / chunks;
    const int c = static_cast<int>(idx - r * chunks) * 8;
    const uintptr_t a = begin + static_cast<uintptr_t>(r * lds + c) * 2u;
    const uintptr_t lo = a & ~static_cast<uintptr_t>(15);
    const int o = static_cast<int>(a - lo);
    uint4 w;
    if (c + 8 <= cols && lo >= begin && lo + (o ? 32u : 16u) <= end) {
      const uint4 c0 = __ldg(reinterpret_cast<const uint4*>(lo));
      w = o ? shift_chunks(c0, __ldg(reinterpret_cast<const uint4*>(lo + 16)), o) : c0;
    } else {
      const unsigned short* sp = reinterpret_cast<const unsigned short*>(a);
      unsigned short v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (c + i < cols) ? sp[i] : static_cast<unsigned short>(0);
      w.x = v[0] | (static_cast<unsigned>(v[1]) << 16);
      w.y = v[2] | (static_cast<unsigned>(v[3]) << 16);
      w.z = v[4] | (static_cast<unsigned>(v[5]) << 16);
      w.w = v[6] | (static_cast<unsigned>(v[7]) << 16);
    }
    *reinterpret_cast<uint4*>(dst + r * ldd + c) = w;
  }
}


// Self-test of the bounded waits: one thread waits on an mbarrier that
// nothing will complete, gives up after limit_ns exactly as the GEMM
// kernels' roles do, and records the error bit in the device error word.
__global__ void bounded_wait_selftest(int* err, unsigned long long limit_ns, unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    if (!mbar_wait_limit(&bar, 0, &abort_flag, limit_ns)) atomicOr(err, kDevErrTimeoutSelfTest);
    *waited_ns = globaltimer_ns() - t0;
  }
}

// C = act(beta * D + bias) for an empty reduction (K = 0) with a fused
// epilogue: the accumulator is 0, so alpha plays no part.
__global__ void epilogue_only_f16(GemmParams p) {
  const long long total = static_cast<long long>(p.M) * p.N;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = idx / p.N;
    const int c = static_cast<int>(idx - r * p.N);
    const float d = (p.beta != 0.0f) ? __half2float(p.D[r * p.ldd + c]) : 0.0f;
    const float b = (p.bias != nullptr) ? __half2float(p.bias[c]) : 0.0f;
    p.C[r * p.ldc + c] = __float2half_rn(epilogue_value(p, 0.0f, d, b));
  }
}

enum MenuCol { kColTileM = 0, kColTileN, kColTileK, kColStages, kColMmaSm, kColRaster, kColGroup, kColSplitK };

__device__ int g_device_error = 0;

namespace {

thread_local std::string t_last_error;

int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

int fail_cuda(cudaError_t e, const char* what) {
  return fail(GEMM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      return static_cast<EncodeTiledFn>(nullptr);
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  int max_smem_optin = 0;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GEMM_ERR_UNSUPPORTED, "device index out of range");
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo d;
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_dev[dev] = d;
  });
  *out = g_dev[dev];
  if (out->major != 10 || out->minor != 0) {
    return fail(GEMM_ERR_UNSUPPORTED, "the kernel bank is built for sm_100a (B200); device is sm_" +
                                          std::to_string(out->major) + std::to_string(out->minor));
  }
  return GEMM_OK;
}

bool tma_addressable(const void* p, int64_t pitch_elems) {
  return (reinterpret_cast<uintptr_t>(p) % 16u) == 0 && (pitch_elems % 8) == 0;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

struct Plan {
  bool skinny = false;  // tile_m < 128: gemm_skinny_f16, split_k = CTAs per cluster
  int tile_m = 0, tile_n = 0, stages = 0, cg = 1, raster = 0, group = 1, split_k = 1;
  int tiles_m = 0, tiles_n = 0, num_tiles = 0, kb_total = 0;
  bool streamk = false;
  int workers = 0;    // persistent CTAs (CTA pairs for cg = 2)
  int dp_tiles = 0;   // stream-K: tiles walked data-parallel first
  int sk_workers = 0;  // stream-K: workers sharing the stream-K region
  int64_t sk_iters = 0;  // stream-K: iterations of the stream-K region
  int max_parts = 1;  // partial slots per tile
  bool pack_a = false, pack_b = false;
  size_t off_partials = 0, off_pack_a = 0, off_pack_b = 0, total = 0;
  int64_t lda_packed = 0, ldb_packed = 0;
};

constexpr size_t kCounterBytes = static_cast<size_t>(kCounterSlots) * sizeof(unsigned int);

// Stream-K: the worker that owns (tile, K-block) iteration x when T
// iterations are split evenly over W workers (same formula as the kernel).
int64_t sk_owner(int64_t x, int64_t T, int64_t W) { return ((x + 1) * W - 1) / T; }

// How the operands are stored and what the epilogue computes (gemm_launch_ex).
struct OpDesc {
  int trans_a = 0;  // 0: A stored M x K; 1: A stored K x M
  int trans_b = 0;  // 0: B stored K x N; 1: B stored N x K
  float alpha = 1.0f, beta = 0.0f;
  const void* D = nullptr;
  int64_t ldd = 0;
  const void* bias = nullptr;
  int act = 0;
  const void* const* peers = nullptr;  // fused all-gather targets (gemm_launch_gather)
  int n_peers = 0;
  void* mc_C = nullptr;  // multicast address of C's rows (gemm_launch_multicast)
  bool epi() const { return alpha != 1.0f || beta != 0.0f || bias != nullptr || act != 0; }
};

int make_plan(const void* A, const void* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
              int trans_a, int trans_b, int cfg_id, int sms, Plan* pl) {
  if (cfg_id < 0 || cfg_id >= IDB_MENU_SIZE) {
    return fail(GEMM_ERR_BAD_CFG, "cfg_id " + std::to_string(cfg_id) + " out of range [0, " +
                                      std::to_string(IDB_MENU_SIZE) + ")");
  }
  if (M < 0 || N < 0 || K < 0) return fail(GEMM_ERR_INVALID_ARG, "M, N, K must be >= 0");
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1) {
    return fail(GEMM_ERR_UNSUPPORTED, "M, N, K must each be < 2^31");
  }
  const int* row = kMenu[cfg_id];
  if (row[kColTileM] < kBM) {
    // Skinny kernel: one cluster of split_k CTAs per (tile_m x tile_n) block of
    // C; the K blocks are divided among the cluster.  A cluster size above
    // the number of K blocks is lowered to the largest power of two that
    // still gives every CTA work (same GEMM).
    pl->skinny = true;
    pl->tile_m = row[kColTileM];
    pl->tile_n = row[kColTileN];
    pl->stages = row[kColStages];
    pl->tiles_m = static_cast<int>((M + pl->tile_m - 1) / pl->tile_m);
    pl->tiles_n = static_cast<int>((N + pl->tile_n - 1) / pl->tile_n);
    const int64_t blocks = static_cast<int64_t>(pl->tiles_m) * pl->tiles_n;
    pl->kb_total = static_cast<int>((K + kBK - 1) / kBK);
    int s = row[kColSplitK];
    while (s > 1 && s > pl->kb_total) s /= 2;
    pl->split_k = s;
    if (blocks * s > (1ll << 31) - 1) return fail(GEMM_ERR_UNSUPPORTED, "too many output tiles");
    pl->num_tiles = static_cast<int>(blocks);
    pl->workers = static_cast<int>(blocks);
    pl->max_parts = 1;
  } else {
  pl->tile_m = row[kColTileM];
  pl->tile_n = row[kColTileN];
  pl->cg = row[kColMmaSm];
  pl->stages = row[kColStages];
  pl->raster = row[kColRaster];
  pl->group = row[kColGroup];
  pl->tiles_m = static_cast<int>((M + pl->tile_m - 1) / pl->tile_m);
  pl->tiles_n = static_cast<int>((N + pl->tile_n - 1) / pl->tile_n);
  const int64_t tiles = static_cast<int64_t>(pl->tiles_m) * pl->tiles_n;
  if (tiles > (1ll << 30)) return fail(GEMM_ERR_UNSUPPORTED, "too many output tiles");
  pl->num_tiles = static_cast<int>(tiles);
  pl->kb_total = static_cast<int>((K + kBK - 1) / kBK);
  // A split count above the number of K blocks cannot give every slice work;
  // it is clamped (the result is the same GEMM).  split_k = 0 selects
  // stream-K.
  pl->split_k = row[kColSplitK];
  pl->streamk = (pl->split_k == 0) && pl->kb_total > 0;
  if (pl->split_k < 1) pl->split_k = 1;
  if (pl->split_k > pl->kb_total) pl->split_k = pl->kb_total > 0 ? pl->kb_total : 1;
  const int64_t units = static_cast<int64_t>(pl->num_tiles) * pl->split_k;
  const int64_t slots = sms / pl->cg;
  pl->workers = static_cast<int>(units < slots ? units : slots);
  pl->max_parts = pl->split_k;
  if (pl->streamk) {
    // Hybrid stream-K.  A last wave at most half full: every full wave runs
    // data-parallel and the last wave's R tiles are split over 2R workers,
    // each tile in two K halves (2 partial slots, one fix-up).  Otherwise
    // all full waves but the last run data-parallel and the remaining 1-2
    // waves' worth of tiles are split evenly by iterations over all workers.
    const int64_t T_all = static_cast<int64_t>(pl->num_tiles) * pl->kb_total;
    pl->workers = static_cast<int>(T_all < slots ? T_all : slots);
    const int64_t full_waves = pl->num_tiles / pl->workers;
    const int64_t rem = pl->num_tiles - full_waves * pl->workers;
    pl->sk_workers = pl->workers;
    if (full_waves >= 1 && rem > 0 && 2 * rem <= pl->workers && pl->kb_total >= 2) {
      pl->dp_tiles = static_cast<int>(full_waves * pl->workers);
      pl->sk_workers = static_cast<int>(2 * rem);
    } else {
      pl->dp_tiles = static_cast<int>(full_waves > 1 ? (full_waves - 1) * pl->workers : 0);
    }
    const int64_t T = static_cast<int64_t>(pl->num_tiles - pl->dp_tiles) * pl->kb_total;
    pl->sk_iters = T;
    int64_t mp = 1;
    for (int64_t tile = pl->dp_tiles; tile < pl->num_tiles; ++tile) {
      const int64_t t0 = (tile - pl->dp_tiles) * pl->kb_total;
      const int64_t parts =
          sk_owner(t0 + pl->kb_total - 1, T, pl->sk_workers) - sk_owner(t0, T, pl->sk_workers) + 1;
      if (parts > mp) mp = parts;
    }
    pl->max_parts = static_cast<int>(mp);
  }
  // tickets and partial slots per 128-row half of a tile (one per CTA of a pair)
  if (pl->max_parts > 1 && static_cast<int64_t>(pl->num_tiles) * pl->cg > kCounterSlots) {
    return fail(GEMM_ERR_UNSUPPORTED, "split-K / stream-K support at most 65536 output tile halves");
  }
  }
  pl->pack_a = M > 0 && K > 0 && !tma_addressable(A, lda);
  pl->pack_b = N > 0 && K > 0 && !tma_addressable(B, ldb);
  size_t off = 0;
  if (pl->max_parts > 1 || pl->pack_a || pl->pack_b) off = kCounterBytes;
  if (pl->max_parts > 1) {
    pl->off_partials = off;
    off += static_cast<size_t>(pl->num_tiles) * pl->cg * pl->max_parts * kBM * pl->tile_n * sizeof(float);
    off = static_cast<size_t>(round_up(static_cast<int64_t>(off), 256));
  }
  // A packed copy keeps the operand's stored orientation (rows x cols below).
  // Its pitch is rounded up to 64 elements, so that every row starts on a
  // 128-byte line: a 128-byte TMA box row then touches one line, not two
  // (3-4% faster than 16-byte rows on the 777- and 2049-element pitches).
  if (pl->pack_a) {
    pl->lda_packed = round_up(trans_a ? M : K, 64);
    pl->off_pack_a = off;
    off += static_cast<size_t>(trans_a ? K : M) * pl->lda_packed * 2;
    off = static_cast<size_t>(round_up(static_cast<int64_t>(off), 256));
  }
  if (pl->pack_b) {
    pl->ldb_packed = round_up(trans_b ? K : N, 64);
    pl->off_pack_b = off;
    off += static_cast<size_t>(trans_b ? N : K) * pl->ldb_packed * 2;
    off = static_cast<size_t>(round_up(static_cast<int64_t>(off), 256));
  }
  pl->total = off;
  return GEMM_OK;
}

// swizzled = true: 128-byte swizzle (operand tiles and the main kernel's C
// boxes); false: plain row-major boxes (the skinny kernel's C blocks).
int encode_2d(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t pitch_elems, int box_inner,
              int box_outer, const char* what, bool swizzled = true) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GEMM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch_elems) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzled ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(GEMM_ERR_CUDA, std::string("cuTensorMapEncodeTiled(") + what + ") failed with CUresult " +
                                   std::to_string(static_cast<int>(r)));
  }
  return GEMM_OK;
}

// Recently encoded tensor maps of the calling thread.  A map depends only on
// the address, extents, pitch, box and swizzle, so repeated launches on the same
// buffers (the common case: a tuner loop, a model step) reuse it instead of
// encoding it again.
struct MapCacheEntry {
  const void* base = nullptr;
  int64_t inner = 0, outer = 0, pitch = 0;
  int box_inner = 0, box_outer = 0;
  bool swizzled = true;
  bool valid = false;
  CUtensorMap map;
};
constexpr int kMapCacheSize = 32;   // A, B, C and, for the fused all-gather, up to 2 x 7 peer C buffers
thread_local MapCacheEntry t_map_cache[kMapCacheSize];
thread_local int t_map_next = 0;

int encode_2d_cached(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t pitch_elems,
                     int box_inner, int box_outer, const char* what, bool swizzled = true) {
  for (const MapCacheEntry& e : t_map_cache) {
    if (e.valid && e.base == base && e.inner == inner && e.outer == outer && e.pitch == pitch_elems &&
        e.box_inner == box_inner && e.box_outer == box_outer && e.swizzled == swizzled) {
      *map = e.map;
      return GEMM_OK;
    }
  }
  const int st = encode_2d(map, base, inner, outer, pitch_elems, box_inner, box_outer, what, swizzled);
  if (st != GEMM_OK) return st;
  MapCacheEntry& e = t_map_cache[t_map_next];
  t_map_next = (t_map_next + 1) % kMapCacheSize;
  e.base = base;
  e.inner = inner;
  e.outer = outer;
  e.pitch = pitch_elems;
  e.box_inner = box_inner;
  e.box_outer = box_outer;
  e.swizzled = swizzled;
  e.map = *map;
  e.valid = true;
  return GEMM_OK;
}

// Device address of the error word, looked up once per device.
int* g_err_word[kMaxDevices] = {};
cudaError_t g_err_status[kMaxDevices] = {};
std::once_flag g_err_once[kMaxDevices];

int launch_pack(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t rows, int64_t cols,
                cudaStream_t stream) {
  const int64_t chunks = rows * ((cols + 7) / 8);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  pack_rows_f16<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const __half*>(src), lds, static_cast<__half*>(dst), ldd, static_cast<int>(rows),
      static_cast<int>(cols));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GEMM_OK : fail_cuda(e, "pack_rows_f16 launch");
}

int launch_impl(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                int64_t ldc, const OpDesc& op, int cfg_id, void* ws, size_t ws_bytes, void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (M < 0 || N < 0 || K < 0) return fail(GEMM_ERR_INVALID_ARG, "M, N, K must be >= 0");
  if ((op.trans_a != 0 && op.trans_a != 1) || (op.trans_b != 0 && op.trans_b != 1)) {
    return fail(GEMM_ERR_INVALID_ARG, "trans_a and trans_b must be 0 or 1");
  }
  if (op.act < GEMM_ACT_NONE || op.act > GEMM_ACT_GELU) {
    return fail(GEMM_ERR_INVALID_ARG, "activation must be GEMM_ACT_NONE, GEMM_ACT_RELU or GEMM_ACT_GELU");
  }
  if (M == 0 || N == 0) return GEMM_OK;
  if (!C || (K > 0 && (!A || !B))) return fail(GEMM_ERR_INVALID_ARG, "A, B and C must be non-null");
  const int64_t a_cols = op.trans_a ? M : K, b_cols = op.trans_b ? K : N;
  if (lda < a_cols || ldb < b_cols || ldc < N) {
    return fail(GEMM_ERR_INVALID_ARG, std::string("pitches must satisfy lda >= ") + (op.trans_a ? "M" : "K") +
                                          ", ldb >= " + (op.trans_b ? "K" : "N") + ", ldc >= N");
  }
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) % 2u) {
    return fail(GEMM_ERR_INVALID_ARG, "A, B and C must be 2-byte aligned (fp16)");
  }
  if (op.beta != 0.0f && (!op.D || op.ldd < N || reinterpret_cast<uintptr_t>(op.D) % 2u)) {
    return fail(GEMM_ERR_INVALID_ARG, "beta != 0 needs a 2-byte aligned D with ldd >= N");
  }
  if (op.bias && reinterpret_cast<uintptr_t>(op.bias) % 2u) {
    return fail(GEMM_ERR_INVALID_ARG, "bias must be 2-byte aligned (fp16)");
  }
  if (op.n_peers < 0 || op.n_peers > kMaxPeers || (op.n_peers > 0 && !op.peers)) {
    return fail(GEMM_ERR_INVALID_ARG, "n_peers must be in [0, " + std::to_string(kMaxPeers) +
                                          "] with a peer pointer array");
  }
  for (int i = 0; i < op.n_peers; ++i) {
    if (!op.peers[i] || reinterpret_cast<uintptr_t>(op.peers[i]) % 2u) {
      return fail(GEMM_ERR_INVALID_ARG, "peer C pointers must be non-null and 2-byte aligned");
    }
  }
  if (cfg_id < 0 || cfg_id >= IDB_MENU_SIZE) {
    return fail(GEMM_ERR_BAD_CFG, "cfg_id " + std::to_string(cfg_id) + " out of range [0, " +
                                      std::to_string(IDB_MENU_SIZE) + ")");
  }
  DeviceInfo dinfo;
  int st = device_info(&dinfo);
  if (st != GEMM_OK) return st;
  Plan pl;
  st = make_plan(A, B, M, N, K, lda, ldb, op.trans_a, op.trans_b, cfg_id, dinfo.sms, &pl);
  if (st != GEMM_OK) return st;

  GemmParams p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = static_cast<__half*>(C);
  p.ldc = ldc;
  p.a_mn = op.trans_a;
  p.b_kmaj = op.trans_b;
  p.epi = op.epi() ? 1 : 0;
  p.act = op.act;
  p.alpha = op.alpha;
  p.beta = op.beta;
  p.D = op.beta != 0.0f ? static_cast<const __half*>(op.D) : nullptr;
  p.ldd = op.beta != 0.0f ? op.ldd : 0;
  p.bias = static_cast<const __half*>(op.bias);
  p.n_peers = op.n_peers;
  p.peer_tma = 0;
  for (int i = 0; i < kMaxPeers; ++i) {
    p.peer_C[i] = i < op.n_peers ? static_cast<__half*>(const_cast<void*>(op.peers[i])) : nullptr;
  }
  std::memset(p.peer_map, 0, sizeof(p.peer_map));
  p.mc_C = static_cast<__half*>(op.mc_C);
  if ((op.n_peers > 0 || op.mc_C) && (pl.skinny || pl.max_parts > 1 || K == 0)) {
    return fail(GEMM_ERR_UNSUPPORTED, "the fused all-gather needs K > 0 and a configuration without split-K / "
                                      "stream-K and with tile_m >= 128");
  }
  if (K == 0) {
    // Empty reduction: C = 0 (the reference kernel's loop body never runs),
    // or act(beta * D + bias) with a fused epilogue.
    if (p.epi) {
      const long long total = M * N;
      long long blocks = (total + 255) / 256;
      if (blocks > 148 * 8) blocks = 148 * 8;
      epilogue_only_f16<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
      cudaError_t e = cudaGetLastError();
      return e == cudaSuccess ? GEMM_OK : fail_cuda(e, "epilogue_only_f16 launch");
    }
    cudaError_t e = cudaMemset2DAsync(C, static_cast<size_t>(ldc) * 2, 0, static_cast<size_t>(N) * 2,
                                      static_cast<size_t>(M), stream);
    return e == cudaSuccess ? GEMM_OK : fail_cuda(e, "cudaMemset2DAsync");
  }
  if (pl.total > 0 && (ws == nullptr || ws_bytes < pl.total)) {
    return fail(GEMM_ERR_WORKSPACE, "workspace of " + std::to_string(pl.total) + " bytes required, got " +
                                        std::to_string(ws == nullptr ? 0 : ws_bytes));
  }
  if (pl.total > 0 && (reinterpret_cast<uintptr_t>(ws) % 256u) != 0) {
    return fail(GEMM_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  const Variant* var = nullptr;
  const SkinnyVariant* svar = nullptr;
  if (pl.skinny) {
    if (op.trans_a) {
      return fail(GEMM_ERR_UNSUPPORTED, "skinny configurations (tile_m < 128) read A stored M x K (trans_a = 0)");
    }
    for (const SkinnyVariant& v : kSkinnyVariants) {
      if (v.tm == pl.tile_m && v.tn == pl.tile_n && v.stages == pl.stages) svar = &v;
    }
    if (!svar) return fail(GEMM_ERR_BAD_CFG, "no compiled skinny kernel for this configuration");
  } else {
    for (const Variant& v : kVariants) {
      if (v.bn == pl.tile_n && v.stages == pl.stages && v.cg == pl.cg) var = &v;
    }
    if (!var) return fail(GEMM_ERR_BAD_CFG, "no compiled kernel for this configuration");
  }

  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const void* a_src = A;
  int64_t a_ld = lda;
  const void* b_src = B;
  int64_t b_ld = ldb;
  if (pl.pack_a) {
    st = launch_pack(A, lda, wsb + pl.off_pack_a, pl.lda_packed, op.trans_a ? K : M, op.trans_a ? M : K, stream);
    if (st != GEMM_OK) return st;
    a_src = wsb + pl.off_pack_a;
    a_ld = pl.lda_packed;
  }
  if (pl.pack_b) {
    st = launch_pack(B, ldb, wsb + pl.off_pack_b, pl.ldb_packed, op.trans_b ? N : K, op.trans_b ? K : N, stream);
    if (st != GEMM_OK) return st;
    b_src = wsb + pl.off_pack_b;
    b_ld = pl.ldb_packed;
  }

  CUtensorMap tmA, tmB, tmC;
  std::memset(&tmC, 0, sizeof(tmC));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  std::call_once(g_err_once[dev], [dev] {
    g_err_status[dev] = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_err_word[dev]), g_device_error);
  });
  if (g_err_status[dev] != cudaSuccess) return fail_cuda(g_err_status[dev], "cudaGetSymbolAddress(g_device_error)");
  p.err = g_err_word[dev];

  if (pl.skinny) {
    // A: [tile_m rows x 64 K] boxes; B: [128 n x 64 K] (stored N x K) or
    // [64 K x 64 n] atoms (stored K x N); C: plain [min(tile_n / S, 256) x
    // tile_m] boxes written by TMA stores when C is TMA-addressable, else
    // per-thread stores.
    st = encode_2d_cached(&tmA, a_src, K, M, a_ld, kBK, pl.tile_m, "A");
    if (st != GEMM_OK) return st;
    if (op.trans_b) {
      st = encode_2d_cached(&tmB, b_src, K, N, b_ld, kBK, kSkinnyN, "B (stored N x K)");
    } else {
      st = encode_2d_cached(&tmB, b_src, N, K, b_ld, 64, kBK, "B");
    }
    if (st != GEMM_OK) return st;
    p.kb_total = pl.kb_total;
    p.tiles_m = pl.tiles_m;
    p.tiles_n = pl.tiles_n;
    p.num_tiles = pl.num_tiles;
    p.split_k = pl.split_k;
    p.partials = nullptr;
    p.counters = nullptr;
    const bool c_tma = tma_addressable(C, ldc);
    if (c_tma) {
      st = encode_2d_cached(&tmC, C, N, M, ldc, skinny_c_box(pl.tile_n / pl.split_k), pl.tile_m, "C", false);
      if (st != GEMM_OK) return st;
    }
    p.c_tma = c_tma ? 1 : 0;
    e = svar->fn(tmA, tmB, tmC, p, pl.num_tiles * pl.split_k, pl.split_k, stream);
    if (e != cudaSuccess) return fail_cuda(e, "skinny gemm kernel launch");
    return GEMM_OK;
  }

  // Boxes: K-major A [64 K x 128 rows]; M-major A, and B either way, in
  // 64 x 64 atoms (see the producer in gemm_sm100_kernel.cuh).
  if (op.trans_a) {
    st = encode_2d_cached(&tmA, a_src, M, K, a_ld, 64, kBK, "A (stored K x M)");
  } else {
    st = encode_2d_cached(&tmA, a_src, K, M, a_ld, kBK, kBM, "A");
  }
  if (st != GEMM_OK) return st;
  if (op.trans_b) {
    st = encode_2d_cached(&tmB, b_src, K, N, b_ld, kBK, 64, "B (stored N x K)");
  } else {
    st = encode_2d_cached(&tmB, b_src, N, K, b_ld, 64, kBK, "B");
  }
  if (st != GEMM_OK) return st;
  // With a multicast C every box leaves through multimem stores instead.
  const bool c_tma = !op.mc_C && tma_addressable(C, ldc);
  if (c_tma) {
    st = encode_2d_cached(&tmC, C, N, M, ldc, kStoreCols, kStoreRows, "C");
    if (st != GEMM_OK) return st;
    // Fused all-gather: each peer's copy of C gets the same map at its own
    // address, so every staged box goes there by one TMA store.
    bool peers_tma = p.n_peers > 0;
    for (int i = 0; i < p.n_peers; ++i) peers_tma = peers_tma && tma_addressable(op.peers[i], ldc);
    if (peers_tma) {
      for (int i = 0; i < p.n_peers; ++i) {
        st = encode_2d_cached(&p.peer_map[i], op.peers[i], N, M, ldc, kStoreCols, kStoreRows, "peer C");
        if (st != GEMM_OK) return st;
      }
      p.peer_tma = 1;
    }
  }

  p.tiles_m = pl.tiles_m;
  p.tiles_n = pl.tiles_n;
  p.num_tiles = pl.num_tiles;
  p.split_k = pl.split_k;
  p.kb_total = pl.kb_total;
  p.streamk = pl.streamk ? 1 : 0;
  p.max_parts = pl.max_parts;
  p.dp_tiles = pl.dp_tiles;
  p.sk_workers = pl.streamk ? pl.sk_workers : pl.workers;
  p.total_iters = pl.streamk ? pl.sk_iters : static_cast<long long>(pl.num_tiles) * pl.kb_total;
  p.raster = pl.raster;
  p.group = pl.group;
  p.c_tma = c_tma ? 1 : 0;
  p.partials = pl.max_parts > 1 ? reinterpret_cast<float*>(wsb + pl.off_partials) : nullptr;
  p.counters = pl.max_parts > 1 ? reinterpret_cast<unsigned int*>(wsb) : nullptr;

  // persistent grid: one CTA (or CTA pair) per SM (pair), at most one per work unit
  const int grid = pl.workers * pl.cg;
  e = var->fn(tmA, tmB, tmC, p, grid, stream);
  if (e != cudaSuccess) return fail_cuda(e, "gemm kernel launch");
  return GEMM_OK;
}

}  // namespace

void record_last_error(const std::string& msg) { t_last_error = msg; }

// Imported peer pointer -> base of the opened allocation (for gemm_ipc_close).
std::mutex g_ipc_mu;
std::map<void*, void*>* g_ipc_bases = new std::map<void*, void*>();

}  // namespace idb

using namespace idb;

extern "C" {

int gemm_num_cfgs(void) { return IDB_MENU_SIZE; }

int gemm_cfg_num_cols(void) { return IDB_MENU_COLS; }

const char* gemm_cfg_col_name(int col) {
  if (col < 0 || col >= IDB_MENU_COLS) return nullptr;
  return kMenuColumns[col];
}

int gemm_cfg_row(int cfg_id, int* out, int n) {
  if (cfg_id < 0 || cfg_id >= IDB_MENU_SIZE) return fail(GEMM_ERR_BAD_CFG, "cfg_id out of range");
  if (!out || n < 0) return fail(GEMM_ERR_INVALID_ARG, "out must be non-null and n >= 0");
  for (int i = 0; i < n && i < IDB_MENU_COLS; ++i) out[i] = kMenu[cfg_id][i];
  return GEMM_OK;
}

int gemm_cfg_find(const int* knobs, int n) {
  if (!knobs || n != IDB_MENU_COLS) return -1;
  // The menu is sorted lexicographically: binary search.
  int lo = 0, hi = IDB_MENU_SIZE - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    int cmp = 0;
    for (int i = 0; i < IDB_MENU_COLS && cmp == 0; ++i) {
      cmp = (kMenu[mid][i] < knobs[i]) ? -1 : (kMenu[mid][i] > knobs[i]) ? 1 : 0;
    }
    if (cmp == 0) return mid;
    if (cmp < 0) lo = mid + 1;
    else hi = mid - 1;
  }
  return -1;
}

size_t gemm_workspace_bytes_ex(const void* A, const void* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, int trans_a, int trans_b, int cfg_id) {
  Plan pl;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // Stream-K workspace depends on the SM count of the current device (148
  // on a B200; assumed when no device is visible).
  int sms = 148;
  DeviceInfo dinfo;
  if (device_info(&dinfo) == GEMM_OK && dinfo.sms > 0) {
    sms = dinfo.sms;
  } else {
    cudaGetLastError();
    t_last_error.clear();
  }
  if (make_plan(A, B, M, N, K, lda, ldb, trans_a, trans_b, cfg_id, sms, &pl) != GEMM_OK) return 0;
  return pl.total;
}

size_t gemm_workspace_bytes(const void* A, const void* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                            int64_t ldb, int cfg_id) {
  return gemm_workspace_bytes_ex(A, B, M, N, K, lda, ldb, 0, 0, cfg_id);
}

size_t gemm_workspace_counter_bytes(void) { return kCounterBytes; }

int gemm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                int64_t ldc, int cfg_id, void* workspace, size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  return launch_impl(A, B, C, M, N, K, lda, ldb, ldc, OpDesc{}, cfg_id, workspace, workspace_bytes, stream);
}

int gemm_launch_ex(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                   int64_t ldb, int64_t ldc, int trans_a, int trans_b, float alpha, float beta, const void* D,
                   int64_t ldd, const void* bias, int activation, int cfg_id, void* workspace,
                   size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  OpDesc op;
  op.trans_a = trans_a;
  op.trans_b = trans_b;
  op.alpha = alpha;
  op.beta = beta;
  op.D = D;
  op.ldd = ldd;
  op.bias = bias;
  op.act = activation;
  return launch_impl(A, B, C, M, N, K, lda, ldb, ldc, op, cfg_id, workspace, workspace_bytes, stream);
}

int gemm_launch_gather(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, int64_t ldc, const void* const* peer_C, int n_peers, int cfg_id, void* workspace,
                       size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  OpDesc op;
  op.peers = peer_C;
  op.n_peers = n_peers;
  return launch_impl(A, B, C, M, N, K, lda, ldb, ldc, op, cfg_id, workspace, workspace_bytes, stream);
}

int gemm_launch_multicast(const void* A, const void* B, void* C, void* C_mc, int64_t M, int64_t N, int64_t K,
                          int64_t lda, int64_t ldb, int64_t ldc, int cfg_id, void* workspace,
                          size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (!C_mc) return fail(GEMM_ERR_INVALID_ARG, "C_mc must be non-null");
  if (reinterpret_cast<uintptr_t>(C_mc) % 16u || reinterpret_cast<uintptr_t>(C) % 16u || N % 8 || ldc % 8) {
    return fail(GEMM_ERR_UNSUPPORTED, "the multicast all-gather needs 16-byte aligned C and C_mc and N and ldc "
                                      "multiples of 8");
  }
  OpDesc op;
  op.mc_C = C_mc;
  return launch_impl(A, B, C, M, N, K, lda, ldb, ldc, op, cfg_id, workspace, workspace_bytes, stream);
}

int gemm_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  t_last_error.clear();
  if (!ptr || !handle || !offset) return fail(GEMM_ERR_INVALID_ARG, "ptr, handle and offset must be non-null");
  // The handle names the whole allocation that holds ptr; the offset locates ptr in it.
  CUdeviceptr base = 0;
  size_t size = 0;
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      return static_cast<RangeFn>(nullptr);
    }
    return reinterpret_cast<RangeFn>(f);
  }();
  if (!range) return fail(GEMM_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    return fail(GEMM_ERR_INVALID_ARG, "ptr is not device memory of this process");
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail_cuda(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return GEMM_OK;
}

int gemm_ipc_import(const void* handle, int64_t offset, void** ptr) {
  t_last_error.clear();
  if (!handle || !ptr || offset < 0) return fail(GEMM_ERR_INVALID_ARG, "handle and ptr must be non-null, offset >= 0");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail_cuda(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<uint8_t*>(base) + offset;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  (*g_ipc_bases)[*ptr] = base;
  return GEMM_OK;
}

int gemm_ipc_close(void* ptr) {
  t_last_error.clear();
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_ipc_mu);
    auto it = g_ipc_bases->find(ptr);
    if (it == g_ipc_bases->end()) return fail(GEMM_ERR_INVALID_ARG, "ptr was not returned by gemm_ipc_import");
    base = it->second;
    g_ipc_bases->erase(it);
  }
  cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? GEMM_OK : fail_cuda(e, "cudaIpcCloseMemHandle");
}

int gemm_launch_knobs(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                      int64_t ldb, int64_t ldc, const int* knobs, int n, void* workspace, size_t workspace_bytes,
                      void* stream) {
  t_last_error.clear();
  const int id = gemm_cfg_find(knobs, n);
  if (id < 0) {
    std::string t = "(";
    for (int i = 0; knobs && i < n; ++i) t += (i ? "," : "") + std::to_string(knobs[i]);
    return fail(GEMM_ERR_BAD_CFG, "knob tuple " + t + ") is not in the kernel bank menu");
  }
  return launch_impl(A, B, C, M, N, K, lda, ldb, ldc, OpDesc{}, id, workspace, workspace_bytes, stream);
}

int gemm_default_cfg(int64_t M, int64_t N, int64_t K) {
  // Heuristic used when no tuned entry exists:
  //  * enough 256 x 512 (else 256 x 256) tiles to fill the 74 CTA pairs of a
  //    B200: CTA-pair (cta_group::2) kernel, 4 stages;
  //  * otherwise one CTA per 128-row tile, the widest tile_n that still
  //    gives ~one wave, and split-K when the output has too few tiles to
  //    occupy the 148 SMs.
  const int kSms = 148;
  const int64_t pairs = kSms / 2;
  const int64_t kb = (K + kBK - 1) / kBK;
  if (M >= 1 && M <= 64) {
    // Few rows: the skinny kernel (C^T tiles of 128 columns, split-K inside a
    // cluster).  The smallest row tile that holds M, the deepest ring that
    // fits, and the largest cluster that keeps about one wave with >= 4 K
    // blocks per CTA.
    // Measured on B200: clusters of 8 cost more to launch than they save,
    // and when 128-column blocks alone fill more than half the SMs, 256-column
    // blocks in clusters of 2 stream B faster (512 contiguous bytes per row)
    // for up to 32 rows; at 64 rows their 5-stage ring is too shallow.
    const int tm = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    const int64_t blocks = (N + kSkinnyN - 1) / kSkinnyN;
    const int64_t wide = (N + 2 * kSkinnyN - 1) / (2 * kSkinnyN);
    if (tm <= 32 && blocks > pairs && wide * 2 <= kSms && kb >= 8) {
      int knobs[IDB_MENU_COLS] = {tm, 2 * kSkinnyN, kBK, 6, 1, 0, 1, 2};
      return gemm_cfg_find(knobs, IDB_MENU_COLS);
    }
    const int stages = tm == 16 ? 12 : (tm == 32 ? 10 : 8);
    int s = 1;
    while (s < 4 && blocks * 2 * s <= kSms && kb / (2 * s) >= 4) s *= 2;
    int knobs[IDB_MENU_COLS] = {tm, kSkinnyN, kBK, stages, 1, 0, 1, s};
    return gemm_cfg_find(knobs, IDB_MENU_COLS);
  }
  // Fraction of the last persistent wave's slots that have work.
  auto wave_fill = [pairs](int64_t tiles) {
    const int64_t waves = (tiles + pairs - 1) / pairs;
    return static_cast<double>(tiles) / static_cast<double>(waves * pairs);
  };
  const int64_t wide_pair_tiles = ((M + 255) / 256) * ((N + 511) / 512);
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  // 256 x 512 tiles on CTA pairs: A is loaded once for two 256-column
  // halves, the least L2 traffic per FLOP in the bank -- unless their last
  // wave leaves many pairs idle and 256 x 256 tiles fill the waves better.
  if (wide_pair_tiles >= pairs && !(wave_fill(wide_pair_tiles) < 0.93 && wave_fill(pair_tiles) > 0.97)) {
    int knobs[IDB_MENU_COLS] = {2 * kBM, 512, kBK, 4, 2, 1, 8, 1};
    return gemm_cfg_find(knobs, IDB_MENU_COLS);
  }
  if (pair_tiles >= pairs) {
    int knobs[IDB_MENU_COLS] = {2 * kBM, 256, kBK, 4, 2, 0, 8, 1};
    return gemm_cfg_find(knobs, IDB_MENU_COLS);
  }
  int tile_n = 256, stages = 4;
  const int64_t tm = (M + kBM - 1) / kBM;
  if (tm * ((N + 255) / 256) < kSms) {
    tile_n = 128;
    stages = 6;
  }
  const int64_t tiles = tm * ((N + tile_n - 1) / tile_n);
  int split = 1;
  if (tiles < kSms / 2 && kb >= 8) {
    const int choices[] = {16, 12, 8, 6, 4, 3, 2};
    for (int c : choices) {
      if (tiles * c <= kSms + kSms / 4 && kb / c >= 4) {
        split = c;
        break;
      }
    }
  }
  int knobs[IDB_MENU_COLS] = {kBM, tile_n, kBK, stages, 1, 0, 8, split};
  return gemm_cfg_find(knobs, IDB_MENU_COLS);
}

int gemm_selftest_wait_timeout(uint64_t limit_ns, uint64_t* waited_ns) {
  t_last_error.clear();
  if (limit_ns == 0 || limit_ns > 1000000000ull) {
    return fail(GEMM_ERR_INVALID_ARG, "limit_ns must be in (0, 1e9]");
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GEMM_ERR_UNSUPPORTED, "device index out of range");
  std::call_once(g_err_once[dev], [dev] {
    g_err_status[dev] = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_err_word[dev]), g_device_error);
  });
  if (g_err_status[dev] != cudaSuccess) return fail_cuda(g_err_status[dev], "cudaGetSymbolAddress(g_device_error)");
  unsigned long long* d_waited = nullptr;
  e = cudaMalloc(&d_waited, sizeof(unsigned long long));
  if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc");
  bounded_wait_selftest<<<1, 32>>>(g_err_word[dev], limit_ns, d_waited);
  e = cudaGetLastError();
  unsigned long long h = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h, d_waited, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(d_waited);
  if (e != cudaSuccess) return fail_cuda(e, "bounded_wait_selftest");
  if (waited_ns) *waited_ns = h;
  return GEMM_OK;
}

int gemm_device_error(int device, int* code) {
  t_last_error.clear();
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (device != prev && (e = cudaSetDevice(device)) != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
  int v = 0;
  const int zero = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e == cudaSuccess && v != 0) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail_cuda(e, "reading the device error word");
  if (code) *code = v;
  if (v != 0) return fail(GEMM_ERR_DEVICE_TIMEOUT, "a kernel gave up on a bounded wait (error bits " +
                                                       std::to_string(v) + ")");
  return GEMM_OK;
}

const char* gemm_last_error(void) { return t_last_error.c_str(); }

const char* gemm_status_string(int status) {
  switch (status) {
    case GEMM_OK: return "GEMM_OK";
    case GEMM_ERR_INVALID_ARG: return "GEMM_ERR_INVALID_ARG";
    case GEMM_ERR_BAD_CFG: return "GEMM_ERR_BAD_CFG";
    case GEMM_ERR_WORKSPACE: return "GEMM_ERR_WORKSPACE";
    case GEMM_ERR_CUDA: return "GEMM_ERR_CUDA";
    case GEMM_ERR_UNSUPPORTED: return "GEMM_ERR_UNSUPPORTED";
    case GEMM_ERR_DEVICE_TIMEOUT: return "GEMM_ERR_DEVICE_TIMEOUT";
    default: return "GEMM_ERR_UNKNOWN";
  }
}

}  // extern "C"
