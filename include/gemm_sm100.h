/*
 * gemm_sm100.h -- C ABI of the B200 (sm_100a) FP16 GEMM kernel bank.
 *
 * C[M,N] (fp16) = A[M,K] (fp16) * B[K,N] (fp16), fp32 accumulation, all
 * matrices row-major with element pitches lda / ldb / ldc.
 *
 * This library replaces the reference extension `infinite_dreams_ext`
 * (src/gemm_ext.cpp:123-132) and its launcher chain
 * (src/gemm_cuda.cu:5-15, generated gemm_try_bank_NNN from
 * src/gen_gemm_bank.py:216-236).  Every entry point below names the
 * reference interface it replaces.  The signatures carry plain pointers and
 * sizes only; no torch types cross this boundary.
 *
 * Ownership: the caller owns A, B, C and the workspace.  gemm_launch is
 * asynchronous on the caller's stream and allocates nothing.  Calls from
 * several host threads are safe; launches that share one workspace must not
 * overlap on the GPU.
 *
 * Errors: every entry point returns a status code (never fails silently; the
 * reference launched nothing and returned an uninitialised tensor when a tile
 * was not in its menu).  gemm_last_error() gives a message for the calling
 * thread's most recent failure.
 */
#ifndef INFINITE_DREAMS_GEMM_SM100_H_
#define INFINITE_DREAMS_GEMM_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define GEMM_OK 0
#define GEMM_ERR_INVALID_ARG 1     /* bad sizes, pitches, null pointers       */
#define GEMM_ERR_BAD_CFG 2         /* cfg_id / knob tuple not in the menu      */
#define GEMM_ERR_WORKSPACE 3       /* workspace missing or too small           */
#define GEMM_ERR_CUDA 4            /* a CUDA runtime / driver call failed      */
#define GEMM_ERR_UNSUPPORTED 5     /* device is not sm_100 or shape too large  */
#define GEMM_ERR_DEVICE_TIMEOUT 6  /* a kernel gave up on a bounded wait       */

/* Number of configurations in the menu.
 * Replaces: gemm_cfg_menu().size() (generated gemm_cfg_menu.h,
 * src/gen_gemm_bank.py:239-251), seen through gemm_cfg_table_cpu
 * (src/gemm_ext.cpp:108-120). */
int gemm_num_cfgs(void);

/* Number of knob columns per menu row (tile_m, tile_n, tile_k, stages,
 * mma_sm, raster, group, split_k). Replaces the fixed 5 columns of
 * gemm_cfg_table_cpu (src/gemm_ext.cpp:108-120). */
int gemm_cfg_num_cols(void);

/* Name of knob column `col` ("tile_m", ...), or NULL if out of range. */
const char* gemm_cfg_col_name(int col);

/* Copies menu row `cfg_id` into out[0..n). Returns GEMM_OK or
 * GEMM_ERR_BAD_CFG / GEMM_ERR_INVALID_ARG.
 * Replaces: one row of gemm_cfg_table_cpu (src/gemm_ext.cpp:108-120). */
int gemm_cfg_row(int cfg_id, int* out, int n);

/* Menu index of a knob tuple (n = gemm_cfg_num_cols()), or -1.
 * Replaces: the exact-match 5-tuple compare of TRY_CFG
 * (src/gemm_kernels.cuh:87-96) and the tuner's _TUPLE_TO_ID
 * (infinite_dreams/tuner.py:25-27). */
int gemm_cfg_find(const int* knobs, int n);

/* Workspace bytes gemm_launch needs for this problem and config (0 when the
 * config uses no split-K and both A and B are TMA-addressable: base 16-byte
 * aligned and pitch a multiple of 8 elements).  The first
 * gemm_workspace_counter_bytes() bytes of any non-empty workspace must be
 * zero before its first use; every successful launch leaves them zero.
 * No counterpart in the reference (it had no workspace, gemm_ext.cpp:35). */
size_t gemm_workspace_bytes(const void* A, const void* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                            int64_t ldb, int cfg_id);

/* Size of the zero-initialised ticket region at the head of a workspace. */
size_t gemm_workspace_counter_bytes(void);

/* Launch C = A*B with menu configuration cfg_id on `stream` (a cudaStream_t,
 * NULL = legacy default stream).  Asynchronous.
 * Replaces: gemm_forward_cfg (src/gemm_ext.cpp:95-106) ->
 * gemm_forward_cuda_impl (src/gemm_ext.cpp:22-52) ->
 * gemm_forward_cuda_launcher (src/gemm_cuda.cu:5-15). */
int gemm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                int64_t ldb, int64_t ldc, int cfg_id, void* workspace, size_t workspace_bytes, void* stream);

/* Same as gemm_launch but the configuration is given as a knob tuple
 * (n = gemm_cfg_num_cols()); a tuple that is not in the menu is an error.
 * Replaces: gemm_forward(A,B,tile_m,tile_n,tile_k,tm,tn)
 * (src/gemm_ext.cpp:57-93), which silently launched nothing on a miss. */
int gemm_launch_knobs(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                      int64_t ldb, int64_t ldc, const int* knobs, int n, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Activations of the fused epilogue (gemm_launch_ex). */
#define GEMM_ACT_NONE 0
#define GEMM_ACT_RELU 1 /* max(x, 0)                                    */
#define GEMM_ACT_GELU 2 /* x * Phi(x) = 0.5 x (1 + erf(x / sqrt(2)))    */

/* C = act(alpha * op(A) * op(B) + beta * D + bias), rounded once to fp16.
 *  op(A) = A (stored M x K, lda >= K) when trans_a = 0, or A^T with A stored
 *          K x M (lda >= M) when trans_a = 1;
 *  op(B) = B (stored K x N, ldb >= N) when trans_b = 0, or B^T with B stored
 *          N x K (ldb >= K) when trans_b = 1;
 *  D     = fp16 M x N with pitch ldd >= N; read only when beta != 0, and may
 *          be C itself (in-place accumulate);
 *  bias  = fp16[N] added to every row, or NULL; it must not overlap C;
 *  activation = GEMM_ACT_*.
 * The epilogue runs in fp32 on the fp32 accumulator.  With alpha = 1,
 * beta = 0, no bias and no activation the result is exactly gemm_launch's.
 * Transposed operands are read in place: the tensor cores take either major
 * order from shared memory, so no transposed copy is made.  Any cfg_id
 * serves every layout; the workspace comes from gemm_workspace_bytes_ex.
 * Extends gemm_launch beyond the reference, whose op took only row-major
 * A and B (made contiguous first, src/gemm_ext.cpp:89-90) and returned A*B. */
int gemm_launch_ex(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                   int64_t ldb, int64_t ldc, int trans_a, int trans_b, float alpha, float beta, const void* D,
                   int64_t ldd, const void* bias, int activation, int cfg_id, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Workspace bytes gemm_launch_ex needs (operands stored as trans_a/trans_b
 * say); gemm_workspace_bytes is this with trans_a = trans_b = 0. */
size_t gemm_workspace_bytes_ex(const void* A, const void* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, int trans_a, int trans_b, int cfg_id);

/* Fused all-gather for M-row sharding over the GPUs of one node (one
 * process per GPU).  Same as gemm_launch, and each finished tile of C is
 * also stored, over NVLink, at the same offset and pitch ldc into
 * peer_C[0..n_peers) -- the copies of the full C on the other GPUs (opened
 * with gemm_ipc_import), already offset to this rank's rows.  When C and
 * every peer copy are TMA-addressable, each staged box goes to the peers by
 * TMA stores beside the local one; otherwise the epilogue warps copy it
 * with 16-byte stores.  The transfer overlaps the GEMM tile by tile.  The
 * caller learns that every peer has
 * finished writing into its own C from a collective issued after the
 * launch on the same stream (the stream orders it after this grid on every
 * rank).  n_peers <= GEMM_MAX_PEERS; the configuration must have
 * tile_m >= 128 and split_k = 1 (GEMM_ERR_UNSUPPORTED otherwise).
 * Extends the reference, which ran on one GPU; replaces a separate NCCL
 * all-gather of the C row blocks. */
#define GEMM_MAX_PEERS 7
int gemm_launch_gather(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, int64_t ldc, const void* const* peer_C, int n_peers, int cfg_id,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Multicast all-gather: same as gemm_launch_gather, but every rank's full C
 * is bound to one NVLink multicast object (NVLS) and C_mc is the multicast
 * address of this rank's rows (C is their ordinary address on this GPU).
 * Each finished box of C is stored once, through C_mc, and NVSwitch writes
 * it into every rank's copy, this rank's included: the GPU sends each byte
 * of C once instead of once per peer.  C_mc must come from a multicast
 * mapping that covers M rows of pitch ldc; C and C_mc 16-byte aligned, N
 * and ldc multiples of 8, tile_m >= 128 and split_k = 1
 * (GEMM_ERR_UNSUPPORTED otherwise).  Completion across ranks as for
 * gemm_launch_gather.  Extends the reference, which ran on one GPU. */
int gemm_launch_multicast(const void* A, const void* B, void* C, void* C_mc, int64_t M, int64_t N, int64_t K,
                          int64_t lda, int64_t ldb, int64_t ldc, int cfg_id, void* workspace,
                          size_t workspace_bytes, void* stream);

/* CUDA IPC of device memory between the processes of one node, for
 * gemm_launch_gather.  gemm_ipc_export writes the GEMM_IPC_HANDLE_BYTES-byte
 * handle of the allocation that holds ptr and ptr's offset inside it;
 * another process passes both to gemm_ipc_import to map that memory (peer
 * access enabled) and gets the same address in its own space;
 * gemm_ipc_close unmaps it.  No counterpart in the reference. */
#define GEMM_IPC_HANDLE_BYTES 64
int gemm_ipc_export(const void* ptr, void* handle, int64_t* offset);
int gemm_ipc_import(const void* handle, int64_t offset, void** ptr);
int gemm_ipc_close(void* ptr);

/* A reasonable configuration for a shape when no tuned entry exists.
 * No counterpart in the reference (its tuner had no per-shape dispatch). */
int gemm_default_cfg(int64_t M, int64_t N, int64_t K);

/* Reads and clears the device-side error word of `device` (synchronises
 * that device).  *code receives the OR of the kernels' error bits (0 = none).
 * Returns GEMM_OK, or GEMM_ERR_DEVICE_TIMEOUT when *code != 0.
 * No counterpart in the reference (C10_CUDA_KERNEL_LAUNCH_CHECK only,
 * src/gemm_ext.cpp:50). */
int gemm_device_error(int device, int* code);

/* Self-test of the kernels' bounded waits: launches one thread that waits on
 * an mbarrier nothing completes, gives up after limit_ns (<= 1 s) exactly as
 * the GEMM kernels' roles do, and sets an error bit in the device error word,
 * which the next gemm_device_error reports (GEMM_ERR_DEVICE_TIMEOUT) and
 * clears.  Synchronises the device; *waited_ns receives the time the wait
 * took.  No fault, trap or hang is involved, and the context stays usable.
 * No counterpart in the reference, which had no bounded waits. */
int gemm_selftest_wait_timeout(uint64_t limit_ns, uint64_t* waited_ns);

/* Size of the static scratch array behind gemm_launch_noalloc (32 MiB). */
#define GEMM_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* gemm_launch for callers that cannot allocate device memory: a runtime that
 * hands its operators only input/output pointers and a stream, or code that
 * shares the GPU with a framework whose allocator has reserved nearly all of
 * its memory (cudaMalloc would fail, fragment that pool, or synchronise the
 * device).  Same arguments and results as gemm_launch, minus the workspace:
 * split-K partials, tickets and repacked operands go to a file-scope
 * __device__ array of GEMM_NOALLOC_SCRATCH_BYTES that every GPU loading the
 * library keeps until exit.  A problem needing more scratch than that
 * (gemm_workspace_bytes) returns GEMM_ERR_WORKSPACE without launching.  The
 * first call on a device looks up the array's address (make it before any
 * stream capture); each call clears the ticket region on `stream`.  All
 * calls on a device share the array, so calls whose kernels overlap on the
 * GPU race; serialise them.  Nothing here calls cudaMalloc or cudaFree.
 * No counterpart in the reference. */
int gemm_launch_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                        int64_t ldb, int64_t ldc, int cfg_id, void* stream);

/* Message for the calling thread's last failing call ("" if none). */
const char* gemm_last_error(void);

/* Human-readable name of a status code. */
const char* gemm_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* INFINITE_DREAMS_GEMM_SM100_H_ */
