/*
 * bsattn.h -- C ABI of the B200 (sm_100a) block-sparse causal attention forward.
 *
 * This library replaces the Python/Triton entry point of sissississi-013/usagi:
 *
 *   block_sparse_attn_fwd(q, k, v, row_ptr, col_idx, seq_lens) -> (o, lse)
 *       kernels/v4_leaderboard_0740ms.py:242-243  (same in v7 :251-252, v1 :504-505)
 *   _run_csr(...)  host glue: flatten to [B*H, T, D], int32 metadata, grid launch
 *       kernels/v4_leaderboard_0740ms.py:143-179
 *   _fwd_csr(...)  the Triton device kernel
 *       kernels/v4_leaderboard_0740ms.py:31-136
 *   setup(suite_specs, device, variants)  precompiles Triton variants
 *       kernels/v4_leaderboard_0740ms.py:189-238  (nothing to precompile here: the kernel is
 *       built ahead of time for sm_100a; bsattn_setup only checks the device)
 *   PythonCudaLauncher.__call__  ctypes cuLaunchKernel launcher, RuntimeError on failure
 *       kernels/v1_baseline.py:75-130  (replaced by bsattn_fwd's own launch + return codes)
 *
 * Conventions
 *   - All tensor pointers are DEVICE pointers of the current CUDA device.
 *   - q, k, v, o are contiguous [B, H, T, D] with D == 128 and T % 128 == 0, 16-byte aligned.
 *   - row_ptr: int32, for head bh = b*H + h its nqb+1 offsets start at row_ptr + bh*rp_stride_bh
 *     (rp_stride_bh may be 0 to share one pattern across all heads).
 *   - col_idx: int32, head bh's column list starts at col_idx + bh*ci_stride_bh and holds
 *     max_nnz entries (ci_stride_bh may be 0).
 *   - seq_lens: int32 [B] valid length per batch entry, or NULL for "all T".
 *   - lse: float32 [B, H, T] natural-log logsumexp, or NULL to skip it.
 *   - stream: a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Calls are asynchronous on `stream`; nothing is allocated and nothing synchronises.
 *   - Functions return 0 on success or a negative BSATTN_E* code.
 */
#ifndef USAGI_B200_BSATTN_H
#define USAGI_B200_BSATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BSATTN_API __attribute__((visibility("default")))
#else
#define BSATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BSATTN_OK = 0,
  BSATTN_E_SHAPE = -1,      /* B, H, T or D out of range, T % 128 != 0, D != 128          */
  BSATTN_E_ALIGN = -2,      /* q/k/v/o not 16-byte aligned                                  */
  BSATTN_E_NULL = -3,       /* required pointer is NULL                                     */
  BSATTN_E_WORKSPACE = -4,  /* workspace NULL or smaller than bsattn_workspace_bytes()      */
  BSATTN_E_CUDA = -5,       /* CUDA runtime error (launch, attribute, device query)         */
  BSATTN_E_TMA = -6,        /* cuTensorMapEncodeTiled unavailable or failed                 */
  BSATTN_E_DEVICE = -7,     /* current device is not an sm_100 part                         */
  BSATTN_E_CSR = -8,        /* (device-reported) CSR row or column index out of range       */
  BSATTN_E_TIMEOUT = -9,    /* (device-reported) a pipeline wait exceeded its time limit    */
  BSATTN_E_DTYPE = -10,     /* unsupported dtype code                                       */
  BSATTN_E_PLAN = -11       /* work list does not match the call (or has an id out of range) */
};

/* dtype_flags of bsattn_fwd: element types of the inputs and of `o`, OR-ed together.
 *   BSATTN_OUT_F16 / BSATTN_OUT_BF16: o is fp16 / bf16 (the reference stored bf16, v4 :132, :152).
 *   BSATTN_IN_BF16: q and k are bf16 (the reference's input type, v4 :215); v is fp16 either way,
 *     because the reference multiplies fp16(P) by fp16(V) (v4 :103, :123) and one tensor-core MMA
 *     takes both operands in the same type.  bsattn_bf16_to_f16 converts a bf16 V. */
enum { BSATTN_OUT_F16 = 0, BSATTN_OUT_BF16 = 1, BSATTN_IN_BF16 = 2 };

/* Bytes of device workspace bsattn_fwd needs (error word, scheduler state). Zero it once
 * before first use (cudaMemset); the kernel leaves it ready for the next call. One workspace
 * per concurrently running stream. */
BSATTN_API size_t bsattn_workspace_bytes(void);

/* Forward pass: o = softmax(q k^T * scale, CSR block mask, causal diagonal) v.
 * Replaces block_sparse_attn_fwd / _run_csr / _fwd_csr (kernels/v4_leaderboard_0740ms.py:31-243).
 * scale <= 0 selects 1/sqrt(D) (the reference's fixed _SCORE_SCALE, v4 :19). */
BSATTN_API int bsattn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
               const int32_t* row_ptr, const int32_t* col_idx, const int32_t* seq_lens,
               int B, int H, int T, int D,
               int64_t rp_stride_bh, int64_t ci_stride_bh, int max_nnz,
               float scale, int dtype_flags,
               void* workspace, size_t workspace_bytes, void* stream);

/* bsattn_fwd with an optional work list (plan, device memory, from bsattn_plan for the same B, H,
 * T, row_ptr and seq_lens; plan_grid = the grid it was built for).  plan == NULL is bsattn_fwd.
 * Replaces the reference's fixed (qb, b*h) program grid (kernels/v4_leaderboard_0740ms.py:166-177)
 * with a persistent grid whose CTAs take balanced item lists.  A list that does not match the
 * call is reported as BSATTN_E_PLAN through bsattn_check_error and the kernel does no work. */
BSATTN_API int bsattn_fwd_plan(const void* q, const void* k, const void* v, void* o, float* lse,
                               const int32_t* row_ptr, const int32_t* col_idx,
                               const int32_t* seq_lens, int B, int H, int T, int D,
                               int64_t rp_stride_bh, int64_t ci_stride_bh, int max_nnz,
                               float scale, int dtype_flags, const int32_t* plan, int plan_grid,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Work list for bsattn_fwd_plan, built on the host (row_ptr and seq_lens are HOST arrays, laid
 * out as for bsattn_fwd).  Items are sorted by tile count, largest first, and dealt to `grid`
 * CTAs in snake order, which keeps every CTA within one item of the mean.  Build it once per
 * pattern, copy it to the device, reuse it.  bsattn_plan_bytes gives the size in bytes. */
BSATTN_API int bsattn_plan_bytes(int B, int H, int T, int grid, size_t* bytes);
BSATTN_API int bsattn_plan(const int32_t* row_ptr, int64_t rp_stride_bh, const int32_t* seq_lens,
                           int B, int H, int T, int max_nnz, int grid, int32_t* plan,
                           size_t plan_bytes);

/* Forward pass over analytic rows, with no row_ptr / col_idx: row i of every head lists the
 * first global_blocks blocks not covered by the window, then blocks max(0, i-window+1) .. i, so
 * it holds min(i + 1, global_blocks + window) blocks in ascending order, the diagonal last.
 * Replaces the reference's analytic kernels _fwd_window (global_blocks == 0,
 * kernels/v1_baseline.py:144-224) and _fwd_window_global (kernels/v1_baseline.py:227-322); the
 * result is bit-identical to bsattn_fwd_plan with the same rows as CSR (bsattn_build_csr with
 * BSATTN_CSR_WINDOW / BSATTN_CSR_PREFIX_WINDOW).  window >= 1, global_blocks >= 0.  plan may
 * come from bsattn_plan_window (or be NULL); the other arguments are those of bsattn_fwd_plan. */
BSATTN_API int bsattn_fwd_window(const void* q, const void* k, const void* v, void* o, float* lse,
                                 const int32_t* seq_lens, int B, int H, int T, int D, int window,
                                 int global_blocks, float scale, int dtype_flags,
                                 const int32_t* plan, int plan_grid, void* workspace,
                                 size_t workspace_bytes, void* stream);
/* Work list for bsattn_fwd_window (seq_lens is a HOST array or NULL). */
BSATTN_API int bsattn_plan_window(const int32_t* seq_lens, int B, int H, int T, int window,
                                  int global_blocks, int grid, int32_t* plan, size_t plan_bytes);

/* Allocation-free variant of bsattn_fwd.  No counterpart in the reference: its Python entry
 * point allocated outputs and metadata with torch on every call.
 *
 * For callers that cannot allocate device memory where they call attention (for example code
 * running inside an arena or pool it does not own, or a C caller without a CUDA allocator):
 * instead of a caller-provided workspace it uses a fixed 256-byte scratch array compiled into
 * the library, one per GPU, held until the process exits.  It calls no cudaMalloc, cudaFree or
 * other allocating routine.  The caller still provides q, k, v, o, lse and the CSR arrays, with
 * the same meaning and limits as bsattn_fwd; the scratch need does not depend on B, H or T, and
 * a build whose workspace would not fit the array is rejected with BSATTN_E_WORKSPACE.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress);
 *     make that first call before capturing `stream` into a CUDA graph.
 *   - Every call on a device shares the scratch.  Each call clears its error word on `stream`
 *     before the kernel; calls that overlap on the GPU (different streams) race on it.
 *   - status (optional, device or pinned host int*): receives 0, BSATTN_E_CSR or
 *     BSATTN_E_TIMEOUT for this call, written on `stream` after the kernel.  When the call
 *     itself returns non-zero (an argument or launch error), nothing was enqueued after the
 *     failure point and *status is left untouched. */
BSATTN_API int bsattn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                                  const int32_t* row_ptr, const int32_t* col_idx,
                                  const int32_t* seq_lens, int B, int H, int T, int D,
                                  int64_t rp_stride_bh, int64_t ci_stride_bh, int max_nnz,
                                  float scale, int dtype_flags, int* status, void* stream);

/* Reads and clears the device error word of `workspace` (synchronises `stream`).
 * *status receives 0, BSATTN_E_CSR or BSATTN_E_TIMEOUT. Replaces the RuntimeError the
 * reference's launcher raised on a failed launch (kernels/v1_baseline.py:126-128). */
BSATTN_API int bsattn_check_error(void* workspace, void* stream, int* status);

/* Checks that the current device can run the kernel and configures it (shared-memory
 * carve-out). Idempotent. Counterpart of setup() (kernels/v4_leaderboard_0740ms.py:189-238). */
BSATTN_API int bsattn_setup(void);

/* Upper bound on a pipeline wait inside the kernel, in nanoseconds (default 2e9).
 * A wait that exceeds it makes the kernel stop, free its tensor memory and report
 * BSATTN_E_TIMEOUT through bsattn_check_error. Applies to later launches in this process. */
BSATTN_API void bsattn_set_timeout_ns(uint64_t ns);

/* Test hook (no counterpart in the reference): while enabled, later launches make their
 * QK^T-issuing thread first wait on a barrier that nothing signals, so that the wait runs
 * into the bsattn_set_timeout_ns bound and the launch ends with BSATTN_E_TIMEOUT. Used to
 * test the timeout path on a GPU without faulting it. Off by default. */
BSATTN_API void bsattn_test_unsignalled_wait(int enable);

/* Converts n bf16 values at src to fp16 at dst (round to nearest even; exact for values inside
 * the fp16 range) on `stream`: the v.to(tl.float16) of the reference's P V product (v4 :103, :123)
 * done once per call instead of per tile.  n % 8 == 0; src and dst 16-byte aligned. */
BSATTN_API int bsattn_bf16_to_f16(const void* src, void* dst, int64_t n, void* stream);

/* CSR patterns built on the device.  No counterpart in the reference, which received row_ptr /
 * col_idx from its harness (kernels/v4_leaderboard_0740ms.py:242); these build the families the
 * harness used.  Every row is ascending and ends with its diagonal (v4 :78-86, :107).
 *   BSATTN_CSR_WINDOW         row i = max(0, i-window+1) .. i                      (prefix == 0)
 *   BSATTN_CSR_PREFIX_WINDOW  row i = {0 .. min(prefix-1, i)} U {max(0, i-window+1) .. i}
 *   BSATTN_CSR_RETRIEVAL      row i = {i-1, i} U min(n_random, i-1) distinct blocks of 0 .. i-2,
 *                             drawn from a counter-based generator keyed by (seed, head, row)
 * bsattn_csr_nnz gives the column count of one head (row_ptr[nqb]); col_idx rows are ci_stride
 * apart (ci_stride >= nnz), row_ptr is [n_heads, nqb + 1] contiguous.  The window families do not
 * depend on the head or the seed: build one head and share it (stride 0). */
enum { BSATTN_CSR_WINDOW = 0, BSATTN_CSR_PREFIX_WINDOW = 1, BSATTN_CSR_RETRIEVAL = 2 };
BSATTN_API int bsattn_csr_nnz(int kind, int nqb, int prefix, int window, int n_random,
                              int64_t* nnz);
BSATTN_API int bsattn_build_csr(int kind, int nqb, int prefix, int window, int n_random,
                                uint64_t seed, int n_heads, int32_t* row_ptr, int32_t* col_idx,
                                int64_t ci_stride, void* stream);

/* Peer-memory plumbing for gathering o shards onto one GPU (one process per GPU).  No counterpart
 * in the reference, which has no multi-GPU code.  The attention kernel is persistent and occupies
 * every SM, so a gather that runs while it computes must not need SMs: these let each rank copy
 * its finished heads straight into the root rank's output buffer with the copy engines (a DMA
 * over NVLink).
 *   bsattn_ipc_export: CUDA IPC handle (BSATTN_IPC_HANDLE_BYTES bytes into `handle`) of the
 *     allocation holding device pointer `ptr`, and ptr's byte offset inside that allocation.
 *   bsattn_ipc_open: maps an exported allocation into the CURRENT device's context (peer access
 *     enabled) and returns the mapped address of base + offset in *ptr; one open per handle and
 *     process.  bsattn_ipc_close takes that same pointer and the same offset.
 *   bsattn_peer_copy: enqueues a copy of `bytes` from src to dst on `stream` (either may be a
 *     mapped peer address); no SM work for a device-to-peer copy. */
#define BSATTN_IPC_HANDLE_BYTES 64
BSATTN_API int bsattn_ipc_export(const void* ptr, void* handle, uint64_t* offset);
BSATTN_API int bsattn_ipc_open(const void* handle, uint64_t offset, void** ptr);
BSATTN_API int bsattn_ipc_close(void* ptr, uint64_t offset);
BSATTN_API int bsattn_peer_copy(void* dst, const void* src, size_t bytes, void* stream);

/* Human-readable text for a BSATTN_E* code. */
BSATTN_API const char* bsattn_strerror(int code);

/* ABI version of this header (major*100 + minor): 102.  Minor 1 added dtype flags
 * (BSATTN_IN_BF16, bsattn_bf16_to_f16), work lists (bsattn_plan, bsattn_fwd_plan, BSATTN_E_PLAN)
 * and device-built CSR patterns (bsattn_build_csr); minor 2 the analytic window rows
 * (bsattn_fwd_window, bsattn_plan_window).  Every 100 call keeps its meaning. */
BSATTN_API int bsattn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* USAGI_B200_BSATTN_H */
