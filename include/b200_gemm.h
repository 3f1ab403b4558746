/*
 * b200_gemm.h - C ABI of the B200 (sm_100a) FP16 GEMM library
 * (libb200gemm.so).  Plain pointers, sizes and a stream handle; no C++ or
 * torch types, so it binds from ctypes, cffi, cgo or JNI alike.
 *
 * Numerics: C = A * B with fp16 inputs, an fp32 accumulator and one
 * round-to-nearest-even conversion to fp16 per output element (alpha = 1,
 * beta = 0), the arithmetic of the reference kernels' epilogue
 * (tensorcore_gemm/gemm.cu:1360-1361).
 *
 * Layouts (all row-major with a leading dimension in ELEMENTS):
 *   A  M x K, element (i, k) at A[i * lda + k]
 *   B  b_layout = B200_B_ROW_MAJOR: K x N, element (k, j) at B[k * ldb + j]
 *      b_layout = B200_B_COL_MAJOR: stored N x K ("colb", pre-transposed),
 *                 element (k, j) at B[j * ldb + k]
 *   C  M x N, element (i, j) at C[i * ldc + j]
 *
 * Requirements (TMA): every base pointer 16-byte aligned and every leading
 * dimension a multiple of 8 elements (16 bytes).  Any M, N, K >= 0 is
 * accepted; no M/N/K divisibility is required.
 */
#ifndef B200_GEMM_H_
#define B200_GEMM_H_

#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B200_B_ROW_MAJOR 0
#define B200_B_COL_MAJOR 1

#define B200_A_ROW_MAJOR 0 /* A stored M x K, element (i, k) at A[i * lda + k] */
#define B200_A_COL_MAJOR 1 /* A stored K x M, element (i, k) at A[k * lda + i] */

/* Return codes. */
#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad layout, ld too small */
#define B200_ERR_MISALIGNED 2       /* base pointer not 16 B aligned or ld not a multiple of 8 */
#define B200_ERR_TOO_LARGE 3        /* a dimension beyond 2^31 - 1 */
#define B200_ERR_CUDA 4             /* a CUDA runtime call or the kernel launch failed */
#define B200_ERR_TENSOR_MAP 5       /* cuTensorMapEncodeTiled unavailable or rejected the map */
#define B200_ERR_DEVICE 6           /* the device error word was set (a bounded wait timed out) */
#define B200_ERR_UNSUPPORTED_DEVICE 7 /* current device is not sm_100 */
#define B200_ERR_WORKSPACE 8        /* workspace missing, too small or not 256-byte aligned */
#define B200_ERR_SCRATCH_LIMIT 9    /* b200_gemm_f16_noalloc: more scratch needed than it has */

/*
 * C = A * B on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Asynchronous: returns after the launch.  Replaces the reference's native
 * entry `root_gemm_cuda(A, B, mode)` (tensorcore_gemm/gemm.py:32-153): mode
 * ids 2/3 there are b_layout = B200_B_ROW_MAJOR here, mode ids 4/5
 * (`use_colb`, gemm.py:43) are B200_B_COL_MAJOR.  Unlike the reference the
 * caller owns C (the reference allocated it with torch::empty, gemm.py:61).
 */
B200_API int b200_gemm_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                  int64_t ldb, int64_t ldc, int b_layout, void* stream);

/*
 * Operands that TMA cannot address directly (a base pointer not 16-byte
 * aligned, or a leading dimension that is not a multiple of 8 elements --
 * e.g. K or N odd) are handled by this pair of calls.  The reference accepted
 * such shapes only through its torch.matmul fallback (tensorcore_gemm/gemm.py
 * :185-192, 219-221) and ran them out of bounds through gemm_pretransposed
 * (gemm.py:209-216).
 *
 * b200_gemm_workspace_size returns the device workspace in bytes that
 * b200_gemm_f16_ws needs for these operands (0 when every operand is already
 * TMA-compatible), or a negative B200_ERR_* code.  b200_gemm_f16_ws copies each
 * incompatible operand into the workspace with a 16-byte row pitch, multiplies,
 * and copies C back when C itself was incompatible; all on `stream`.  The
 * workspace must be 256-byte aligned device memory of at least that size and
 * must not be reused until the call's work on `stream` has finished.
 */
B200_API int64_t b200_gemm_workspace_size(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                                          int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int b_layout);
B200_API int b200_gemm_f16_ws(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                              int64_t ldb, int64_t ldc, int b_layout, void* workspace, int64_t workspace_bytes,
                              void* stream);

/*
 * Allocation-free variant of b200_gemm_f16_ws.  No counterpart in the
 * reference.  For callers that must not allocate device memory: code whose
 * device memory belongs to a host framework's pool or arena that forbids side
 * allocations, and latency-critical paths that cannot take cudaMalloc's
 * implicit device synchronisation.  Operands that need re-pitching are copied
 * into a fixed 32 MiB scratch array compiled into this library (every GPU that
 * loads the library keeps it until the process exits); the call itself
 * allocates nothing.  Every tile runs whole: the split of a partial last wave
 * along K that b200_gemm_f16 may use (its partial sums go to a per-stream
 * workspace allocated on first use) is never taken here, so deep-K shapes with
 * a thin last wave can run a few percent slower than through b200_gemm_f16.
 * The first launch of each kernel variant in a process may load that kernel's
 * code onto the device (CUDA's lazy module loading); that is the driver's
 * doing, not an allocation by this call.  Returns B200_ERR_SCRATCH_LIMIT when the re-pitched
 * operands (b200_gemm_workspace_size) would exceed 32 MiB; operands that need
 * no re-pitch are not limited.
 *
 * The first call on a device looks up the scratch array's device address
 * (once per device); make that first call before any stream capture.  All
 * calls share the one array and it keeps the last call's contents, so calls
 * whose work overlaps on the GPU (other streams, other host threads) race on
 * it: order them on one stream or synchronise between them.
 */
B200_API int b200_gemm_f16_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                   int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* stream);

/*
 * General form: C = alpha * A * B + beta * C, with either layout for A and
 * for B, and an optional workspace for operands TMA cannot address (sized by
 * b200_gemm_workspace_size_ex; NULL / 0 when none is needed).  alpha and beta
 * are the reference kernels' epilogue parameters (tensorcore_gemm/gemm.cu
 * :1073 signature, epilogue :1360-1364: fp16_rn(alpha * acc) when beta == 0,
 * else fp16_rn(alpha * acc + beta * C_old)); the reference launcher fixed them
 * to 1 and 0 (gemm.py:87).  A column-major A (a transposed view of a K x M
 * buffer) is read in place; the reference made such inputs contiguous first
 * (gemm.py:213-225).  With beta != 0, C must hold the old values on entry.
 */
B200_API int b200_gemm_f16_ex(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                              int64_t ldb, int64_t ldc, int a_layout, int b_layout, float alpha, float beta,
                              void* workspace, int64_t workspace_bytes, void* stream);
B200_API int64_t b200_gemm_workspace_size_ex(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                                             int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int a_layout,
                                             int b_layout);

/*
 * K-means assignment fused into the skinny GEMM (the consumer the reference's
 * K = 256 "K-means-like" shapes stand for, README.md:44): for every point
 * (row of X, M x K) the index of the centroid minimising
 * score_j = ||c_j||^2 - 2 x . c_j  (= ||x - c_j||^2 - ||x||^2), without
 * writing the M x N product.  Centroids are K x N row-major
 * (cent_layout = B200_B_ROW_MAJOR) or stored N x K (B200_B_COL_MAJOR).
 * 1 <= K <= 256; X and Cent TMA-compatible (16-byte bases, pitches multiple
 * of 8).  Ties go to the smaller index.  out_score (optional) receives the
 * winning score.  The workspace (b200_kmeans_workspace_size bytes, 256-byte
 * aligned) holds the centroid norms and per-point keys.  No counterpart in
 * the reference, which stops at the GEMM.
 */
B200_API int64_t b200_kmeans_workspace_size(int64_t M, int64_t N);
B200_API int b200_kmeans_assign_f16(const void* X, const void* Cent, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                    int64_t ldcent, int cent_layout, void* workspace, int64_t workspace_bytes,
                                    int32_t* out_idx, float* out_score, void* stream);

/*
 * Gathered output: C = A * B for this rank's row shard, where every finished
 * C block is written both to C (this GPU's copy of the gathered matrix, at
 * the shard's first row) and to each of the `n_peers` (<= 7) buffers in
 * peer_c -- the other GPUs' copies, mapped into this process by
 * b200_ipc_open, each pointer at the same shard offset, all with pitch ldc.
 * The all-gather of C so runs tile by tile under the GEMM, as plain 16-byte
 * stores over NVLink.  The reference has no multi-GPU code; this is the
 * fused form of its optional gathered-output step (a GEMM followed by an
 * all-gather of the C shards).  Operands must be TMA-compatible as given
 * (B200_ERR_MISALIGNED otherwise).  The kernel never waits on a peer: when
 * the call's work on `stream` is done, this rank's stores are visible to
 * every peer; the caller synchronises the ranks (a device-side barrier such
 * as a one-element NCCL all-reduce on the same stream) before any rank reads
 * the rows that others wrote.
 */
B200_API int b200_gemm_f16_gather(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                  int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* const* peer_c,
                                  int n_peers, void* stream);

/*
 * Device buffers shareable across processes (legacy CUDA IPC), for the
 * gathered output above.  b200_ipc_alloc allocates `bytes` on the current
 * device and writes its b200_ipc_handle_size()-byte handle; another process
 * maps it with b200_ipc_open and unmaps it with b200_ipc_close; the owner
 * frees it with b200_ipc_free after every peer has closed it.  No multicast
 * object is created.  No counterpart in the reference.
 */
B200_API int b200_ipc_handle_size(void);
B200_API int b200_ipc_alloc(int64_t bytes, void** ptr, void* handle);
B200_API int b200_ipc_free(void* ptr);
B200_API int b200_ipc_open(const void* handle, void** ptr);
B200_API int b200_ipc_close(void* ptr);

/* Human-readable text of a return code (static storage). Counterpart of the
 * TORCH_CHECK messages of the reference launcher (gemm.py:33-47, 150-152). */
B200_API const char* b200_gemm_strerror(int code);

/* Reads and clears the device error word of the current device (0 = none;
 * see DeviceError in csrc/sm100_ptx.cuh).  Synchronises the device.  No
 * counterpart in the reference, whose kernels have no bounded waits. */
B200_API int b200_gemm_last_device_error(void);

/* Number of SMs the persistent scheduler launches on for the current device
 * (0 on error).  No counterpart in the reference. */
B200_API int b200_gemm_sm_count(void);

/* Kernel variants for b200_gemm_set_variant. */
#define B200_VARIANT_AUTO 0 /* shape heuristic (default) */
#define B200_VARIANT_CTA1 1 /* 1-CTA persistent kernel, 128 x 256 tiles */
#define B200_VARIANT_PAIR 2 /* 2-CTA cluster (cta_group::2) kernel, 256 x 256 tiles */
#define B200_VARIANT_SKINNY 3 /* K <= 256: B slice resident in shared memory, A streamed */
#define B200_VARIANT_PAIR_WIDE 4 /* 2-CTA cluster kernel, 512 x 256 tiles (B reused by two MMAs) */
#define B200_VARIANT_PAIR_WIDE_224 5 /* the same kernel with 512 x 224 tiles */
#define B200_VARIANT_PAIR_WIDE_192 6 /* the same kernel with 512 x 192 tiles */

/* Process-wide override of the kernel the library picks, for tests and
 * tuning; every variant computes the same product.  Returns
 * B200_ERR_INVALID_ARGUMENT for an unknown variant.  No counterpart in the
 * reference (its mode string chose among kernels; here the mode only selects
 * the B layout). */
B200_API int b200_gemm_set_variant(int variant);

/* The launch plan the library would use for an M x N x K product on a GPU
 * with `sm_count` SMs (assuming sm_count / 2 resident 2-CTA clusters): the
 * kernel variant (B200_VARIANT_*, honouring b200_gemm_set_variant) and, for
 * B200_VARIANT_PAIR, the number of K ranges its partial last wave is split
 * into (1 = none).  Host-only: touches no GPU.  No counterpart in the
 * reference, whose mode string chose the kernel. */
B200_API int b200_gemm_plan(int64_t M, int64_t N, int64_t K, int sm_count, int* variant, int* k_ranges);

/* Self-test of the kernels' failure path: launches one thread that waits on
 * a barrier nothing arrives at, with a bounded wait of `limit_ns`
 * (1 ns .. 1 s), on the legacy default stream of the current device.  The
 * wait gives up, records cause 5 in the device error word and the kernel
 * returns; the context stays usable.  Returns the error word it read (5 when
 * the bounded wait works; the word is cleared again), or a negative
 * B200_ERR_* code.  No counterpart in the reference. */
B200_API int b200_gemm_selftest_bounded_wait(int64_t limit_ns);

/* Self-test of the split last wave's failure path: runs C = A * B (A M x K,
 * B K x N row-major, C M x N, dense pitches) on the 256 x 256 pair kernel
 * with its last wave split along K, but the last unit of each split tile
 * issues none of its loads of the other K ranges' parts, so its bounded wait
 * (`limit_ns`, 1 ns .. 1 s) runs out.  Those tiles are then left unstored
 * (C keeps what it held there), the device error word records cause 6, and
 * the context stays usable.  Synchronises; returns the error word it read
 * (6 when the path works; the word and the tail counters are cleared again),
 * or a negative B200_ERR_* code (-B200_ERR_INVALID_ARGUMENT when the shape's
 * pair launch has no split last wave, e.g. 2560 x 2048 x 8192 does).  No
 * counterpart in the reference. */
B200_API int b200_gemm_selftest_split_fixup(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                            int64_t limit_ns, void* stream);

/* Library ABI version (major * 100 + minor). */
B200_API int b200_gemm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B200_GEMM_H_ */
