/*
 * arc_b200.h — C ABI of the B200 (sm_100a) GEMM library behind the `arc` Python API.
 *
 * The reference binds its GEMM through TVM-FFI: arc/mm.py:30 defines the typed
 * function `void matmul(TensorView a, TensorView b, TensorView out)` and arc/mm.py:48
 * exports it (`TVM_FFI_DLL_EXPORT_TYPED_FUNC(matmul, (arc::matmul))`, i.e. the C symbol
 * `__tvm_ffi_matmul`). Its A8W4 role is the third-party call
 * `deep_gemm.fp8_fp4_gemm_nt((a, sa), (b, sb), out, recipe_a, recipe_b)` at
 * tests/a8w4.py:48 and :70. This header replaces both with plain C entry points:
 * raw device pointers, sizes and a CUDA stream, no framework types.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers of the current CUDA device; the caller owns
 *     every buffer (the reference allocates `out` in Python, arc/mm.py:76-77). The
 *     fused all-gather calls are the exception: they also take other GPUs' buffers,
 *     mapped into this process with arc_ipc_open.
 *   - Work is enqueued on `stream` and the call returns without synchronising, as the
 *     reference launches on the caller's stream (arc/mm.py:38,44).
 *   - The return value is an arc_status_t. Where the reference would exit() the
 *     process on a CUDA error (arc/include/common.cuh:8-28) or raise an
 *     AssertionError on a bad shape (arc/mm.py:74-75), these calls return a nonzero
 *     status instead; arc_last_error() holds a one-line description for the calling
 *     thread.
 *   - Kernels never wait without a bound: a pipeline wait that exceeds 2 s records a
 *     bit in a per-device status word (read with arc_device_status()) and the kernel
 *     returns.
 *   - Nothing here allocates device memory (arc_ipc_open maps a peer's existing
 *     allocation; it allocates none).
 */
#ifndef ARC_B200_H_
#define ARC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *cudaStream_t;

typedef enum arc_status {
  ARC_OK = 0,
  ARC_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, K mismatch */
  ARC_ERR_UNSUPPORTED = 2,      /* shape/alignment/recipe outside what the kernels cover */
  ARC_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed */
  ARC_ERR_NO_DEVICE = 4,        /* no sm_100 device is current */
  ARC_ERR_DEVICE_TIMEOUT = 5    /* a kernel abandoned a wait (see arc_device_status) */
} arc_status_t;

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int arc_version(void);

/* Static string for a status code. */
const char *arc_status_string(int status);

/* Description of the last failure on the calling thread ("" if none). */
const char *arc_last_error(void);

/*
 * bf16 GEMM, C[M,N] = A[M,K] . B[N,K]^T with fp32 accumulation and bf16 output.
 * Replaces: arc/mm.py:30-45 (`arc::matmul` host shim, exported at arc/mm.py:48) and
 * the kernel arc/include/mm.cuh:31-216.
 * A, B, C: bf16 (uint16 storage), row-major with leading dimensions lda >= K,
 * ldb >= K, ldc >= N in elements. Requirements: M, N, K >= 1; base pointers 16-byte
 * aligned; lda, ldb, ldc multiples of 8. (The reference additionally requires
 * M % 32 == 0, N % 128 == 0, K % 128 == 0, arc/mm.py:75; those shapes are a subset.)
 */
int arc_matmul_bf16(const void *A, const void *B, void *C, int M, int N, int K, int lda,
                    int ldb, int ldc, cudaStream_t stream);

/*
 * A8W4 GEMM: int8 activations x packed int4 weights with K-group scales.
 *   P[m,n,g] = sum_{k in group g} A[m,k] * W[n,k]                  (int32, exact)
 *   C[m,n]   = bf16( sa[m] * sum_g f32(sb[n,g]) * P[m,n,g] )
 * Replaces the A8W4 call of the reference, deep_gemm.fp8_fp4_gemm_nt at
 * tests/a8w4.py:48 / :70 (same NT layout and (data, scale) pairing), with the
 * int8 x int4 recipe.
 *   A    [M][K]      int8, contiguous
 *   sa   [M]         fp32 per-token scale
 *   Wp   [N][K/2]    uint8; byte j of a row holds w[2j] in bits 3:0 and w[2j+1] in
 *                    bits 7:4, each a two's-complement int4 (the nibble order of
 *                    arc/testing/quant.py:82-83)
 *   sb   [N][K/group] bf16 (uint16 storage)
 *   C    [M][N]      bf16 (uint16 storage)
 *   partials_dbg     NULL, or [M][N][K/group] int32 that receives every P[m,n,g]
 *                    (a slow debugging mode for bit-exact checks)
 * Requirements: group == 128; K % 128 == 0; M, N >= 1; N % 8 == 0; A, Wp, C 16-byte
 * aligned.
 */
int arc_a8w4_gemm(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                  uint16_t *C, int M, int N, int K, int group, cudaStream_t stream,
                  int32_t *partials_dbg);

/*
 * arc_a8w4_gemm with flags (the reference's call has none; same role, tests/a8w4.py:48).
 *   ARC_A8W4_PREPACKED       Wp is in the layout of arc_a8w4_prepack_weights (no partials
 *                            dump then).
 *   ARC_A8W4_STATIC_WEIGHTS  Wp and sb are not written by the kernel that directly precedes
 *                            this call on `stream`. Every A8W4 kernel is launched with
 *                            programmatic dependent launch: it may start while the
 *                            preceding kernel still runs and reads A and sa, and writes C,
 *                            only after that kernel has completed. With this flag the
 *                            decode kernel (M <= 32) also streams and unpacks Wp and sb
 *                            before that point, so consecutive GEMMs on one stream overlap
 *                            their weight traffic. Weights written by any earlier work
 *                            (an upload, a copy, a kernel before the preceding one) are
 *                            fine. Without the flag nothing is read before the preceding
 *                            kernel completes.
 */
#define ARC_A8W4_PREPACKED 1u
#define ARC_A8W4_STATIC_WEIGHTS 2u
int arc_a8w4_gemm_ex(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                     uint16_t *C, int M, int N, int K, int group, unsigned flags, cudaStream_t stream,
                     int32_t *partials_dbg);

/*
 * Weight pre-pack (no reference counterpart: the reference stores weights only in the
 * packing of arc/testing/quant.py:82-83, which Wp above follows). Reorders the nibbles
 * inside every 16-byte piece of Wp [N][K/2] (32 codes, k = 32q .. 32q+31) so that byte j
 * holds code 32q+j in bits 3:0 and code 32q+j+16 in bits 7:4. Shape, size and strides
 * are unchanged. Wq may be Wp itself (in place); any other overlap is rejected. Runs on
 * `stream`, reading and writing N*K/2 bytes once. Requirements: K % 32 == 0; Wp, Wq
 * 16-byte aligned.
 */
int arc_a8w4_prepack_weights(const uint8_t *Wp, uint8_t *Wq, int N, int K, cudaStream_t stream);

/*
 * arc_a8w4_gemm on weights in the pre-packed layout (arc_a8w4_prepack_weights). Same
 * arithmetic, results bit-identical to arc_a8w4_gemm on the original Wp; the kernels'
 * int4 -> int8 expansion is a mask and shift instead of byte permutes. No partials dump.
 */
int arc_a8w4_gemm_prepacked(const int8_t *A, const float *sa, const uint8_t *Wq, const uint16_t *sb,
                            uint16_t *C, int M, int N, int K, int group, cudaStream_t stream);

/* The work decomposition arc_a8w4_gemm picks for a shape (host-only, no GPU needed). */
typedef struct arc_a8w4_plan {
  int split;        /* 1: K-split clusters with on-chip reduction; 0: persistent tiles */
  int token_tile;   /* tokens (rows of A) per tile: 16, 32, 64 or 128 */
  int weight_rows;  /* weight rows (output columns) per tile: 128 */
  int k_split;      /* CTAs per cluster along K (split == 1) */
  int grid;         /* CTAs launched */
  int load_stages;  /* depth of the TMA ring */
  int groups_per_stage; /* K-groups fetched per ring stage */
} arc_a8w4_plan_t;

int arc_a8w4_describe_plan(int M, int N, int K, int num_sms, arc_a8w4_plan_t *plan);

/*
 * A8W4 decode GEMM with the all-gather of its output fused into the epilogue (the
 * multi-GPU step after the reference's single-GPU call, tests/a8w4.py:48: one process
 * per GPU, weight columns sharded). Rank `rank` of `world` (<= 8) holds the weight
 * columns [rank*N, (rank+1)*N) (Wp [N][K/2], sb [N][K/128]); outs[i] is rank i's full
 * output [M][world*N] bf16, mapped into this process (CUDA IPC). Every output tile is
 * stored by TMA straight into all `world` outputs over NVLink, so no separate gather
 * runs. Decode batches only (1 <= M <= 32); other arguments as arc_a8w4_gemm. The
 * other ranks' writes into this rank's output are complete only after
 * arc_peer_barrier; a call overwrites the output of the previous one on every rank.
 */
int arc_a8w4_gemm_gather(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                         uint16_t *const *outs, int world, int rank, int M, int N, int K,
                         cudaStream_t stream);

/*
 * The fused all-gather GEMM and its barrier in ONE launch (no reference counterpart: the
 * reference is single-GPU; the call shape is still tests/a8w4.py:48's, per rank). Same as
 * arc_a8w4_gemm_gather_ex followed by arc_peer_barrier on the same flag arrays, except that
 * the kernel's last CTA to finish runs the barrier, so the step costs one launch. flags[i]
 * is rank i's flag array of world + 2 uint32 words, zeroed once: the world epochs and the
 * barrier count of arc_peer_barrier, then a count of finished CTAs that the kernel leaves
 * at zero. The wait for the peers gives up after 2 s and reports kStatusTimeoutPeer through
 * arc_device_status. Every rank must make the same sequence of calls.
 */
int arc_a8w4_gemm_gather_sync(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                              uint16_t *const *outs, uint32_t *const *flags, int world, int rank, int M,
                              int N, int K, unsigned gemm_flags, cudaStream_t stream);

/* arc_a8w4_gemm_gather with the flags of arc_a8w4_gemm_ex (ARC_A8W4_STATIC_WEIGHTS; the
 * fused gather takes weights in the reference packing only). */
int arc_a8w4_gemm_gather_ex(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                            uint16_t *const *outs, int world, int rank, int M, int N, int K,
                            unsigned flags, cudaStream_t stream);

/*
 * Stream-ordered barrier of the ranks of a fused all-gather. flags[i] is rank i's array
 * of world + 1 uint32 words, zeroed once and mapped into this process: words 0..world-1
 * hold the last epoch each rank announced, word `world` counts the barriers rank i has
 * passed. The call takes this rank's next epoch from its counter, announces it in every
 * rank's array and waits on `stream` until this rank's array holds that epoch from every
 * rank. Every rank must call it the same number of times. The epoch is kept in device
 * memory, so a CUDA graph that captured the call replays correctly. The wait gives up
 * after 2 s and reports it through arc_device_status.
 */
int arc_peer_barrier(uint32_t *const *flags, int world, int rank, cudaStream_t stream);

/* arc_peer_barrier with the bound of its wait given in nanoseconds (0 < timeout_ns <= 2 s):
 * a barrier whose peers have not announced within it sets the kStatusTimeoutPeer bit
 * (1 << 6) of arc_device_status and returns. Where the reference would exit() on a failed
 * CUDA call (arc/include/common.cuh:8-28), a missing peer is reported here. */
int arc_peer_barrier_ex(uint32_t *const *flags, int world, int rank, uint64_t timeout_ns,
                        cudaStream_t stream);

/*
 * CUDA IPC for the buffers of a fused all-gather (no reference counterpart: the reference
 * is single-GPU). arc_ipc_export writes the ARC_IPC_HANDLE_BYTES-byte handle of the
 * device allocation that holds `ptr` and ptr's byte offset inside it. arc_ipc_open maps a
 * handle exported by ANOTHER process into the CURRENT device's context (make the GPU
 * whose kernels will access the buffer current first), enabling peer access from it to
 * the owner's GPU; *ptr = mapping + offset, *base is what arc_ipc_close takes. A process
 * opens each handle once; the owner frees the allocation only after every importer
 * closed it.
 */
#define ARC_IPC_HANDLE_BYTES 64
int arc_ipc_export(const void *ptr, void *handle, uint64_t *offset);
int arc_ipc_open(const void *handle, uint64_t offset, void **ptr, void **base);
int arc_ipc_close(void *base);

/*
 * FP8 x FP4 GEMM with UE8M0 block scales, the recipe of the reference's A8W4 test
 * (tests/a8w4.py:29-30 quantisation, :48 the deep_gemm.fp8_fp4_gemm_nt call with
 * recipe_a = (1, 128), recipe_b = (1, 32)):
 *   C[m,n] = bf16( sum_k A[m,k] sfa[m,k/128] * W[n,k] sfw[n,k/32] )   (fp32 accumulate)
 *   A    [M][K]      float8 e4m3 (uint8 storage), contiguous
 *   sfa  [M][K/128]  fp32 powers of two (UE8M0 values)
 *   Wp   [N][K/2]    uint8, two e2m1 codes per byte (magnitude index | sign << 3), the even
 *                    k in the low nibble (arc/testing/quant.py:51-84)
 *   sfw  [N][K/32]   fp32 powers of two
 *   C    [M][N]      bf16 (uint16 storage)
 * Requirements: K % 128 == 0; N % 8 == 0; M, N >= 1; A, C, sfw 16-byte aligned, Wp
 * 32-byte aligned, sfa 4-byte aligned. Large problems with K % 512 == 0 and a 16-byte
 * aligned sfa run on CTA pairs.
 */
int arc_fp8_fp4_gemm(const uint8_t *A, const float *sfa, const uint8_t *Wp, const float *sfw,
                     uint16_t *C, int M, int N, int K, cudaStream_t stream);

/*
 * The same GEMM with a caller-owned workspace, which lets problems with fewer 128 x 128
 * output tiles than SMs (decode batches) split K over several CTAs per tile: each writes
 * an fp32 partial into the workspace and the last one of a tile sums them in a fixed
 * order (results do not depend on timing) and stores the tile. Same role and call shape
 * as arc_fp8_fp4_gemm (tests/a8w4.py:48); the workspace has no counterpart there.
 *   workspace   256-byte aligned device memory of at least
 *               arc_fp8_fp4_workspace_bytes(M, N, K) bytes, all ZERO before its first use;
 *               every call leaves it ready for the next (its tile counters back at zero)
 *               unless a kernel wait timed out (arc_device_status), after which it must be
 *               zeroed again. Calls that share a workspace must not run concurrently.
 *   A NULL or too small workspace runs the GEMM without the K split.
 */
int arc_fp8_fp4_gemm_ws(const uint8_t *A, const float *sfa, const uint8_t *Wp, const float *sfw,
                        uint16_t *C, int M, int N, int K, void *workspace, size_t workspace_bytes,
                        cudaStream_t stream);

/* Workspace bytes arc_fp8_fp4_gemm_ws uses for this shape on the current device (0: no
 * K split for it). */
int arc_fp8_fp4_workspace_bytes(int M, int N, int K, size_t *bytes);

/*
 * The FP8 x FP4 GEMM of arc_fp8_fp4_gemm_ws for callers that cannot allocate device
 * memory: no cudaMalloc, cudaFree or allocating routine is called. It has no counterpart
 * in the reference. Callers who need it: operator plugins whose host framework budgets
 * all device memory itself and hands the operator only its input and output tensors,
 * and hosts that must not call cudaMalloc on the request path (it may synchronise the
 * device and its latency is unbounded). Operands and output are the caller's, as in
 * arc_fp8_fp4_gemm. The K split of decode-sized problems keeps its partials and tile
 * counters in a 4 MiB array built into the library, which every GPU that loads the
 * library holds until the process exits; shapes whose split would need more than that
 * (4096 + S*M*N*4 bytes, S the split count) run without the split, like
 * arc_fp8_fp4_gemm. Every argument is checked before anything is enqueued. The first
 * call on a device looks up that device's address of the array (cudaGetSymbolAddress)
 * and should come before any stream capture. Every call uses the same array and clears
 * its counters on `stream` first, so calls whose kernels overlap on the GPU (other
 * streams, other host threads) race and give wrong results: issue them in one stream
 * order.
 */
int arc_fp8_fp4_gemm_noalloc(const uint8_t *A, const float *sfa, const uint8_t *Wp, const float *sfw,
                             uint16_t *C, int M, int N, int K, cudaStream_t stream);

/*
 * Per-token int8 quantisation of bf16 activations, the producer of the A8W4 GEMM's
 * activation operand:
 *   amax[m] = max(max_k |x[m,k]|, 1e-4),  sa[m] = amax[m] / 127  (fp32),
 *   q[m,k]  = clamp(round_half_even(x[m,k] / sa[m]), -127, 127)  (int8).
 * Replaces the role of the reference's per-token activation cast
 * (arc/testing/quant.py:30-48, per_token_cast_to_fp8) for the int8 recipe; results
 * equal the host quantizer arc.quant.per_token_cast_to_int8 bit for bit.
 *   x  [M][ldx] bf16 (uint16 storage), q [M][ldq] int8, sa [M] fp32.
 * Requirements: M, K >= 1; ldx, ldq >= K; x 2-byte and sa 4-byte aligned (16-byte
 * aligned rows with K, ldx, ldq multiples of 8 take the vector path).
 */
int arc_quantize_int8(const void *x, int8_t *q, float *sa, int M, int K, int ldx, int ldq,
                      cudaStream_t stream);

/*
 * Probe builds only (libarcb200_probe.so, compiled with -DARC_PROBE and loaded by the
 * Python package when the ARC_PROBE environment variable is set). Attaches a device
 * buffer of at least 64 uint64 per CTA; every kernel launched afterwards on the
 * current device writes %clock64 stamps (SM cycles, comparable within one CTA) of
 * its pipeline milestones into buffer[blockIdx.x * 64 + slot]. NULL detaches. Replaces the reference's probe mode
 * (arc/mm.py:60-65, arc/include/common.cuh:30-39, stamps printed at
 * arc/include/mm.cuh:201-211). Returns ARC_ERR_UNSUPPORTED in regular builds.
 */
int arc_probe_attach(void *buffer, size_t bytes);

/*
 * Name of the kernel the library launches for an operation of this shape on the
 * current device (op: ARC_OP_MATMUL_BF16, ARC_OP_A8W4 or ARC_OP_FP8_FP4; the FP8 x FP4
 * answer assumes a 16-byte aligned sfa), e.g. "gemm_bf16_pair_kernel", written into
 * name[0..len). The shape is not checked beyond what the choice needs; the
 * ARC_BF16_CTAS / ARC_FP8FP4_KERNEL overrides apply. The reference has one kernel per
 * operation, so it has no counterpart; this serves profiling (matching ncu launch lists).
 */
#define ARC_OP_MATMUL_BF16 0
#define ARC_OP_A8W4 1
#define ARC_OP_FP8_FP4 2
int arc_kernel_name(int op, int M, int N, int K, char *name, int len);

/*
 * Device status word of `device`: a bit mask of the pipeline waits that timed out
 * since it was last cleared (0 = healthy). Synchronises the device. When `clear`
 * is nonzero the word is reset to 0 after reading.
 */
int arc_device_status(int device, uint32_t *status, int clear);

#ifdef __cplusplus
}
#endif

#endif /* ARC_B200_H_ */
