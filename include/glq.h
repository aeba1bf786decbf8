/*
 * glq.h -- C ABI of the B200 (sm_100a) linear fragment library, libglq.so.
 *
 * The library computes the FP16/BF16 linear fragment of the GEMM lab:
 *
 *     Y[m, n] = epilogue( sum_k A[m, k] * B[k, n] )        (FP32 accumulate)
 *
 * where B is the lab's [K, N] operand.  A weight matrix stored the way a
 * linear layer stores it, W[N, K] row-major (K-contiguous), is the B operand
 * viewed as W^T, i.e. b_k_stride = 1 and b_n_stride = ldw.  That K-contiguous
 * view is the primary fast layout; the lab's own B[K, N] row-major layout
 * (b_k_stride = N, b_n_stride = 1) is accepted through the same entry point.
 *
 * Every entry point is stateless apart from a per-device one-time set-up
 * (kernel attributes, the TMA encoder entry point) and the shared counter
 * array of glq_linear_gather_static, thread-safe, stream-ordered
 * on the caller's stream, never allocates device memory and never throws
 * across the boundary: each returns a glq_status.  All pointers are device
 * pointers unless stated otherwise.  `stream` is a cudaStream_t (NULL is the
 * legacy default stream).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   - gemm_lab::launch_* (csrc/ptx_mma.cuh:220,772,796,827,931,978,1031):
 *     void launch_X(const T* a, const T* b, T* c, int m, int n, int k,
 *                   cudaStream_t) with B = [K, N] row-major.
 *   - gemm_lab::launch_ptx_mma_splitk (csrc/ptx_mma.cuh:931-965) and
 *     ptx_mma_splitk_workspace_bytes (csrc/ptx_mma.cuh:926-929).
 *   - The Triton operator bodies of kernels.py (triton_matmul_into
 *     kernels.py:148-171, triton_bias_silu_into kernels.py:252-280,
 *     triton_splitk_matmul_into kernels.py:396-441) that the Python binding
 *     of this library re-exports under the same names.
 *   - Error convention: GEMM_LAB_CUDA_CHECK (include/gemm_lab/cuda_check.hpp:
 *     39-65) throws std::runtime_error; here the same failures are returned
 *     as status codes and glq_status_string() gives the text.
 */
#ifndef GLQ_H_
#define GLQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLQ_ABI_VERSION 3

/* Element types (inputs, bias and output share one type). */
enum glq_dtype {
  GLQ_DTYPE_F16 = 0,
  GLQ_DTYPE_BF16 = 1
};

/* Epilogue applied in FP32 before the single store of Y.
 * GLQ_EPILOGUE_BIAS_SILU is y = v * sigmoid(v), v = acc + bias[n]
 * (kernels.py:191-249, _matmul_bias_silu_kernel). */
enum glq_epilogue {
  GLQ_EPILOGUE_NONE = 0,
  GLQ_EPILOGUE_BIAS = 1,
  GLQ_EPILOGUE_BIAS_SILU = 2
};

/* GPU path taken by one call; reported through path_out.  Every path is a
 * GPU kernel of this library (or no launch at all for "empty"). */
enum glq_path {
  GLQ_PATH_EMPTY = 0,     /* M == 0 or N == 0: nothing to write, no launch */
  GLQ_PATH_ZERO_K = 1,    /* K == 0: fill kernel writes epilogue(0 [+ bias]) */
  GLQ_PATH_GEMV_M1 = 2,   /* M == 1, K-contiguous W: vectorised warp GEMV */
  GLQ_PATH_TC = 3,        /* tcgen05 + TMA + TMEM GEMM, no K split */
  GLQ_PATH_TC_SPLITK = 4, /* same, K split across a cluster, DSMEM merge */
  GLQ_PATH_TAIL = 5,      /* tcgen05 or GEMV kernel on a ragged N/K edge */
  GLQ_PATH_STRIDED = 6,   /* generic kernel: non-unit inner stride (no workspace) */
  GLQ_PATH_UNALIGNED = 7, /* generic kernel: rows or base not 16-B aligned (no workspace) */
  GLQ_PATH_TC_KN = 8,     /* tcgen05 GEMM with an N-contiguous B = [K, N]
                             (the lab's own layout): MN-major W tiles */
  GLQ_PATH_REPACKED = 9,  /* strided or unaligned operands copied into the
                             caller's workspace with 16-B aligned rows, then
                             the tcgen05 or GEMV kernel on the copies */
  GLQ_PATH_TC_LDG = 10,   /* K-contiguous A or W rows not 16-B aligned (odd
                             K, pitch or base), W = B^T K-contiguous:
                             tcgen05 GEMM that loads those rows by row class
                             with TMA and aligns them in shared memory (no
                             copy, no workspace) */
  GLQ_PATH_COUNT = 11
};

enum glq_status {
  GLQ_OK = 0,
  GLQ_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad dtype/epilogue value */
  GLQ_ERR_SHAPE = 2,            /* negative or too large M/N/K, bad strides */
  GLQ_ERR_SPLIT = 3,            /* split_k outside 0..GLQ_MAX_SPLIT */
  GLQ_ERR_WORKSPACE = 4,        /* partial-sum workspace smaller than needed or not 4-B aligned */
  GLQ_ERR_OUTPUT_LAYOUT = 5,    /* y_row_stride < N */
  GLQ_ERR_CUDA = 6,             /* CUDA runtime or driver call failed */
  GLQ_ERR_DEVICE = 7,           /* no device, or not a compute 10.0 GPU */
  GLQ_ERR_DEVICE_TIMEOUT = 8,   /* an in-kernel bounded wait expired */
  GLQ_ERR_SCRATCH = 9,          /* request beyond the static scratch of
                                   glq_linear_gather_static */
  GLQ_STATUS_COUNT = 10
};

#define GLQ_MAX_SPLIT 8

/* Per-call flags of glq_linear_ex (bitwise OR). */
enum glq_flags {
  /* Launch without programmatic dependent launch.  By default the tcgen05
   * and GEMV kernels are launched with it: a kernel lets the next kernel of
   * the stream begin launching early, and every kernel waits for its
   * predecessor to complete (griddepcontrol.wait) before it touches global
   * memory, so stream order semantics are unchanged. */
  GLQ_FLAG_NO_PDL = 1u << 0,
  /* The weight operand B is not written by the kernel that precedes this call
   * in the stream (true for inference weights).  The kernel then starts
   * streaming B before the dependency wait, overlapping the predecessor's
   * tail.  Only A, bias and Y wait for the predecessor. */
  GLQ_FLAG_STATIC_WEIGHTS = 1u << 1
};

/*
 * glq_linear -- the one general entry point.
 *
 *   A[m, k]   at A + m * a_row_stride + k * a_col_stride        (elements)
 *   B[k, n]   at B + k * b_k_stride   + n * b_n_stride          (elements)
 *   bias[n]   at bias + n (contiguous; required unless epilogue NONE)
 *   Y[m, n]   at Y + m * y_row_stride + n                        (unit column stride)
 *   A, B, bias and Y are 2-byte aligned (GLQ_ERR_INVALID_ARGUMENT otherwise).
 *
 * split_k: 0 = library choice; 1..GLQ_MAX_SPLIT = split the K reduction into
 *   that many contiguous ranges merged in-kernel in split order (the merge is
 *   deterministic).  A path that cannot split reports split 1.
 * workspace: optional (may be NULL).  When non-NULL it receives the FP32
 *   per-split partial sums in the lab's [split, M, N] layout
 *   (kernels.py:431-439), and must hold glq_workspace_bytes() bytes and be
 *   4-byte aligned (GLQ_ERR_WORKSPACE otherwise).  The
 *   merge itself never needs it.  For operands the TMA kernels cannot
 *   address, a workspace of glq_linear_workspace_bytes() bytes instead
 *   holds their aligned copies (GLQ_PATH_REPACKED).
 * path_out, split_out: optional host pointers receiving the path taken and
 *   the split count used.
 *
 * Replaces: gemm_lab::launch_* / launch_ptx_mma_splitk (csrc/ptx_mma.cuh:
 *   220-965) and the launch bodies of kernels.py:148-171, 252-280, 396-441.
 */
int glq_linear(int dtype,
               const void* A, int64_t a_row_stride, int64_t a_col_stride,
               const void* B, int64_t b_k_stride, int64_t b_n_stride,
               const void* bias, int epilogue,
               void* Y, int64_t y_row_stride,
               int64_t M, int64_t N, int64_t K,
               int split_k, void* workspace, size_t workspace_bytes,
               void* stream, int* path_out, int* split_out);

/*
 * glq_linear_ex -- glq_linear with per-call flags (enum glq_flags).
 * glq_linear(...) == glq_linear_ex(..., 0).  No reference counterpart: the
 * reference's launches have no dependency control.
 */
int glq_linear_ex(int dtype,
                  const void* A, int64_t a_row_stride, int64_t a_col_stride,
                  const void* B, int64_t b_k_stride, int64_t b_n_stride,
                  const void* bias, int epilogue,
                  void* Y, int64_t y_row_stride,
                  int64_t M, int64_t N, int64_t K,
                  int split_k, void* workspace, size_t workspace_bytes,
                  void* stream, unsigned int flags, int* path_out, int* split_out);

/*
 * glq_linear_f16 -- FP16 form with the argument order of the lab's proposed
 * native shim: A with (lda, a_col_stride), B with (b_row_stride = k stride,
 * b_col_stride = n stride), nullable bias selecting bias+SiLU.
 * Replaces: triton_bias_silu_into / triton_matmul_into (kernels.py:148-171,
 * 252-280) for FP16.
 */
int glq_linear_f16(const void* A, int64_t lda, int64_t a_col_stride,
                   const void* B, int64_t b_row_stride, int64_t b_col_stride,
                   const void* bias, void* Y, int64_t ldy,
                   int M, int N, int K, int split_k,
                   void* workspace, size_t workspace_bytes,
                   void* stream, int* path_out);

/*
 * glq_matmul -- C = A * B for contiguous row-major A[M, K], B[K, N],
 * C[M, N] of `dtype`.  Replaces the launch signature shared by every native
 * implementation: void launch_X(const T* a, const T* b, T* c, int m, int n,
 * int k, cudaStream_t) (csrc/ptx_mma.cuh:220,772,796,827,978,1031).
 */
int glq_matmul(int dtype, const void* a, const void* b, void* c,
               int m, int n, int k, void* stream);

/*
 * glq_splitk_matmul -- forced split-K C = A * B (contiguous row-major), the
 * per-split FP32 partials written to `partial` ([splits, M, N]) and merged
 * in-kernel.  Replaces launch_ptx_mma_splitk(a, b, c, m, n, k, partial,
 * splits, stream) (csrc/ptx_mma.cuh:931-965).  partial may be NULL.
 */
int glq_splitk_matmul(int dtype, const void* a, const void* b, void* c,
                      int m, int n, int k, float* partial, int splits,
                      void* stream);

/*
 * glq_workspace_bytes -- bytes of the optional partial-sum workspace for a
 * call of this shape with this split_k (0 = the library's choice for a
 * K-contiguous problem).  Replaces ptx_mma_splitk_workspace_bytes
 * (csrc/ptx_mma.cuh:926-929) and TritonSplitKPlan.workspace_bytes
 * (kernels.py:461-464).  Pure host function.
 */
size_t glq_workspace_bytes(int64_t M, int64_t N, int64_t K, int split_k);

/*
 * glq_linear_workspace_bytes -- bytes of workspace with which a glq_linear
 * call on exactly these operands (pointers and strides) takes the repacked
 * path: every operand the TMA kernels cannot address (base or row pitch not
 * 16-byte aligned, overlapping rows, or no unit stride) is first copied into
 * the workspace with 16-byte aligned rows, and the call then runs the
 * tcgen05 or GEMV kernel on the copies (path GLQ_PATH_REPACKED).  0 when
 * the operands are addressable as they are, and when the tcgen05 kernel
 * aligns them itself (K-contiguous rows of A and of W = B^T whose base or
 * pitch is off 16 bytes, at most 128 tokens: GLQ_PATH_TC_LDG, no copy; above
 * 128 tokens such operands are copied when the workspace allows, since every
 * token tile would re-align the same weight tiles).  Given less, such a call
 * runs the generic kernel (GLQ_PATH_STRIDED / GLQ_PATH_UNALIGNED), or
 * GLQ_PATH_TC_LDG for those K-contiguous rows, as it does when the workspace
 * is not 16-byte aligned.  When the workspace
 * serves a repack it holds no split partials.  Pure host function.
 * No counterpart in the reference: the lab's Triton kernel reads any
 * contiguous layout through masked loads (kernels.py:103-129) and sends
 * strided views to torch (qualification.py:58-64).
 */
size_t glq_linear_workspace_bytes(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride,
                                  const void* B, int64_t b_k_stride, int64_t b_n_stride, int64_t M,
                                  int64_t N, int64_t K);

/*
 * glq_plan -- the path and split a glq_linear call with these arguments
 * would take, without launching anything (pure host function; pointer
 * arguments are only inspected for alignment).  Replaces the per-call path
 * selection of qualification.path (qualification.py:58-59) and
 * ptx_mma_split_count (csrc/ptx_mma.cuh:889-924).  sm_count 0 = 148.
 * It plans a call without workspace: for operands that a workspace of
 * glq_linear_workspace_bytes() bytes would repack, it reports
 * GLQ_PATH_STRIDED / GLQ_PATH_UNALIGNED.
 */
int glq_plan(int dtype,
             const void* A, int64_t a_row_stride, int64_t a_col_stride,
             const void* B, int64_t b_k_stride, int64_t b_n_stride,
             int64_t y_row_stride, int64_t M, int64_t N, int64_t K,
             int split_k, int sm_count, int* path_out, int* split_out);

/* Ranks one fused-gather call can address. */
#define GLQ_MAX_RANKS 8

/*
 * glq_linear_gather -- one rank's share of a column-parallel (N-sharded)
 * linear layer with the all-gather fused into the kernel's epilogue.  This
 * rank computes Y_r = epilogue(A . B_r) for its N-slice exactly as glq_linear
 * does (same planner, tensor-core paths only), and the epilogue stores every
 * output element straight into all `world` ranks' output buffers over
 * NVLink (plain peer stores; no TMA multicast, no library kernel touches
 * peer memory).  The last CTA to finish then publishes `epoch` into slot
 * [rank] of every rank's signal array and waits (bounded) until all `world`
 * slots of its own array reached `epoch`; when the kernel completes, this
 * rank's output buffer holds every rank's slice.
 *
 * y_ranks[r]      device pointer (mapped in this process) to rank r's output
 *                 [M, N * world] row-major buffer, row pitch y_row_stride;
 *                 this rank writes columns [y_col_offset, y_col_offset + N).
 * signal_ranks[r] device pointer (mapped in this process) to rank r's array
 *                 of `world` uint64 slots, zero-initialised once.
 * counter         this rank's device arrival counter, zero before the first
 *                 call; every call leaves it zero.
 * epoch           strictly larger than the previous call's, equal on all
 *                 ranks for the same call.
 * Requires K > 0 and operands the tensor-core paths take (K-contiguous or
 * N-contiguous B, 16-byte aligned); otherwise GLQ_ERR_INVALID_ARGUMENT.  A
 * peer that never publishes sets a bit in the device error word
 * (glq_device_error) after the wait budget; the kernel still returns.
 *
 * No reference counterpart: the reference has no multi-GPU path.  It
 * replaces the local GEMM followed by an NCCL all_gather_into_tensor and
 * the [P, M, N/P] -> [M, N] layout copy of the column-parallel layer.
 */
int glq_linear_gather(int dtype,
                      const void* A, int64_t a_row_stride, int64_t a_col_stride,
                      const void* B, int64_t b_k_stride, int64_t b_n_stride,
                      const void* bias, int epilogue,
                      void* const* y_ranks, int64_t y_row_stride, int64_t y_col_offset,
                      int64_t M, int64_t N, int64_t K, int split_k,
                      int rank, int world,
                      uint64_t* const* signal_ranks, unsigned int* counter, uint64_t epoch,
                      void* stream, unsigned int flags, int* path_out, int* split_out);

/* Arrival-counter slots in the static scratch of glq_linear_gather_static
 * (one 32-bit word each: 256 bytes per GPU that loads the library). */
#define GLQ_STATIC_GATHER_SLOTS 64

/*
 * glq_linear_gather_static -- glq_linear_gather for callers that cannot
 * allocate device memory.  The fused gather needs one private, zeroed 32-bit
 * arrival counter per rank besides its inputs and outputs; some callers have
 * no way to get one: a plugin or foreign-language host that only receives
 * device pointers from its framework (the weights, the activations and the
 * communicator's peer-mapped output and signal buffers) and owns no
 * allocator, or a pipeline that must not call cudaMalloc because that
 * synchronises the device.  This entry point takes the counter from a
 * fixed array compiled into the library instead: GLQ_STATIC_GATHER_SLOTS
 * words, held by every GPU that loads the library until the process exits.
 * `counter_slot` picks the word; a slot outside 0..GLQ_STATIC_GATHER_SLOTS-1
 * is rejected with GLQ_ERR_SCRATCH.  Every other argument and the result are
 * those of glq_linear_gather (the caller still passes the inputs, the
 * outputs and the signal slots), and nothing is allocated.
 *
 * Every argument is checked before the slot is touched: a refused call
 * (odd element pointer, bad rank or epoch, ...) returns its status without
 * writing the array.  An accepted call clears its slot on the caller's
 * stream (one stream-ordered 4-byte memset) and then launches.  All calls
 * share the array: calls that use the same slot and overlap on the GPU
 * (different streams, or several layers in flight) race and corrupt each
 * other's completion; give such calls different slots.  The first call on a
 * device looks up the array's device address with that device current (a
 * host-side query: nothing is written and the device is not synchronised);
 * make that first call before any stream capture.
 *
 * No counterpart in the reference (it has no multi-GPU path and no
 * allocation-free entry points).
 */
int glq_linear_gather_static(int dtype,
                             const void* A, int64_t a_row_stride, int64_t a_col_stride,
                             const void* B, int64_t b_k_stride, int64_t b_n_stride,
                             const void* bias, int epilogue,
                             void* const* y_ranks, int64_t y_row_stride, int64_t y_col_offset,
                             int64_t M, int64_t N, int64_t K, int split_k,
                             int rank, int world,
                             uint64_t* const* signal_ranks, int counter_slot, uint64_t epoch,
                             void* stream, unsigned int flags, int* path_out, int* split_out);

/* Names of paths and statuses (static strings, never NULL). */
const char* glq_path_name(int path);
const char* glq_status_string(int status);

/*
 * glq_device_error -- read (and with clear != 0, reset) the sticky error word
 * that this library's kernels set when a bounded in-kernel wait expires, for
 * the current device.  Synchronises the device.  *word_out is 0 when no
 * kernel has reported a problem.
 */
int glq_device_error(unsigned int* word_out, int clear);

/* ABI version (GLQ_ABI_VERSION) and the compiled target, e.g. "sm_100a". */
int glq_abi_version(void);
const char* glq_build_target(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GLQ_H_ */
