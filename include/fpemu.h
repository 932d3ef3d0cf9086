/*
 * fpemu.h -- C ABI of libfpemu.so, the B200 (sm_100a) implementation of
 * Ozaki scheme II FP64 matrix multiplication on INT8 tensor cores.
 *
 * Plain C: pointers, sizes and strides, a CUDA stream passed as void*, and
 * int status codes.  No exceptions cross this boundary, nothing here
 * allocates device memory, and every call is asynchronous on the given stream
 * (stream == NULL is the legacy default stream).  All device pointers must be
 * on the current CUDA device.
 *
 * Each entry point names the reference code it replaces (paths inside
 * thezettascale/fp-emulation).  Matrices are row-major in the reference's
 * sense: element (i, j) of A lives at A[i*sA_row + j*sA_col] (strides in
 * elements, so a transposed view is just swapped strides).
 */
#ifndef FPEMU_H_
#define FPEMU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FPEMU_ABI_VERSION 1

/* Status codes.  The Python layer maps INVALID/UNSUPPORTED_DTYPE/NO_MODULI to
 * the reference's exception types (TypeError at ozaki.py:99-104, ValueError at
 * ozaki.py:29). */
enum {
    FPEMU_OK = 0,
    FPEMU_ERR_INVALID = 1,       /* bad argument: null pointer, negative size, bad stride */
    FPEMU_ERR_NO_MODULI = 2,     /* k too large for the prime list (ozaki.py:29) */
    FPEMU_ERR_UNSUPPORTED = 3,   /* k beyond the exact int32 accumulation limit, ... */
    FPEMU_ERR_WORKSPACE = 4,     /* workspace too small or misaligned */
    FPEMU_ERR_CUDA = 5,          /* a CUDA runtime/driver call failed */
    FPEMU_ERR_TIMEOUT = 6,       /* a device-side wait gave up (see fpemu_device_error) */
    FPEMU_ERR_NO_DEVICE = 7      /* current device is not sm_100 */
};

/* Human-readable name of a status code, and the last error detail recorded by
 * a call on this host thread. */
const char *fpemu_status_string(int status);
const char *fpemu_last_error(void);
int fpemu_abi_version(void);

/* ---- host-side planning -------------------------------------------------- */

/* ozaki.py:20-29 (_n_moduli) and ozaki.py:109 (moduli = _PRIMES[:n_mod]):
 * fewest leading odd primes (3, 5, 7, ...) whose product exceeds
 * 2*k*2^(2*bits).  `moduli` may be NULL, else it receives n_mod entries.
 * Returns FPEMU_ERR_NO_MODULI when the 30 primes do not suffice. */
int fpemu_plan_moduli(int64_t k, int bits, int *n_mod, int32_t *moduli);

/* ozaki.py:62-80 (_crt_weights): w_i = M_i * (M_i^-1 mod p_i) as (hi, mid, lo)
 * doubles, M as (M_hi, M_lo), inv_M = 1/(double)M.  Exact 128-bit integer
 * arithmetic; n_mod <= 25. */
int fpemu_crt_weights(int n_mod, double *wh, double *wm, double *wl, double *M_hi,
                      double *M_lo, double *inv_M);

/* Largest inner dimension whose per-modulus int32 accumulation is exact:
 * k * (p_max - 1)^2 < 2^31 (reference: implicit in crt_kernel.cu:51). */
int64_t fpemu_max_k(int n_mod);

/* Device bytes of workspace fpemu_ozaki2_dgemm needs for this problem. */
size_t fpemu_workspace_size(int64_t m, int64_t n, int64_t k, int n_mod);

/* ---- the one-shot operation ---------------------------------------------- */

/* C[m x n] (row stride ldc) = A[m x k] * B[k x n], emulated FP64.
 * Replaces ozaki.py:95-119 (_ozaki2_forward) with its CUDA branch
 * _cuda_crt.py:33-72 -> crt_kernel.cu:19-146.
 *   bits   : precision of the caller's dtype (53 fp64, 24 fp32, 11 fp16, 8 bf16;
 *            ozaki.py:12-17); A and B are always passed as float64.
 *   n_mod  : 0 = the reference's choice fpemu_plan_moduli(k, bits); otherwise
 *            use the first n_mod primes (for modulus-count sweeps).
 * One split kernel per operand, then one persistent tcgen05 GEMM whose
 * epilogue reduces each accumulator mod p and reconstructs C. */
int fpemu_ozaki2_dgemm(int64_t m, int64_t n, int64_t k, const double *A, int64_t sA_row,
                       int64_t sA_col, const double *B, int64_t sB_row, int64_t sB_col,
                       double *C, int64_t ldc, int bits, int n_mod, void *workspace,
                       size_t workspace_bytes, void *stream);

/* Output element types of the _ex entry points. */
#define FPEMU_C_F64 0
#define FPEMU_C_F32 1

/* fpemu_ozaki2_dgemm with the output's dtype cast and an nn.Linear bias fused
 * into the epilogue: C (c_dtype) = cast(A @ B) + bias[j], in that order and
 * with one rounding each -- ozaki.py:117-118 (`.to(orig_dtype)`) followed by
 * nn.py:20-21 (`out + self.bias`).  bias: n elements of C's type, or NULL. */
int fpemu_ozaki2_gemm_ex(int64_t m, int64_t n, int64_t k, const double *A, int64_t sA_row,
                         int64_t sA_col, const double *B, int64_t sB_row, int64_t sB_col,
                         void *C, int64_t ldc, int c_dtype, const void *bias, int bits, int n_mod,
                         void *workspace, size_t workspace_bytes, void *stream);

/* ---- stages (each is also the parity tap for one step of the reference) -- */

/* ozaki.py:32-46 (_scale_to_int + _residues) for one operand, fused:
 * X is rows x k (element (r, t) at X[r*s_row + t*s_k]); per row r
 *   exps[r] = frexp(max(max_t |X[r,t]|, 1e-300)).exponent
 *   res[l][r][t] = (X[r,t] * 2^(bits - exps[r]) rounded half-even) mod p_l in [0, p_l)
 * res is int8 [n_mod][rows][res_ld] (plane stride res_plane), k contiguous;
 * columns k..res_ld-1 are written as 0.  res_ld % 16 == 0.
 * For B [k x n] pass its transpose view (rows = n, s_row = sB_col, s_k = sB_row),
 * which yields the column exponents (ozaki.py:35) and K-major residues.
 * `colmax_scratch` (rows uint64 values) is needed when s_k != 1, else NULL. */
int fpemu_split(int64_t rows, int64_t k, const double *X, int64_t s_row, int64_t s_k, int bits,
                int n_mod, int8_t *res, int64_t res_ld, int64_t res_plane, int32_t *exps,
                uint64_t *colmax_scratch, void *stream);

/* ozaki.py:49-59 (_matmul_residues), CUDA branch _cuda_crt.py:33-42 ->
 * crt_kernel.cu:19-94 (cuBLASLt batched GEMM + mod_reduce):
 *   mode 0: out int32 [n_mod][m][n] = a_res[l] @ b_res[l]^T  (raw products)
 *   mode 1: out uint8 [n_mod][m][n] = that mod p_l           (reduced residues)
 * a_res int8 [n_mod][m][res_ld], b_res int8 [n_mod][n][res_ld] (both K-major). */
int fpemu_gemm_residues(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t *a_res,
                        const int8_t *b_res, int64_t res_ld, int mode, void *out,
                        void *workspace, size_t workspace_bytes, void *stream);

/* ozaki.py:83-92 (_reconstruct), CUDA branch _cuda_crt.py:45-72 ->
 * crt_kernel.cu:96-146: C[i][j] from uint8 residues [n_mod][m][n]. */
int fpemu_crt_reconstruct(int64_t m, int64_t n, int n_mod, const uint8_t *res,
                          const int32_t *row_exp, const int32_t *col_exp, int bits, double *C,
                          int64_t ldc, void *stream);

/* The fused GEMM + mod + CRT stage on residues that are already split
 * (crt_kernel.cu:19-146 in one kernel).  b_res_plane is the plane stride of
 * b_res (n * res_ld when the planes are packed; larger for a column chunk of a
 * bigger residue buffer).  max_ctas > 0 caps the persistent grid (the
 * multi-GPU driver leaves SMs free for NCCL's kernels); 0 uses every SM.  The
 * multi-GPU driver calls this per column chunk of B as its residues arrive. */
int fpemu_gemm_crt(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t *a_res,
                   const int8_t *b_res, int64_t res_ld, int64_t b_res_plane,
                   const int32_t *row_exp, const int32_t *col_exp, int bits, double *C,
                   int64_t ldc, int max_ctas, void *workspace, size_t workspace_bytes,
                   void *stream);

/* fpemu_gemm_crt with the output cast and bias of fpemu_ozaki2_gemm_ex (used
 * with cached residues of a static operand, e.g. an nn.Linear weight). */
int fpemu_gemm_crt_ex(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t *a_res,
                      const int8_t *b_res, int64_t res_ld, int64_t b_res_plane,
                      const int32_t *row_exp, const int32_t *col_exp, int bits, void *C,
                      int64_t ldc, int c_dtype, const void *bias, int max_ctas, void *workspace,
                      size_t workspace_bytes, void *stream);

/* fpemu_gemm_crt for a product whose columns come from several column blocks
 * of C: column j of this product is written to C column
 *     (j / col_seg) * col_seg_stride + j % col_seg
 * (1 <= col_seg <= col_seg_stride).  The multi-GPU product over a
 * column-sharded B uses it: a column chunk of the all-gathered B holds one
 * strip of col_seg columns from each GPU's block of col_seg_stride columns.
 * No counterpart in the reference (which has no multi-GPU path). */
int fpemu_gemm_crt_segmented(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t *a_res,
                             const int8_t *b_res, int64_t res_ld, int64_t b_res_plane,
                             const int32_t *row_exp, const int32_t *col_exp, int bits, double *C,
                             int64_t ldc, int64_t col_seg, int64_t col_seg_stride, int max_ctas,
                             void *workspace, size_t workspace_bytes, void *stream);

/* Allocation-free variant of fpemu_gemm_crt.  It has no counterpart in the
 * reference.  For callers that cannot allocate device memory -- code running
 * where cudaMalloc is not allowed (inside a host application that owns the
 * allocator, or a runtime that forbids allocation between launches) -- it
 * needs no workspace argument: the fused kernel stages its residues in a
 * static device array of FPEMU_NOALLOC_SCRATCH_BYTES (64 MiB) that is part of
 * the library, so every GPU that loads the library holds it until the process
 * exits.  The caller still passes all inputs and the output C.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) and caches it; make that first call before any
 *    stream capture.
 *  - The kernel grid shrinks to the CTAs whose staging fits the array
 *    (n_mod * 32 KiB per CTA: 80 CTAs at n_mod = 25), so large problems run
 *    slower than through fpemu_gemm_crt; a modulus count whose staging does not
 *    fit one CTA pair is rejected with FPEMU_ERR_WORKSPACE.
 *  - All calls share the array and it keeps the last call's contents (nothing
 *    in it needs to start at zero).  Calls that overlap on the GPU -- on two
 *    streams, or from two host threads -- race on it and corrupt each other.
 *  - Calls no cudaMalloc, cudaFree or other allocating routine. */
#define FPEMU_NOALLOC_SCRATCH_BYTES (64u << 20)
int fpemu_gemm_crt_noalloc(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t *a_res,
                           const int8_t *b_res, int64_t res_ld, const int32_t *row_exp,
                           const int32_t *col_exp, int bits, double *C, int64_t ldc,
                           void *stream);

/* Kernels one fpemu_gemm_crt / _ex / _segmented call launches for an m x n
 * product on the current device: 1 (the fused GEMM + CRT kernel) or 2 (the
 * split form for products with few tiles per CTA pair: the residue GEMM, then
 * the CRT kernel; FPEMU_GEMM_PATH forces one).  0 on error.  No counterpart in
 * the reference. */
int fpemu_gemm_kernels(int64_t m, int64_t n);

/* Workspace bytes fpemu_gemm_crt / fpemu_gemm_residues need (the epilogue's
 * per-CTA residue staging, or the split form's residues). */
size_t fpemu_gemm_workspace_size(int64_t m, int64_t n, int n_mod);

/* ---- device status ---------------------------------------------------------- */

/* Synchronise the current device and read (optionally clear) the first error a
 * kernel of this library recorded on it (a bounded wait that timed out).
 * *code is FPEMU_OK when nothing was recorded.  where/block/detail may be NULL.
 * When a GEMM wait times out, the output tiles the kernel could not finish are
 * written as NaN, so a failed product never looks like a result.
 * No counterpart in the reference (whose kernels have no waits); it replaces
 * the TORCH_CHECK error path of crt_kernel.cu:63,75. */
int fpemu_device_error(int *code, int *where, int *block, int *detail, int clear);

/* Make the kernels of this library on the current device also record their
 * first error in pinned host memory (allocated once per process; no device
 * memory), so that fpemu_poll_error can see it without synchronising.  Call
 * once per device, outside stream capture.  No counterpart in the reference. */
int fpemu_watch_errors(void);

/* Non-blocking: the first error recorded on the current device by kernels that
 * have finished (FPEMU_OK if none so far).  Needs fpemu_watch_errors on this
 * device; clear with fpemu_device_error(..., clear = 1).  No counterpart in the
 * reference. */
int fpemu_poll_error(int *code, int *where, int *block, int *detail);

#ifdef __cplusplus
}
#endif

#endif /* FPEMU_H_ */
