/* C ABI of the B200 (sm_100a) MXFP8 quantizer and fused SwiGLU-LoRA MLP.
 *
 * Every entry point takes plain device pointers, element counts / leading dimensions and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream), returns an `int` status
 * (0 = ok, negative = mxm_status) and never synchronizes the stream.  Buffers are owned by the
 * caller (in the Python host layer: torch allocations on the input's device).  A failure message
 * is kept per host thread and returned by mxm_last_error().
 *
 * Data formats (the reference's, scripts/mxfp8.py:36,78-86):
 *   bf16        row-major, 2 bytes per element
 *   E4M3 codes  1 byte per element (torch.float8_e4m3fn)
 *   E8M0 scales 1 byte per 32 contiguous elements along the quantized axis, in the cuBLAS /
 *               tcgen05 128x4 blocked layout: the scale of (row r, 32-block kb) of a [R, K]
 *               operand sits at byte
 *                 ((r / 128) * (K / 128) + kb / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + kb % 4
 *               and the buffer holds ceil(R / 128) * (K / 128) * 512 bytes; rows >= R get scale 0.
 *
 * Reference interfaces replaced (paths relative to the reference project root) are cited per
 * function.
 */
#ifndef MXMLP_H_
#define MXMLP_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXM_ABI_VERSION 1

typedef enum {
  MXM_OK = 0,
  MXM_ERR_ARG = -1,         /* invalid shape / stride / alignment / pointer */
  MXM_ERR_CUDA = -2,        /* a CUDA runtime or driver call failed */
  MXM_ERR_UNSUPPORTED = -3, /* valid request this build does not implement (the caller falls back) */
  MXM_ERR_DEVICE = -4       /* a kernel recorded a device-side error (bounded wait ran out) */
} mxm_status;

/* ABI version (MXM_ABI_VERSION). */
int mxm_version(void);

/* Message of the last failure on this host thread ("" if none). */
const char* mxm_last_error(void);

/* Reads the device-side error flag of the current device into *code (0 = none); clears it when
 * `clear` is nonzero.  Synchronizes the device (host-side diagnostics only). */
int mxm_device_error(int* code, int clear);

/* Number of SMs of the current device (grid sizing; cached per device). */
int mxm_num_sms(void);

/* Row-wise MXFP8 quantization: x bf16 [R, K] (row stride ldx elements, K % 128 == 0)
 * -> q E4M3 [R, K] (row stride ldq) + s E8M0 blocked for [R, K].
 * Replaces mxfp8.mx_quant / _quant_kernel (scripts/mxfp8.py:46-86). */
int mxm_quant_rows(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, int64_t ldq, void* s,
                   void* stream);

/* Column-wise MXFP8 quantization: the row-wise quantization of x^T, i.e. blocks of 32 along R.
 * x bf16 [R, K] (R % 128 == 0, K % 128 == 0) -> qt E4M3 [K, R] + st E8M0 blocked for [K, R].
 * Replaces quant_ref(W.t().contiguous()) (scripts/mxfp8.py:40-43, used at :478,:490). */
int mxm_quant_cols(const void* x, int64_t R, int64_t K, int64_t ldx, void* qt, void* st, void* stream);

/* Both of the above from one read of x (R % 128 == 0, K % 128 == 0).
 * Replaces the quant_ref pair of enable_mxfp8 (scripts/mxfp8.py:477-478,488-490). */
int mxm_quant_both(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, void* s, void* qt, void* st,
                   void* stream);

/* MXFP8 block-scaled GEMM on tcgen05: D[M, N] = dq(A)[M, K] . dq(B)[N, K]^T, fp32 accumulate,
 * bf16 out (row stride ldd).  A, B are E4M3 codes quantized along K (row strides lda, ldb bytes),
 * sa / sb their blocked scales.  K % 128 == 0, N % 256 == 0, any M >= 1.
 * Replaces torch._scaled_mm(qa, qb.t(), sa, sb, out_dtype=bfloat16)
 * (scripts/fused_mlp.py:279,283,309,329). */
int mxm_gemm(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
             int64_t M, int64_t N, int64_t K, void* d, int64_t ldd, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXMLP_H_ */
