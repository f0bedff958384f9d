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
 * `clear` is nonzero.  Returns MXM_ERR_DEVICE (with a message naming the code) when a kernel recorded
 * an error, i.e. one of its bounded waits ran out and it returned early.  Synchronizes the device
 * (host-side diagnostics only).  No counterpart in the reference, whose watchdog is host-side
 * (SlowGuard, scripts/train.py:249-278). */
int mxm_device_error(int* code, int clear);

/* Test entry for the bounded waits: launches one CTA that waits on an mbarrier nothing arrives on, with
 * a wait limit of limit_ns nanoseconds (0 < limit_ns <= 1e8) instead of the kernels' 2 s.  The wait runs
 * out, the kernel records code 9 in the device error flag and returns; mxm_device_error then reports
 * MXM_ERR_DEVICE.  No counterpart in the reference (see mxm_device_error). */
int mxm_selftest_wait(int64_t limit_ns, void* stream);

/* Number of kernels this library has launched in this process (all devices, host-side count). */
unsigned long long mxm_launch_count(void);

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


/* mxm_gemm with a rank-kr LoRA term accumulated on the tensor core into the same fp32 accumulator:
 *   D = bf16( dq(A) dq(B)^T + L[M, kr] . Rm[N, kr]^T )
 * L bf16 with row stride ldl (elements, % 8 == 0), Rm bf16 contiguous [N, kr] (the caller folds the LoRA
 * scaling into Rm), kr in {16, 32, 64}.  Replaces `y = _scaled_mm(...); y.addmm_(xS_down, B_down^T,
 * alpha=s_down)` and `dx = _scaled_mm(...); dx.addmm_(dxa, S)` (scripts/fused_mlp.py:283-284, :329-331);
 * the MX product is not rounded to bf16 before the LoRA add (one rounding instead of the reference's two). */
int mxm_gemm_lora(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                  int64_t M, int64_t N, int64_t K, const void* L, int64_t ldl, const void* Rm, int kr, void* d,
                  int64_t ldd, void* stream);

/* Column-group count for mxm_mlp_fwd_epilogue (reference mlp_fwd grid choice, scripts/fused_mlp.py:203-204). */
int mxm_mlp_fwd_partitions(int64_t T, int64_t N, int r, int* col_groups);

/* Forward epilogue of the fused MLP (reference mlp_fwd / _fwd_kernel, scripts/fused_mlp.py:65-109,198-215):
 *   g = bf16(gu[:, :N] + s_g xs[:, :r] bg^T), u = bf16(gu[:, N:] + s_u xs[:, r:2r] bu^T),
 *   h = bf16(g / (exp(-g) + 1) * u);  qh, sh = MXFP8(h) (row-wise, blocked scales; skipped when qh is NULL);
 *   xsd = bf16(h ad^T).
 * gu bf16 [T, 2N], xs bf16 [T, 2r], bg / bu bf16 [N, r], ad bf16 [r, N], qh [T, N], sh blocked for [T, N],
 * xsd bf16 [T, r].  xsd_part: fp32 [col_groups, T, r] scratch (unused when col_groups == 1). */
int mxm_mlp_fwd_epilogue(const void* gu, const void* xs, const void* bg, const void* bu, const void* ad, int64_t T,
                         int64_t N, int r, float s_g, float s_u, void* qh, void* sh, void* xsd, void* xsd_part,
                         int col_groups, void* stream);

/* The gate|up GEMM with the forward epilogue fused in (reference gu GEMM + _fwd_kernel, scripts/fused_mlp.py:
 * 279-282 and :81-109): from MX codes qa [M, K] and qb = W_gu [2N, K] (rows: gate then up) with their blocked
 * scales, g = bf16(bf16(x W_gate^T) + s_g xs_g bg^T), u likewise, qh / sh = MXFP8(h) [M, N] with
 * h = bf16(silu(g) u), and xsd [M, r] bf16 = bf16(h ad^T).  gu [M, 2N] bf16 = [g | u], the LoRA terms
 * included (what the backward needs: mxm_mlp_bwd_epilogue with gu_lora = 1).
 * xs [M, 2r] bf16 contiguous, bg / bu [N, r], ad [r, N] bf16 contiguous; r = 16; N % 128 == 0.
 * xsd_part: fp32 scratch of slots * M * r elements (mxm_gemm_glu_partition: per = tiles per work unit,
 * grid = CTAs launched, slots = units that can touch one row block).  For M >= 256 the work units are CTA
 * pairs (clusters of two on the tensor cores' cta_group::2 path, 256-row tiles, grid = 2 x pairs), below
 * that single CTAs over 128-row tiles; the choice depends only on M and the device, so the partition and
 * the launch agree. */
int mxm_gemm_glu_partition(int64_t M, int64_t N, int* per, int* grid, int* slots);
int mxm_gemm_glu(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb, int64_t M,
                 int64_t N, int64_t K, void* gu, const void* xs, const void* bg, const void* bu, const void* ad, int r,
                 float s_g, float s_u, void* qh, void* sh, void* xsd_part, void* xsd, void* stream);

/* Row-block size and dxa partial-slot count for the backward epilogue (reference _bwd_grid,
 * scripts/fused_mlp.py:218-232): col_groups = the number of [T, 3r] fp32 slots dxa_part needs. */
int mxm_mlp_bwd_partitions(int64_t T, int64_t N, int r, int* super_block, int* col_groups);

/* Backward epilogue of the fused MLP (reference mlp_bwd / _bwd_kernel, scripts/fused_mlp.py:112-175,235-259).
 * Recomputes g, u, h from gu (gu_lora = 0: gu = [x W_gate^T | x W_up^T] and g = bf16(gu_gate + s_g xs_g bg^T),
 * u likewise, as the reference; gu_lora = 1, rank 16 only: gu already holds g | u, as mxm_gemm_glu writes it);
 * dh = bf16(dhm + dxd ad); du = bf16(dh silu(g)); dg = bf16(dh u sig (g (1-sig) + 1));
 * q / s = MXFP8([dg | du]) [T, 2N] (skipped when q is NULL).  Partial sums (fp32, fixed-order reduction in
 * mxm_mlp_bwd_reduce): dxa_part [col_groups, T, 3r] = [dg bg | du bu | h ad^T], one slot per CTA that
 * worked on a row block (slots a row block does not use are left unwritten);
 * dbg_part / dbu_part [n_super, N, r] = dg^T xa_g / du^T xa_u; dad_part [n_super, r, N] = dxd^T h,
 * n_super = ceil(ceil128(T) / super_block). */
int mxm_mlp_bwd_epilogue(const void* gu, const void* xs, const void* dhm, const void* dxd, const void* bg,
                         const void* bu, const void* ad, int64_t T, int64_t N, int r, float s_g, float s_u,
                         int gu_lora, void* q, void* s, void* dxa_part, void* dbg_part, void* dbu_part,
                         void* dad_part, int super_block, int col_groups, void* stream);

/* Fixed-order reduction of the backward partials (scripts/fused_mlp.py:258-259,316-326):
 * dxa bf16 [T, 2r] = [s_g sum(dxa_g) | s_u sum(dxa_u)], xsd bf16 [T, r] = sum(xS_down),
 * dBg / dBu fp32 [N, r] = s_g / s_u times the sums, dAd fp32 [r, N]. */
int mxm_mlp_bwd_reduce(const void* dxa_part, const void* dbg_part, const void* dbu_part, const void* dad_part,
                       int64_t T, int64_t N, int r, float s_g, float s_u, int super_block, int col_groups, void* dxa,
                       void* xsd, void* dBg, void* dBu, void* dAd, void* stream);

/* out[T, n] = bf16( bf16(A[T, K] B[n, K]^T) * post ) (post == 1: one rounding); n in {16, 32, 64}, K % 128 == 0.
 * The rank-n LoRA-A products: xs = x S^T and dxd = s_d (dy B_down) (scripts/fused_mlp.py:277,311-313). */
int mxm_rowdot(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post, void* out,
               int64_t ldo, void* stream);

/* Row-wise MXFP8 of x [R, K] into columns col_tile_off*128 .. of a wider MX operand [ceil128(R), s_cols]:
 * codes at q[r * ldq + col_tile_off*128 + c], scales in that operand's blocked layout.  The quantize-only
 * mode of the reference's lora_bwd (scripts/mxfp8.py:219-246): one K-concatenated dy for a group's dx. */
int mxm_quant_rows_into(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, int64_t ldq, void* s,
                        int64_t s_cols, int64_t col_tile_off, void* stream);

/* The reference's lora_bwd for one LoRA branch (scripts/mxfp8.py:127-263): dxa_out [T, r] = bf16(scale *
 * dy B) with Bt = B^T [r, N]; dB_out [N, r] fp32 = scale * dy^T xa; and, when q / s are given, the row-wise
 * MXFP8 of dy into columns col_tile_off*128 .. of a [ceil128(T), s_cols] operand from the same read of dy.
 * part: fp32 [chunks, N, r] scratch with mxm_coldot_chunks(T, N) chunking.  N % 128 == 0, r in {16, 32, 64}. */
int mxm_lora_bwd(const void* dy, int64_t ldy, int64_t T, int64_t N, const void* xa, int64_t ldxa, const void* Bt,
                 int r, float scale, void* q, int64_t ldq, void* s, int64_t s_cols, int64_t col_tile_off,
                 void* dxa_out, int64_t ld_dxa, void* dB_out, void* part, int rows_per_chunk, int chunks,
                 void* stream);

/* One branch of a linear group's backward (see mxm_group_lora_bwd). */
typedef struct {
  const void* dy;    /* [T, N] bf16, row stride ldy elements (multiple of 8, 16-byte aligned) */
  int64_t ldy;
  int64_t N;         /* output width of the linear, N % 128 == 0 */
  const void* xa;    /* [T, r] bf16 = this branch's columns of x S^T (row stride ldxa); NULL: no LoRA branch */
  int64_t ldxa;
  const void* Bt;    /* B^T [r, N] bf16 contiguous */
  int r;             /* LoRA rank: 16, 32 or 64 */
  float scale;       /* LoRA scaling */
  void* dxa_out;     /* [T, r] bf16 = bf16(scale * dy B), row stride ld_dxa */
  int64_t ld_dxa;
  void* dB_out;      /* [N, r] fp32 = scale * dy^T xa */
} mxm_group_branch;

/* The backward of a group of MX linears sharing one input, in one call (the reference's one-read grouped
 * backward, scripts/fused_linear.py:219-278, with mxfp8.lora_bwd per branch, scripts/mxfp8.py:219-263):
 * branch i's dy is read once for its row-wise MXFP8 codes -- written into columns [sum_{j<i} N_j, +N_i) of
 * the group's K-concatenated operand q [ceil128(T), s_cols] (row stride ldq) with scales in that operand's
 * blocked layout s -- and, for a LoRA branch, d(xa) and dB.  q / s may be NULL (no dx needed; every branch
 * must then carry a LoRA term).  part: fp32 scratch of part_bytes, at least max over LoRA branches of
 * chunks * N * r * 4 with mxm_coldot_chunks(T, N) chunking.  Returns MXM_ERR_UNSUPPORTED (before any
 * launch) for a LoRA rank the kernels do not take; the caller then runs its general path. */
int mxm_group_lora_bwd(int64_t T, int nb, const mxm_group_branch* br, void* q, int64_t ldq, void* s, int64_t s_cols,
                       void* part, int64_t part_bytes, void* stream);

/* out = bf16(x + bf16(y + scale * xa B^T)) for x, y, out [T, N] bf16 contiguous, xa [T, r] (row stride ldxa),
 * B [N, r] contiguous (reference res_lora, scripts/mxfp8.py:265-296).  N % 64 == 0, r in {16, 32, 64}. */
int mxm_res_lora(const void* x, const void* y, const void* xa, int64_t ldxa, const void* B, int64_t T, int64_t N,
                 int r, float scale, void* out, void* stream);

/* The per-step bf16 forms of the LoRA matrices in one launch (the reference's casts in _MLP.forward /
 * backward, scripts/fused_mlp.py:272-276,282,311,331).  Sources Ag, Au [r, H], Bg, Bu [N, r], Ad [r, N],
 * Bd [H, r], contiguous, all fp32 (src_fp32 = 1) or all bf16.  out (bf16, r * (7H + 3N) elements) =
 * S [2r, H] (= [Ag; Au]) | bg | bu | ad | bd | bds = bf16(bd * s_d) [H, r] | bd^T [r, H] | S^T [H, 2r]. */
int mxm_lora_prep(const void* Ag, const void* Au, const void* Bg, const void* Bu, const void* Ad, const void* Bd,
                  int src_fp32, int64_t H, int64_t N, int r, float s_d, void* out, void* stream);

/* mxm_rowdot plus the row-wise MXFP8 quantization of A from the same read of A: q [T, K] (row stride ldq)
 * and s (blocked layout of a [ceil128(T), K] operand) are exactly mxm_quant_rows(A).  The reference
 * quantizes and multiplies in two passes (scripts/fused_mlp.py:277-278 for x, :307,311 for dy). */
int mxm_rowdot_quant(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post, void* out,
                     int64_t ldo, void* q, int64_t ldq, void* s, void* stream);

/* Row chunking (rows per chunk: a multiple of 64, number of chunks) of mxm_coldot's partial buffer for a
 * [T, K] operand. */
int mxm_coldot_chunks(int64_t T, int64_t K, int* rows_per_chunk, int* chunks);

/* out = bf16( bf16(A[T, K]^T E[T, n]) * post ), written [K, n] (or [n, K] when transpose_out), as bf16, or
 * with out_fp32 as the same (bf16-valued) numbers in fp32 -- the gradient in an fp32 parameter's dtype.
 * part: fp32 [chunks, K, n] scratch; rows_per_chunk a multiple of 64.  K % 64 == 0, n in {16, 32, 64},
 * lda and lde multiples of 8 (16-byte rows), A and E 16-byte aligned.
 * The LoRA weight gradients dA = dxa^T x and dB_down = s_d (dy^T xS_down) (scripts/fused_mlp.py:316-318,333). */
int mxm_coldot(const void* A, int64_t lda, const void* E, int64_t lde, int64_t T, int64_t K, int n, float post,
               int transpose_out, void* part, int rows_per_chunk, int chunks, void* out, int out_fp32, void* stream);

/* Allocation-free variant of mxm_coldot, for callers that cannot allocate device memory: code running
 * inside a custom device allocator (a nested allocation would re-enter it) and services that reserve
 * their whole memory budget up front.  No counterpart in the reference.
 * Same arguments and result as mxm_coldot without the `part` / chunking / `out_fp32` arguments: the
 * output is bf16 only, and the partial sums use one fixed 16 MiB array in device memory that the
 * library holds on every GPU that loads it until the process exits.  Requires K * n <= 4,194,304 (one
 * row chunk of fp32 partials must fit); larger requests fail with MXM_ERR_ARG and a message.  It calls
 * no cudaMalloc / cudaFree and no allocating library routine.  The first call on each device looks up
 * the array's device address (with that device current) and caches it: make that first call before any
 * stream capture.  All calls share the array and it keeps the last call's partials (every value read is
 * written first in the same call, so nothing needs clearing); calls whose executions overlap on the GPU
 * race on it, so serialize them (one stream, or events). */
int mxm_coldot_noalloc(const void* A, int64_t lda, const void* E, int64_t lde, int64_t T, int64_t K, int n,
                       float post, int transpose_out, void* out, void* stream);

/* The row chunking mxm_coldot_noalloc uses for [T, K] x [T, n] on a device with num_sms SMs (0 = the
 * current device): mxm_coldot_chunks' chunking, with fewer and taller chunks where its partials would
 * not fit the fixed scratch (devices with more than about 256 SMs).  A query; no counterpart in the
 * reference. */
int mxm_coldot_noalloc_chunks(int64_t T, int64_t K, int n, int num_sms, int* rows_per_chunk, int* chunks);

#ifdef __cplusplus
}
#endif

#endif /* MXMLP_H_ */
