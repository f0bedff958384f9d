// MXFP8 quantizer for sm_100a: bf16 -> E4M3 codes + E8M0 scales (one per 32 contiguous elements
// along the quantized axis), scales written directly in the 128x4 blocked layout the tcgen05
// block-scaled MMA consumes.  Algorithm of the reference _quant_kernel (scripts/mxfp8.py:46-75):
//   amax = max |x| over the block (NaN if the block holds a NaN)
//   e    = round-up-to-power-of-two(amax / 448) as E8M0        (from amax's bits: mx_e8m0_of_amax)
//   q    = e4m3_rne(clamp(x * rcp(e), -448, 448)),  rcp(e) = 2^(127-e) (special cases 0/254/255)
//
// One CTA owns a 128-row x 128-column tile, which is exactly one 512-byte scale block of the
// blocked layout, so scales are assembled in shared memory and written as 32 coalesced 16-byte
// stores.  Loads are 16-byte vectors (8 bf16), fully coalesced; a 32-element block is 4 lanes,
// reduced with two xor-shuffles.  Memory bound: 3.03 bytes moved per element (rows only),
// 4.06 for rows + columns from one read.
#include "mx_common.cuh"
#include "mx_runtime.h"

namespace {

constexpr int QT = 256;  // threads per CTA

struct Quant8 {
  uint2 codes;   // 8 E4M3 codes
  uint32_t e;    // the block's scale (same in the 4 lanes of the block)
};

// 8 bf16 values held by this lane; lanes 4j..4j+3 form one 32-element block.
__device__ __forceinline__ Quant8 quant8(const float (&v)[8]) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = mx_absmax_nan(m, v[i]);
  m = mx_max_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = mx_max_nan(m, __shfl_xor_sync(0xffffffffu, m, 2));
  Quant8 r;
  r.e = mx_e8m0_of_amax(m);
  const float rcp = mx_e8m0_rcp(r.e);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = mx_e4m3x2(mx_clamp448(v[2 * i] * rcp), mx_clamp448(v[2 * i + 1] * rcp));
  r.codes.x = w[0] | (w[1] << 16);
  r.codes.y = w[2] | (w[3] << 16);
  return r;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x);
  v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z);
  v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
}

// Loads the CTA's 128 x 128 tile (16 rows per pass, 16 lanes per row, 16 bytes per lane),
// quantizes it row-wise and/or stages it in shared memory for the column-wise pass.
template <bool ROWS, bool COLS>
__global__ void __launch_bounds__(QT) k_quant(const __nv_bfloat16* __restrict__ x, int64_t R, int64_t K, int64_t ldx,
                                             uint8_t* __restrict__ q, int64_t ldq, uint8_t* __restrict__ s,
                                             uint8_t* __restrict__ qt, uint8_t* __restrict__ st, int64_t s_tiles,
                                             int64_t tile_off) {
  __shared__ __align__(16) uint8_t s_rows[512];
  __shared__ __align__(16) uint8_t s_cols[512];
  extern __shared__ __align__(16) uint16_t s_tile[];  // [128][128] bf16 bits (COLS only)

  const int tid = threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.x * 128;
  const int64_t c0 = (int64_t)blockIdx.y * 128;
  const int rr = tid >> 4;        // row within a pass (0..15)
  const int c8 = (tid & 15) * 8;  // column offset of this lane's 8 elements

  uint4 u[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int64_t row = r0 + p * 16 + rr;
    if (row < R)
      u[p] = __ldg(reinterpret_cast<const uint4*>(x + row * ldx + c0 + c8));
    else
      u[p] = make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int rt = p * 16 + rr;  // row within the tile
    if (ROWS) {
      float v[8];
      unpack8(u[p], v);
      Quant8 qq = quant8(v);
      const int64_t row = r0 + rt;
      if (row < R) *reinterpret_cast<uint2*>(q + row * ldq + c0 + c8) = qq.codes;
      if ((tid & 3) == 0) s_rows[(rt & 31) * 16 + (rt >> 5) * 4 + (c8 >> 5)] = (uint8_t)qq.e;
    }
    if (COLS) *reinterpret_cast<uint4*>(s_tile + rt * 128 + c8) = u[p];
  }

  if (COLS) {
    __syncthreads();
    // thread -> (output row k = input column, r-blocks jb and jb + 2); a warp reads 32 adjacent
    // columns of one smem row at a time (64 contiguous bytes: conflict free).
    const int w = tid >> 5, l = tid & 31;
    const int k = (w & 3) * 32 + l;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int jb = (w >> 2) + 2 * jj;  // 32-row block of the tile (0..3)
      float m = 0.f;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v[i] = __uint_as_float((uint32_t)s_tile[(jb * 32 + i) * 128 + k] << 16);
        m = mx_absmax_nan(m, v[i]);
      }
      const uint32_t e = mx_e8m0_of_amax(m);
      const float rcp = mx_e8m0_rcp(e);
      uint32_t w4[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t a = mx_e4m3x2(mx_clamp448(v[4 * i] * rcp), mx_clamp448(v[4 * i + 1] * rcp));
        const uint32_t b = mx_e4m3x2(mx_clamp448(v[4 * i + 2] * rcp), mx_clamp448(v[4 * i + 3] * rcp));
        w4[i] = a | (b << 16);
      }
      uint8_t* dst = qt + (c0 + k) * R + r0 + jb * 32;
      reinterpret_cast<uint4*>(dst)[0] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      reinterpret_cast<uint4*>(dst)[1] = make_uint4(w4[4], w4[5], w4[6], w4[7]);
      s_cols[(k & 31) * 16 + (k >> 5) * 4 + jb] = (uint8_t)e;
    }
  }
  __syncthreads();
  if (tid < 32) {
    if (ROWS) {
      uint8_t* dst = s + ((int64_t)blockIdx.x * s_tiles + tile_off + blockIdx.y) * 512;
      reinterpret_cast<uint4*>(dst)[tid] = reinterpret_cast<const uint4*>(s_rows)[tid];
    }
  } else if (tid < 64) {
    if (COLS) {
      uint8_t* dst = st + ((int64_t)blockIdx.y * (R >> 7) + blockIdx.x) * 512;
      reinterpret_cast<uint4*>(dst)[tid - 32] = reinterpret_cast<const uint4*>(s_cols)[tid - 32];
    }
  }
}

int check_common(const void* x, int64_t R, int64_t K, int64_t ldx, const char* fn) {
  MX_CHECK_ARG(x != nullptr, "%s: null input", fn);
  MX_CHECK_ARG(R >= 1 && K >= 128 && K % 128 == 0, "%s: need R >= 1 and K %% 128 == 0 (R=%lld K=%lld)", fn,
               (long long)R, (long long)K);
  MX_CHECK_ARG(ldx >= K && ldx % 8 == 0, "%s: row stride %lld must be >= K and a multiple of 8", fn, (long long)ldx);
  MX_CHECK_ARG(mx_aligned(x, 16), "%s: input not 16-byte aligned", fn);
  MX_CHECK_ARG((R + 127) / 128 <= 0x7fffffff && K / 128 <= 65535, "%s: shape too large", fn);
  return MXM_OK;
}

// s_tiles / tile_off: the row-wise scales go to 128-column tiles tile_off .. of the blocked layout of an
// operand s_tiles * 128 columns wide (the codes' columns are placed by the caller through q).
template <bool ROWS, bool COLS>
int launch(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, int64_t ldq, void* s, void* qt, void* st,
           void* stream, int64_t s_tiles = -1, int64_t tile_off = 0) {
  if (s_tiles < 0) s_tiles = K >> 7;
  const size_t smem = COLS ? 128 * 128 * sizeof(uint16_t) : 0;
  if (COLS) {
    cudaError_t e = cudaFuncSetAttribute(k_quant<ROWS, COLS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "quant: set smem");
  }
  dim3 grid((unsigned)((R + 127) / 128), (unsigned)(K / 128));
  k_quant<ROWS, COLS><<<grid, QT, smem, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, R, K, ldx, (uint8_t*)q, ldq, (uint8_t*)s, (uint8_t*)qt, (uint8_t*)st, s_tiles, tile_off);
  mx_note_launch();
  return mx_launch_status("quant kernel launch");
}

}  // namespace

extern "C" int mxm_quant_rows(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, int64_t ldq, void* s,
                              void* stream) {
  if (int st = check_common(x, R, K, ldx, "mxm_quant_rows")) return st;
  MX_CHECK_ARG(q && s, "mxm_quant_rows: null output");
  MX_CHECK_ARG(ldq >= K && ldq % 8 == 0 && mx_aligned(q, 8), "mxm_quant_rows: bad code buffer stride/alignment");
  MX_CHECK_ARG(mx_aligned(s, 16), "mxm_quant_rows: scale buffer not 16-byte aligned");
  return launch<true, false>(x, R, K, ldx, q, ldq, s, nullptr, nullptr, stream);
}

// Row-wise MXFP8 of x [R, K] into columns col_tile_off*128 .. of a wider MX operand [R, s_cols]: codes at
// q[r * ldq + col_tile_off*128 + c], scales in that operand's blocked layout (reference lora_bwd's
// quantize-only mode, scripts/mxfp8.py:219-246, used to build one K-concatenated dy for a group's dx).
extern "C" int mxm_quant_rows_into(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, int64_t ldq, void* s,
                                   int64_t s_cols, int64_t col_tile_off, void* stream) {
  if (int st = check_common(x, R, K, ldx, "mxm_quant_rows_into")) return st;
  MX_CHECK_ARG(q && s, "mxm_quant_rows_into: null output");
  MX_CHECK_ARG(s_cols % 128 == 0 && col_tile_off >= 0 && (col_tile_off * 128 + K) <= s_cols && ldq >= s_cols &&
                   ldq % 8 == 0 && mx_aligned(q, 8) && mx_aligned(s, 16),
               "mxm_quant_rows_into: columns [%lld, %lld) outside the %lld-column operand or bad buffers",
               (long long)(col_tile_off * 128), (long long)(col_tile_off * 128 + K), (long long)s_cols);
  return launch<true, false>(x, R, K, ldx, (uint8_t*)q + col_tile_off * 128, ldq, s, nullptr, nullptr, stream,
                             s_cols >> 7, col_tile_off);
}

extern "C" int mxm_quant_cols(const void* x, int64_t R, int64_t K, int64_t ldx, void* qt, void* st, void* stream) {
  if (int e = check_common(x, R, K, ldx, "mxm_quant_cols")) return e;
  MX_CHECK_ARG(R % 128 == 0, "mxm_quant_cols: R (%lld) must be a multiple of 128", (long long)R);
  MX_CHECK_ARG(qt && st && mx_aligned(qt, 16) && mx_aligned(st, 16), "mxm_quant_cols: bad output buffers");
  return launch<false, true>(x, R, K, ldx, nullptr, 0, nullptr, qt, st, stream);
}

extern "C" int mxm_quant_both(const void* x, int64_t R, int64_t K, int64_t ldx, void* q, void* s, void* qt,
                              void* st, void* stream) {
  if (int e = check_common(x, R, K, ldx, "mxm_quant_both")) return e;
  MX_CHECK_ARG(R % 128 == 0, "mxm_quant_both: R (%lld) must be a multiple of 128", (long long)R);
  MX_CHECK_ARG(q && s && qt && st && mx_aligned(q, 8) && mx_aligned(s, 16) && mx_aligned(qt, 16) &&
                   mx_aligned(st, 16),
               "mxm_quant_both: bad output buffers");
  return launch<true, true>(x, R, K, ldx, q, K, s, qt, st, stream);
}
