// MXFP8 quantizer for sm_100a: bf16 -> E4M3 codes + E8M0 scales (one per 32 contiguous elements
// along the quantized axis), scales written directly in the 128x4 blocked layout the tcgen05
// block-scaled MMA consumes.  Algorithm of the reference _quant_kernel (scripts/mxfp8.py:46-75):
//   amax = max |x| over the block (NaN if the block holds a NaN)
//   e    = round-up-to-power-of-two(amax / 448) as E8M0        (from amax's bits: mx_e8m0_of_amax)
//   q    = e4m3_rne(clamp(x * rcp(e), -448, 448)),  rcp(e) = 2^(127-e) (special cases 0/254/255)
//
// A 128-row x 128-column tile is exactly one 512-byte scale block of the blocked layout, so its scales
// are assembled in shared memory and leave in one piece.  Two kernels: k_quant_tma (persistent, TMA in
// and out, used whenever the buffers are 16-byte aligned) and k_quant (one CTA per tile, 16-byte vector
// loads, the fallback).  Memory bound: 3.03 bytes moved per element one way, 4.06 for rows + columns
// from one read.
#include <algorithm>

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

// ------------------------------------------------------------------------------------------------ TMA path
// Persistent variant for aligned buffers: warp 8 streams 128 x 128 bf16 tiles (two [128 x 64] boxes,
// 128-byte swizzle) into a 3-stage ring; consumer warps 0-7 quantize each tile from shared memory and
// assemble its outputs -- row-wise codes [128 rows x 128 B], column-wise (transposed) codes [128 x 128 B],
// both in the 128-byte swizzled layout, and the two 512-byte scale blocks -- in one of two staging
// buffers, from which one thread writes them with TMA tensor stores and bulk copies while the next tile
// is quantized.  Row pass: two lanes per 32-element block (16 values each, one xor-shuffle for the
// abs-max); column pass: a lane owns two adjacent columns of one 32-row block, read as bf16 pairs, so
// both columns' abs-maxes come from one packed max.  The arithmetic per element is that of quant8.
constexpr int QM_ST = 3, QM_CONS = 8;
constexpr int QM_IN = 128 * 128 * 2;                 // 32 KB input tile
constexpr int QM_OUT = 128 * 128 * 2 + 1024;         // q tile + qt tile + two scale blocks
__host__ __device__ constexpr size_t qm_smem() { return 1024 + (size_t)QM_ST * QM_IN + 2 * (size_t)QM_OUT + 256; }

MX_DEV uint32_t qm_abs2(uint32_t a, uint32_t b) {   // packed |a| max |b| with NaN propagation
  uint32_t r;
  asm("{\n\t.reg .b32 x, y;\n\tabs.bf16x2 x, %1;\n\tabs.bf16x2 y, %2;\n\tmax.NaN.bf16x2 %0, x, y;\n\t}"
      : "=r"(r) : "r"(a), "r"(b));
  return r;
}
MX_DEV uint32_t qm_max2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
MX_DEV float qm_nanmax(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// Two products -> two E4M3 codes (RNE, satfinite: +-inf and |v| > 448 give +-448 as the clamp does);
// a NaN code comes out as 0x7F / 0xFF and is made canonical by qm_nan_canon4.
MX_DEV uint32_t qm_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
MX_DEV uint32_t qm_nan_canon4(uint32_t w) {   // E4M3 NaN bytes (S.1111.111) -> 0x7F
  const uint32_t m = ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
  return w & ~m;
}
MX_DEV void qm_lds128(uint32_t* r, uint32_t a) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
MX_DEV uint32_t qm_lds32(uint32_t a) {
  uint32_t r;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(r) : "r"(a));
  return r;
}
MX_DEV void qm_sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
MX_DEV void qm_bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}
// 16-byte chunk c of row r in a 128-byte-row tile with the 128-byte swizzle
MX_DEV uint32_t qm_sw(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

template <bool ROWS, bool COLS>
__global__ void __launch_bounds__(32 * (QM_CONS + 1), 1)
    k_quant_tma(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_q,
                const __grid_constant__ CUtensorMap tm_qt, uint8_t* __restrict__ s, uint8_t* __restrict__ st,
                int64_t R, int nrt, int nct, int64_t s_tiles, int64_t tile_off, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* outb = ring + QM_ST * QM_IN;   // 2 x [q 16 KB | qt 16 KB | row scales 512 | col scales 512]
  uint64_t* full = reinterpret_cast<uint64_t*>(outb + 2 * QM_OUT);
  uint64_t* empty = full + QM_ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = nrt * nct;
  if (threadIdx.x == 0) {
    for (int i = 0; i < QM_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], QM_CONS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == QM_CONS) {   // TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) break;
        const int tr = t / nct, tc = t % nct;
        uint8_t* dst = ring + stage * QM_IN;
        mbar_arrive_expect_tx(&full[stage], QM_IN);
        tma_load_2d(dst, &tm_x, &full[stage], tc * 128, tr * 128);
        tma_load_2d(dst + QM_IN / 2, &tm_x, &full[stage], tc * 128 + 64, tr * 128);
        ++issued;
        if (++stage == QM_ST) {
          stage = 0;
          phase ^= 1;
        }
      }
      for (int k = 0; k < QM_ST && k < issued; ++k) {   // no copy left in flight
        const int i = issued - 1 - k;
        mbar_wait(&full[i % QM_ST], (uint32_t)((i / QM_ST) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
      }
    }
    return;
  }

  const int tid = threadIdx.x;
  const uint32_t s_ring = smem_u32(ring), s_out = smem_u32(outb);
  int stage = 0, it = 0;
  uint32_t phase = 0;
  for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
    const int tr = t / nct, tc = t % nct;
    // a warp whose wait ran out skips the tile; the consumer warps give up together at the named barrier
    const bool ok = mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE);
    const uint32_t in = s_ring + (uint32_t)stage * QM_IN;           // box b at in + b * 16 KB
    const uint32_t ob = s_out + (uint32_t)(it & 1) * QM_OUT;
    const uint32_t oq = ob, oqt = ob + 16384, ors = ob + 32768, ocs = ob + 32768 + 512;
    uint8_t* rs = outb + (it & 1) * QM_OUT + 32768;
    uint8_t* cs = rs + 512;
    if (ROWS && ok) {
      // lane -> (row pair half, box, 16-column quarter of the box); a warp covers 4 rows x 128 columns
      const int q = lane & 3, rsub = (lane >> 2) & 1, box = (lane >> 3) & 1, rpair = lane >> 4;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t r = (uint32_t)(32 * p + 4 * warp + 2 * rpair + rsub);
        uint32_t v[8];
        qm_lds128(v, in + (uint32_t)box * 16384 + qm_sw(r, (uint32_t)(2 * q)));
        qm_lds128(v + 4, in + (uint32_t)box * 16384 + qm_sw(r, (uint32_t)(2 * q + 1)));
        const uint32_t m2 = qm_max2(qm_max2(qm_abs2(v[0], v[1]), qm_abs2(v[2], v[3])),
                                    qm_max2(qm_abs2(v[4], v[5]), qm_abs2(v[6], v[7])));
        float m = qm_nanmax(bf16_lo(m2), bf16_hi(m2));
        m = qm_nanmax(m, __shfl_xor_sync(0xffffffffu, m, 1));   // the other 16 of the 32-column block
        const uint32_t e = mx_e8m0_of_amax(m);
        const float rcp = mx_e8m0_rcp(e);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = qm_nan_canon4(qm_e4m3x2(bf16_lo(v[2 * i]) * rcp, bf16_hi(v[2 * i]) * rcp) |
                               (qm_e4m3x2(bf16_lo(v[2 * i + 1]) * rcp, bf16_hi(v[2 * i + 1]) * rcp) << 16));
        qm_sts128(oq + qm_sw(r, (uint32_t)(4 * box + q)), w[0], w[1], w[2], w[3]);
        if ((q & 1) == 0) rs[(r & 31) * 16 + (r >> 5) * 4 + 2 * box + (q >> 1)] = (uint8_t)e;
      }
    }
    if (COLS && ok) {
      // warp -> (32-row block jb, box); lane -> columns 2 lane, 2 lane + 1 of the box
      const int jb = warp >> 1, box = warp & 1;
      const uint32_t base = in + (uint32_t)box * 16384 + (uint32_t)((lane & 3) * 4);
      uint32_t v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint32_t r = (uint32_t)(32 * jb + i);
        v[i] = qm_lds32(base + qm_sw(r, (uint32_t)(lane >> 2)));
      }
      uint32_t a[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) a[i] = qm_abs2(v[2 * i], v[2 * i + 1]);
#pragma unroll
      for (int s2 = 8; s2 >= 1; s2 >>= 1)
#pragma unroll
        for (int i = 0; i < s2; ++i) a[i] = qm_max2(a[i], a[i + s2]);
      const uint32_t e0 = mx_e8m0_of_amax(bf16_lo(a[0])), e1 = mx_e8m0_of_amax(bf16_hi(a[0]));
      const float r0 = mx_e8m0_rcp(e0), r1 = mx_e8m0_rcp(e1);
      uint32_t w0[8], w1[8];   // codes of column 2 lane (w0) and 2 lane + 1 (w1), rows 32 jb + 4 i ..
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t x0 = v[4 * i], x1 = v[4 * i + 1], x2 = v[4 * i + 2], x3 = v[4 * i + 3];
        w0[i] = qm_nan_canon4(qm_e4m3x2(bf16_lo(x0) * r0, bf16_lo(x1) * r0) |
                              (qm_e4m3x2(bf16_lo(x2) * r0, bf16_lo(x3) * r0) << 16));
        w1[i] = qm_nan_canon4(qm_e4m3x2(bf16_hi(x0) * r1, bf16_hi(x1) * r1) |
                              (qm_e4m3x2(bf16_hi(x2) * r1, bf16_hi(x3) * r1) << 16));
      }
      const uint32_t c0 = (uint32_t)(64 * box + 2 * lane), c1 = c0 + 1;   // output rows of the qt tile
      qm_sts128(oqt + qm_sw(c0, (uint32_t)(2 * jb)), w0[0], w0[1], w0[2], w0[3]);
      qm_sts128(oqt + qm_sw(c0, (uint32_t)(2 * jb + 1)), w0[4], w0[5], w0[6], w0[7]);
      qm_sts128(oqt + qm_sw(c1, (uint32_t)(2 * jb)), w1[0], w1[1], w1[2], w1[3]);
      qm_sts128(oqt + qm_sw(c1, (uint32_t)(2 * jb + 1)), w1[4], w1[5], w1[6], w1[7]);
      cs[(c0 & 31) * 16 + (c0 >> 5) * 4 + jb] = (uint8_t)e0;
      cs[(c1 & 31) * 16 + (c1 >> 5) * 4 + jb] = (uint8_t)e1;
    }
    fence_proxy_async();   // the staged outputs are read by the bulk stores below
    __syncwarp();
    if (lane == 0 && ok) mbar_arrive(&empty[stage]);
    if (++stage == QM_ST) {
      stage = 0;
      phase ^= 1;
    }
    if (tid == 0) bulk_wait_read0();   // the previous tile's stores have read the other staging buffer
    if (bar_any(1, 32 * QM_CONS, !ok)) break;
    if (tid == 0) {
      if (ROWS) {
        tma_store_2d(&tm_q, outb + (it & 1) * QM_OUT, tc * 128, tr * 128);
        qm_bulk_store(s + ((int64_t)tr * s_tiles + tile_off + tc) * 512, ors, 512);
      }
      if (COLS) {
        tma_store_2d(&tm_qt, outb + (it & 1) * QM_OUT + 16384, tr * 128, tc * 128);
        qm_bulk_store(st + ((int64_t)tc * nrt + tr) * 512, ocs, 512);
      }
      bulk_commit();
    }
  }
  if (tid == 0) bulk_wait0();
  (void)R;
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
  // TMA path: 16-byte aligned rows and buffers (tensor maps), the codes' row stride a multiple of 16
  const bool tma_ok = mx_aligned(x, 16) && ldx % 8 == 0 &&
                      (!ROWS || (mx_aligned(q, 16) && ldq % 16 == 0 && mx_aligned(s, 16))) &&
                      (!COLS || (mx_aligned(qt, 16) && mx_aligned(st, 16) && R % 16 == 0));
  if (tma_ok) {   // from here on a failure is an error, not a reason to fall back
    CUtensorMap tx, tq, tqt;
    int e = mx_make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)K, (uint64_t)R,
                            (uint64_t)(ldx * 2), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!e && ROWS)
      e = mx_make_tmap_2d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, (uint64_t)K, (uint64_t)R, (uint64_t)ldq, 128, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (!e && COLS)
      e = mx_make_tmap_2d(&tqt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qt, (uint64_t)R, (uint64_t)K, (uint64_t)R, 128, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    {
      if (!ROWS) tq = tqt;
      if (!COLS) tqt = tq;
      const int nrt = (int)((R + 127) / 128), nct = (int)(K / 128);
      const int64_t tiles = (int64_t)nrt * nct;
      const int grid = (int)std::min<int64_t>(tiles, mxm_num_sms());
      const size_t smem = qm_smem();
      cudaError_t ce = mx_smem_attr((const void*)k_quant_tma<ROWS, COLS>, smem);
      if (ce != cudaSuccess) return mx_cuda_status(ce, "quant tma: set smem");
      k_quant_tma<ROWS, COLS><<<grid, 32 * (QM_CONS + 1), smem, (cudaStream_t)stream>>>(
          tx, tq, tqt, (uint8_t*)s, (uint8_t*)st, R, nrt, nct, s_tiles, tile_off, mx_dev_error_ptr());
      mx_note_launch();
      return mx_launch_status("quant tma kernel launch");
    }
  }
  const size_t smem = COLS ? 128 * 128 * sizeof(uint16_t) : 0;
  if (COLS) {
    cudaError_t e = mx_smem_attr((const void*)k_quant<ROWS, COLS>, smem);
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
