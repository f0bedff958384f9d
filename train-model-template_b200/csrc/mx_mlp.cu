// The memory-bound passes of the fused SwiGLU-LoRA MLP (reference scripts/fused_mlp.py) on sm_100a.
//
//   k_mlp_fwd   -- the forward epilogue (reference _fwd_kernel, scripts/fused_mlp.py:81-109):
//                  reads gu = [x W_gate^T | x W_up^T] once, adds the LoRA-B terms, SwiGLU, writes h as
//                  MXFP8 (codes + blocked scales) for the down GEMM and xS_down = h A_down^T.
//   k_mlp_bwd   -- the backward epilogue (reference _bwd_kernel, scripts/fused_mlp.py:112-175):
//                  recomputes g, u, h from gu, dh = dh_mx + dxd A_down, SwiGLU backward, writes
//                  [dg | du] as MXFP8 for the dx GEMM, and the LoRA gradient pieces dB_gate, dB_up,
//                  dA_down (summed over rows) and dxa_gate, dxa_up, xS_down (summed over columns).
//   k_rowdot    -- out[T, n] = A[T, K] B[n, K]^T for the rank-n LoRA-A products (x S^T, dy B_down).
//   k_coldot    -- out[K, n] = A[T, K]^T E[T, n] for the LoRA weight gradients (dA, dB_down).
//   k_sum_*     -- fixed-order sums of the per-CTA partial buffers (deterministic, no atomics).
//
// All rank-r products run on the tensor cores with warp-level m16n8k16 bf16 MMAs; the element-wise
// math keeps the reference's rounding points (bf16 after each fp32 expression it rounds).
#include "mx_mma.cuh"
#include "mx_runtime.h"

namespace {

using bf16 = __nv_bfloat16;

// Quantizes one 32-column block of a 16-row warp tile in D-fragment form:
// v[i][0..1] = (row g, cols 8i+2t, +1), v[i][2..3] = (row g+8, same cols), i = 0..3.
// Codes go to q[row * ldq + col0 + ...] for rows < T; scales of rows g and g+8 (always, padded rows
// included) to the blocked layout of a [*, scols] operand.
MX_DEV void quant_block16(const float (&v)[4][4], int64_t row_g, int64_t T, int64_t col0, uint8_t* q, int64_t ldq,
                          uint8_t* s, int64_t scols, int t) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) m = mx_absmax_nan(m, mx_absmax_nan(v[i][2 * h], v[i][2 * h + 1]));
    m = mx_max_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = mx_max_nan(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const uint32_t e = mx_e8m0_rceil(__fdiv_rn(m, 448.0f));
    const float rcp = mx_e8m0_rcp(e);
    const int64_t row = row_g + 8 * h;
    if (row < T) {
      uint8_t* dst = q + row * ldq + col0 + 2 * t;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint16_t*>(dst + 8 * i) =
            mx_e4m3x2(mx_clamp448(v[i][2 * h] * rcp), mx_clamp448(v[i][2 * h + 1] * rcp));
    }
    if (t == 0) s[mx_scale_offset(row, col0 >> 5, scols)] = (uint8_t)e;
  }
}

MX_DEV float silu_part(float g) { return g / (expf(-g) + 1.0f); }

// ------------------------------------------------------------------------------------------------ forward
// CTA = 4 warps x 16 rows; blockIdx.y = column group of `tpg` tiles of BN columns.
template <int R, int BN>
__global__ void __launch_bounds__(128) k_mlp_fwd(const bf16* __restrict__ gu, const bf16* __restrict__ xs,
                                                 const bf16* __restrict__ bg, const bf16* __restrict__ bu,
                                                 const bf16* __restrict__ ad, uint8_t* __restrict__ qh,
                                                 uint8_t* __restrict__ sh, float* __restrict__ xsd_part,
                                                 bf16* __restrict__ xsd_out, int T, int N, float s_g, float s_u,
                                                 int tpg, int write_q) {
  constexpr int KS = R / 16, NT = BN / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t row0 = (int64_t)blockIdx.x * 64 + warp * 16;
  const int64_t ra = row0 + g, rb = ra + 8;
  const bool va = ra < T, vb = rb < T;
  const int64_t N2 = 2 * (int64_t)N;

  uint32_t axg[KS][4], axu[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const bf16* pa = xs + ra * (2 * R) + 16 * kk + 2 * t;
    const bf16* pb = xs + rb * (2 * R) + 16 * kk + 2 * t;
    axg[kk][0] = va ? ld32(pa) : 0u;
    axg[kk][1] = vb ? ld32(pb) : 0u;
    axg[kk][2] = va ? ld32(pa + 8) : 0u;
    axg[kk][3] = vb ? ld32(pb + 8) : 0u;
    axu[kk][0] = va ? ld32(pa + R) : 0u;
    axu[kk][1] = vb ? ld32(pb + R) : 0u;
    axu[kk][2] = va ? ld32(pa + R + 8) : 0u;
    axu[kk][3] = vb ? ld32(pb + R + 8) : 0u;
  }
  float accx[R / 8][4];
#pragma unroll
  for (int j = 0; j < R / 8; ++j) accx[j][0] = accx[j][1] = accx[j][2] = accx[j][3] = 0.f;

  for (int ct = 0; ct < tpg; ++ct) {
    const int n0 = (blockIdx.y * tpg + ct) * BN;
    float hv[NT][4];
    uint32_t hp[NT][2];
    // issue the tile's gu loads first (independent, overlapping latency)
    uint32_t ga[NT], gb[NT], ua[NT], ub[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int64_t c = n0 + 8 * i + 2 * t;
      ga[i] = va ? ld32(gu + ra * N2 + c) : 0u;
      gb[i] = vb ? ld32(gu + rb * N2 + c) : 0u;
      ua[i] = va ? ld32(gu + ra * N2 + N + c) : 0u;
      ub[i] = vb ? ld32(gu + rb * N2 + N + c) : 0u;
    }
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int nc = n0 + 8 * i;
      float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const bf16* pbg = bg + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
        const bf16* pbu = bu + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
        mma16816(dg, axg[kk], ld32g(pbg), ld32g(pbg + 8));
        mma16816(du, axu[kk], ld32g(pbu), ld32g(pbu + 8));
      }
      const float gin[4] = {bf16_lo(ga[i]), bf16_hi(ga[i]), bf16_lo(gb[i]), bf16_hi(gb[i])};
      const float uin[4] = {bf16_lo(ua[i]), bf16_hi(ua[i]), bf16_lo(ub[i]), bf16_hi(ub[i])};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gg = bf16_round_f(gin[e] + s_g * dg[e]);
        const float uu = bf16_round_f(uin[e] + s_u * du[e]);
        hv[i][e] = bf16_round_f(silu_part(gg) * uu);
      }
      hp[i][0] = pack_bf16x2(hv[i][0], hv[i][1]);
      hp[i][1] = pack_bf16x2(hv[i][2], hv[i][3]);
    }
    if (write_q) {
#pragma unroll
      for (int b = 0; b < BN / 32; ++b) {
        const float(&blk)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&hv[4 * b][0]);
        quant_block16(blk, row0 + g, T, n0 + 32 * b, qh, N, sh, N, t);
      }
    }
#pragma unroll
    for (int m = 0; m < BN / 16; ++m) {
      const uint32_t a[4] = {hp[2 * m][0], hp[2 * m][1], hp[2 * m + 1][0], hp[2 * m + 1][1]};
#pragma unroll
      for (int jt = 0; jt < R / 8; ++jt) {
        const bf16* pad = ad + (int64_t)(8 * jt + g) * N + n0 + 16 * m + 2 * t;
        mma16816(accx[jt], a, ld32g(pad), ld32g(pad + 8));
      }
    }
  }
#pragma unroll
  for (int jt = 0; jt < R / 8; ++jt) {
    const int c = 8 * jt + 2 * t;
    if (xsd_out) {
      if (va) *reinterpret_cast<uint32_t*>(xsd_out + ra * R + c) = pack_bf16x2(accx[jt][0], accx[jt][1]);
      if (vb) *reinterpret_cast<uint32_t*>(xsd_out + rb * R + c) = pack_bf16x2(accx[jt][2], accx[jt][3]);
    } else {
      float* P = xsd_part + (int64_t)blockIdx.y * T * R;
      if (va) *reinterpret_cast<float2*>(P + ra * R + c) = make_float2(accx[jt][0], accx[jt][1]);
      if (vb) *reinterpret_cast<float2*>(P + rb * R + c) = make_float2(accx[jt][2], accx[jt][3]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ backward
// CTA = 4 warps; blockIdx.x = super-block of SB rows, blockIdx.y = column group of tpg tiles.
// Column tiles outer (dB / dA accumulate in registers over the super-block's rows), rows inner
// (dxa / xS_down accumulate across the group's tiles in the group's partial rows, which only this
// thread touches).
template <int R, int BN>
__global__ void __launch_bounds__(128) k_mlp_bwd(
    const bf16* __restrict__ gu, const bf16* __restrict__ xs, const bf16* __restrict__ dhm,
    const bf16* __restrict__ dxd, const bf16* __restrict__ bg, const bf16* __restrict__ bu,
    const bf16* __restrict__ ad, uint8_t* __restrict__ q, uint8_t* __restrict__ s, float* __restrict__ dxa_part,
    float* __restrict__ dbg_part, float* __restrict__ dbu_part, float* __restrict__ dad_part, int T, int Tpad, int N,
    float s_g, float s_u, int SB, int tpg, int write_q) {
  constexpr int KS = R / 16, NT = BN / 8, R3 = 3 * R;
  extern __shared__ float red[];  // [4 warps][3][R][BN]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int sbi = blockIdx.x, cg = blockIdx.y;
  const int r_begin = sbi * SB, r_end = min(r_begin + SB, Tpad);
  const int64_t N2 = 2 * (int64_t)N;
  float* P = dxa_part + (int64_t)cg * T * R3;

  for (int ct = 0; ct < tpg; ++ct) {
    const int n0 = (cg * tpg + ct) * BN;
    float aBg[KS][NT][4], aBu[KS][NT][4], aAd[KS][NT][4];
#pragma unroll
    for (int a = 0; a < KS; ++a)
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) aBg[a][i][e] = aBu[a][i][e] = aAd[a][i][e] = 0.f;

    for (int r = r_begin + warp * 16; r < r_end; r += 64) {
      const int64_t ra = r + g, rb = ra + 8;
      const bool va = ra < T, vb = rb < T;
      uint32_t axg[KS][4], axu[KS][4], axd[KS][4];
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const bf16* pa = xs + ra * (2 * R) + 16 * kk + 2 * t;
        const bf16* pb = xs + rb * (2 * R) + 16 * kk + 2 * t;
        const bf16* da = dxd + ra * R + 16 * kk + 2 * t;
        const bf16* db = dxd + rb * R + 16 * kk + 2 * t;
        axg[kk][0] = va ? ld32(pa) : 0u;
        axg[kk][1] = vb ? ld32(pb) : 0u;
        axg[kk][2] = va ? ld32(pa + 8) : 0u;
        axg[kk][3] = vb ? ld32(pb + 8) : 0u;
        axu[kk][0] = va ? ld32(pa + R) : 0u;
        axu[kk][1] = vb ? ld32(pb + R) : 0u;
        axu[kk][2] = va ? ld32(pa + R + 8) : 0u;
        axu[kk][3] = vb ? ld32(pb + R + 8) : 0u;
        axd[kk][0] = va ? ld32(da) : 0u;
        axd[kk][1] = vb ? ld32(db) : 0u;
        axd[kk][2] = va ? ld32(da + 8) : 0u;
        axd[kk][3] = vb ? ld32(db + 8) : 0u;
      }
      uint32_t dgp[NT][2], dup[NT][2], hp[NT][2];
      float dgv[NT][4], duv[NT][4];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int nc = n0 + 8 * i;
        const int64_t c = nc + 2 * t;
        const uint32_t ga = va ? ld32(gu + ra * N2 + c) : 0u, gb = vb ? ld32(gu + rb * N2 + c) : 0u;
        const uint32_t ua = va ? ld32(gu + ra * N2 + N + c) : 0u, ub = vb ? ld32(gu + rb * N2 + N + c) : 0u;
        const uint32_t ha = va ? ld32(dhm + ra * N + c) : 0u, hb = vb ? ld32(dhm + rb * N + c) : 0u;
        float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f}, dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const bf16* pbg = bg + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
          const bf16* pbu = bu + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
          mma16816(dg, axg[kk], ld32g(pbg), ld32g(pbg + 8));
          mma16816(du, axu[kk], ld32g(pbu), ld32g(pbu + 8));
          // B[k = j][n] = A_down[j][n]: (j 2t..2t+1, col g)
          const bf16* p0 = ad + (int64_t)(16 * kk + 2 * t) * N + nc + g;
          mma16816(dd, axd[kk], ld16x2(p0, p0 + N), ld16x2(p0 + 8 * (int64_t)N, p0 + 9 * (int64_t)N));
        }
        const float gin[4] = {bf16_lo(ga), bf16_hi(ga), bf16_lo(gb), bf16_hi(gb)};
        const float uin[4] = {bf16_lo(ua), bf16_hi(ua), bf16_lo(ub), bf16_hi(ub)};
        const float hin[4] = {bf16_lo(ha), bf16_hi(ha), bf16_lo(hb), bf16_hi(hb)};
        float hvv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float gg = bf16_round_f(gin[e] + s_g * dg[e]);
          const float uu = bf16_round_f(uin[e] + s_u * du[e]);
          const float sl = silu_part(gg);
          hvv[e] = bf16_round_f(sl * uu);
          const float dh = bf16_round_f(hin[e] + dd[e]);
          duv[i][e] = bf16_round_f(dh * sl);
          const float sig = 1.0f / (1.0f + expf(-gg));
          dgv[i][e] = bf16_round_f(((dh * uu) * sig) * (gg * (1.0f - sig) + 1.0f));
        }
        hp[i][0] = pack_bf16x2(hvv[0], hvv[1]);
        hp[i][1] = pack_bf16x2(hvv[2], hvv[3]);
        dgp[i][0] = pack_bf16x2(dgv[i][0], dgv[i][1]);
        dgp[i][1] = pack_bf16x2(dgv[i][2], dgv[i][3]);
        dup[i][0] = pack_bf16x2(duv[i][0], duv[i][1]);
        dup[i][1] = pack_bf16x2(duv[i][2], duv[i][3]);
      }
      if (write_q) {
#pragma unroll
        for (int b = 0; b < BN / 32; ++b) {
          const float(&bgv)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&dgv[4 * b][0]);
          const float(&buv)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&duv[4 * b][0]);
          quant_block16(bgv, r + g, T, n0 + 32 * b, q, N2, s, N2, t);
          quant_block16(buv, r + g, T, (int64_t)N + n0 + 32 * b, q, N2, s, N2, t);
        }
      }
      // per-row products, accumulated across the group's column tiles
      float pg[R / 8][4], pu[R / 8][4], px[R / 8][4];
#pragma unroll
      for (int jt = 0; jt < R / 8; ++jt) {
        const int c = 8 * jt + 2 * t;
        float2 z = make_float2(0.f, 0.f);
        float2 g0 = z, g1 = z, u0 = z, u1 = z, x0 = z, x1 = z;
        if (ct > 0) {
          if (va) {
            g0 = *reinterpret_cast<const float2*>(P + ra * R3 + c);
            u0 = *reinterpret_cast<const float2*>(P + ra * R3 + R + c);
            x0 = *reinterpret_cast<const float2*>(P + ra * R3 + 2 * R + c);
          }
          if (vb) {
            g1 = *reinterpret_cast<const float2*>(P + rb * R3 + c);
            u1 = *reinterpret_cast<const float2*>(P + rb * R3 + R + c);
            x1 = *reinterpret_cast<const float2*>(P + rb * R3 + 2 * R + c);
          }
        }
        pg[jt][0] = g0.x; pg[jt][1] = g0.y; pg[jt][2] = g1.x; pg[jt][3] = g1.y;
        pu[jt][0] = u0.x; pu[jt][1] = u0.y; pu[jt][2] = u1.x; pu[jt][3] = u1.y;
        px[jt][0] = x0.x; px[jt][1] = x0.y; px[jt][2] = x1.x; px[jt][3] = x1.y;
      }
#pragma unroll
      for (int m = 0; m < BN / 16; ++m) {
        const uint32_t adg[4] = {dgp[2 * m][0], dgp[2 * m][1], dgp[2 * m + 1][0], dgp[2 * m + 1][1]};
        const uint32_t adu[4] = {dup[2 * m][0], dup[2 * m][1], dup[2 * m + 1][0], dup[2 * m + 1][1]};
        const uint32_t ah[4] = {hp[2 * m][0], hp[2 * m][1], hp[2 * m + 1][0], hp[2 * m + 1][1]};
#pragma unroll
        for (int jt = 0; jt < R / 8; ++jt) {
          const int j = 8 * jt + g;
          const int64_t nn = n0 + 16 * m + 2 * t;
          const bf16* pb = bg + nn * R + j;
          mma16816(pg[jt], adg, ld16x2(pb, pb + R), ld16x2(pb + 8 * R, pb + 9 * R));
          const bf16* pu_ = bu + nn * R + j;
          mma16816(pu[jt], adu, ld16x2(pu_, pu_ + R), ld16x2(pu_ + 8 * R, pu_ + 9 * R));
          const bf16* pad = ad + (int64_t)j * N + nn;
          mma16816(px[jt], ah, ld32g(pad), ld32g(pad + 8));
        }
      }
#pragma unroll
      for (int jt = 0; jt < R / 8; ++jt) {
        const int c = 8 * jt + 2 * t;
        if (va) {
          *reinterpret_cast<float2*>(P + ra * R3 + c) = make_float2(pg[jt][0], pg[jt][1]);
          *reinterpret_cast<float2*>(P + ra * R3 + R + c) = make_float2(pu[jt][0], pu[jt][1]);
          *reinterpret_cast<float2*>(P + ra * R3 + 2 * R + c) = make_float2(px[jt][0], px[jt][1]);
        }
        if (vb) {
          *reinterpret_cast<float2*>(P + rb * R3 + c) = make_float2(pg[jt][2], pg[jt][3]);
          *reinterpret_cast<float2*>(P + rb * R3 + R + c) = make_float2(pu[jt][2], pu[jt][3]);
          *reinterpret_cast<float2*>(P + rb * R3 + 2 * R + c) = make_float2(px[jt][2], px[jt][3]);
        }
      }
      // column products: [j x n] += xa^T (j x rows) . [dg | du | h] (rows x n)
#pragma unroll
      for (int jm = 0; jm < KS; ++jm) {
        const uint32_t tg[4] = {movtrans(axg[jm][0]), movtrans(axg[jm][2]), movtrans(axg[jm][1]), movtrans(axg[jm][3])};
        const uint32_t tu[4] = {movtrans(axu[jm][0]), movtrans(axu[jm][2]), movtrans(axu[jm][1]), movtrans(axu[jm][3])};
        const uint32_t td[4] = {movtrans(axd[jm][0]), movtrans(axd[jm][2]), movtrans(axd[jm][1]), movtrans(axd[jm][3])};
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          mma16816(aBg[jm][i], tg, movtrans(dgp[i][0]), movtrans(dgp[i][1]));
          mma16816(aBu[jm][i], tu, movtrans(dup[i][0]), movtrans(dup[i][1]));
          mma16816(aAd[jm][i], td, movtrans(hp[i][0]), movtrans(hp[i][1]));
        }
      }
    }
    // cross-warp reduction of the column products (fixed order), one partial per super-block
    float* W = red + warp * (3 * R * BN);
#pragma unroll
    for (int jm = 0; jm < KS; ++jm)
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int j0 = 16 * jm + g, nn = 8 * i + 2 * t;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = j0 + (e >> 1) * 8, n = nn + (e & 1);
          W[(0 * R + j) * BN + n] = aBg[jm][i][e];
          W[(1 * R + j) * BN + n] = aBu[jm][i][e];
          W[(2 * R + j) * BN + n] = aAd[jm][i][e];
        }
      }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 3 * R * BN; idx += blockDim.x) {
      const float v = red[idx] + red[3 * R * BN + idx] + red[2 * 3 * R * BN + idx] + red[3 * 3 * R * BN + idx];
      const int which = idx / (R * BN), rem = idx % (R * BN), j = rem / BN, n = rem % BN;
      if (which == 0)
        dbg_part[((int64_t)sbi * N + n0 + n) * R + j] = v;
      else if (which == 1)
        dbu_part[((int64_t)sbi * N + n0 + n) * R + j] = v;
      else
        dad_part[((int64_t)sbi * R + j) * N + n0 + n] = v;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ skinny
// out[t, j] = bf16( bf16(sum_k A[t, k] B[j, k]) * post ) for j < n (n = 16 or 32); post == 1 skips
// the second rounding.  Warp = 16 rows; the reduction index k is permuted consistently in A and B
// so each lane loads 16 contiguous bytes per row per 32 k.
template <int NJ>
__global__ void __launch_bounds__(128) k_rowdot(const bf16* __restrict__ A, int64_t lda, const bf16* __restrict__ B,
                                                int T, int K, float post, bf16* __restrict__ out, int64_t ldo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t ra = ((int64_t)blockIdx.x * 4 + warp) * 16 + g, rb = ra + 8;
  const bool va = ra < T, vb = rb < T;
  float acc[NJ / 8][4];
#pragma unroll
  for (int j = 0; j < NJ / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int k0 = 0; k0 < K; k0 += 32) {
    const uint4 xa = va ? __ldg(reinterpret_cast<const uint4*>(A + ra * lda + k0 + 8 * t)) : z;
    const uint4 xb = vb ? __ldg(reinterpret_cast<const uint4*>(A + rb * lda + k0 + 8 * t)) : z;
    // fragment k slots (2t, 2t+1 | 2t+8, 2t+9) <- actual k (8t, 8t+1 | 8t+2, 8t+3), then (8t+4.. | 8t+6..)
    const uint32_t a0[4] = {xa.x, xb.x, xa.y, xb.y};
    const uint32_t a1[4] = {xa.z, xb.z, xa.w, xb.w};
#pragma unroll
    for (int jt = 0; jt < NJ / 8; ++jt) {
      const uint4 bb = __ldg(reinterpret_cast<const uint4*>(B + (int64_t)(8 * jt + g) * K + k0 + 8 * t));
      mma16816(acc[jt], a0, bb.x, bb.y);
      mma16816(acc[jt], a1, bb.z, bb.w);
    }
  }
#pragma unroll
  for (int jt = 0; jt < NJ / 8; ++jt) {
    const int c = 8 * jt + 2 * t;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[e] = bf16_round_f(acc[jt][e]);
      if (post != 1.0f) v[e] = bf16_round_f(v[e] * post);
    }
    if (va) *reinterpret_cast<uint32_t*>(out + ra * ldo + c) = pack_bf16x2(v[0], v[1]);
    if (vb) *reinterpret_cast<uint32_t*>(out + rb * ldo + c) = pack_bf16x2(v[2], v[3]);
  }
}

// part[chunk, k, j] = sum over the chunk's rows t of A[t, k] E[t, j]   (k < K, j < NJ)
// Warp = 16 consecutive k columns x all NJ; CTA = 4 warps = 64 columns; blockIdx.y = row chunk.
// A^T fragments come from A row-fragments through movmatrix; E is read as the B operand.
template <int NJ>
__global__ void __launch_bounds__(128) k_coldot(const bf16* __restrict__ A, int64_t lda, const bf16* __restrict__ E,
                                                int64_t lde, int T, int K, int rows_per_chunk,
                                                float* __restrict__ part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int k0 = (blockIdx.x * 4 + warp) * 16;
  if (k0 >= K) return;
  const int r0 = blockIdx.y * rows_per_chunk, r1 = min(r0 + rows_per_chunk, T);
  float acc[NJ / 8][4];
#pragma unroll
  for (int j = 0; j < NJ / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  for (int r = r0; r < r1; r += 16) {
    const int64_t ra = r + g, rb = ra + 8;
    const bool va = ra < r1, vb = rb < r1;
    // A tile [16 rows x 16 k] in row-fragment form, then transposed into the A operand [k x rows]
    const bf16* pa = A + ra * lda + k0 + 2 * t;
    const bf16* pb = A + rb * lda + k0 + 2 * t;
    const uint32_t f0 = va ? ld32g(pa) : 0u, f1 = vb ? ld32g(pb) : 0u;
    const uint32_t f2 = va ? ld32g(pa + 8) : 0u, f3 = vb ? ld32g(pb + 8) : 0u;
    const uint32_t at[4] = {movtrans(f0), movtrans(f2), movtrans(f1), movtrans(f3)};
#pragma unroll
    for (int jt = 0; jt < NJ / 8; ++jt) {
      // B[k = rows][col j]: (rows 2t..2t+1, col g)
      const int64_t r2 = r + 2 * t;
      const bf16* pe = E + r2 * lde + 8 * jt + g;
      const uint32_t b0 = ld16z(pe, r2 < r1) | (ld16z(pe + lde, r2 + 1 < r1) << 16);
      const uint32_t b1 = ld16z(pe + 8 * lde, r2 + 8 < r1) | (ld16z(pe + 9 * lde, r2 + 9 < r1) << 16);
      mma16816(acc[jt], at, b0, b1);
    }
  }
  float* P = part + (int64_t)blockIdx.y * K * NJ;
#pragma unroll
  for (int jt = 0; jt < NJ / 8; ++jt) {
    const int j = 8 * jt + 2 * t;
    *reinterpret_cast<float2*>(P + (int64_t)(k0 + g) * NJ + j) = make_float2(acc[jt][0], acc[jt][1]);
    *reinterpret_cast<float2*>(P + (int64_t)(k0 + g + 8) * NJ + j) = make_float2(acc[jt][2], acc[jt][3]);
  }
}

// out[i] = scale * sum_{p < nparts} src[p * stride + i]   (fixed order); bf16 or fp32 output,
// optionally transposed: element i = (a, b) of an [A, B] matrix written at out[b * A + a].
__global__ void k_sum_parts(const float* __restrict__ src, int nparts, int64_t n, int64_t stride, float scale,
                            float post, float* __restrict__ out_f, bf16* __restrict__ out_h, int64_t tr_a,
                            int64_t tr_b) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int p = 0; p < nparts; ++p) v += src[p * stride + i];
    v *= scale;
    int64_t o = i;
    if (tr_a > 0) o = (i % tr_b) * tr_a + i / tr_b;
    if (out_h) {
      float r = bf16_round_f(v);
      if (post != 1.0f) r = bf16_round_f(r * post);
      out_h[o] = __float2bfloat16_rn(r);
    } else {
      out_f[o] = v;
    }
  }
}

// dxa partials [nparts, T, 3R] -> dxa bf16 [T, 2R] (gate part x s_g, up part x s_u) and xS_down bf16 [T, R].
__global__ void k_reduce_dxa(const float* __restrict__ src, int nparts, int T, int R, float s_g, float s_u,
                             bf16* __restrict__ dxa, bf16* __restrict__ xsd) {
  const int64_t n = (int64_t)T * 3 * R;
  const int64_t stride = n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int p = 0; p < nparts; ++p) v += src[p * stride + i];
    const int64_t row = i / (3 * R);
    const int c = (int)(i % (3 * R));
    if (c < R)
      dxa[row * 2 * R + c] = __float2bfloat16_rn(v * s_g);
    else if (c < 2 * R)
      dxa[row * 2 * R + c] = __float2bfloat16_rn(v * s_u);
    else
      xsd[row * R + c - 2 * R] = __float2bfloat16_rn(v);
  }
}

int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)mxm_num_sms() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

// ================================================================================================ C ABI
extern "C" int mxm_mlp_fwd_partitions(int64_t T, int64_t N, int r, int* col_groups) {
  MX_CHECK_ARG(T >= 1 && N >= 128 && N % 128 == 0 && (r == 16 || r == 32) && col_groups, "mxm_mlp_fwd_partitions: bad args");
  const int64_t tpad = (T + 127) / 128 * 128;
  const int64_t nrb = tpad / 64;
  const int nt = (int)(N / 128);
  int cs = nt;
  for (int d = 1; d <= nt; ++d)
    if (nt % d == 0 && nrb * d >= 4 * (int64_t)mxm_num_sms()) {
      cs = d;
      break;
    }
  *col_groups = cs;
  return MXM_OK;
}

extern "C" int mxm_mlp_fwd_epilogue(const void* gu, const void* xs, const void* bg, const void* bu, const void* ad,
                                    int64_t T, int64_t N, int r, float s_g, float s_u, void* qh, void* sh,
                                    void* xsd, void* xsd_part, int col_groups, void* stream) {
  MX_CHECK_ARG(gu && xs && bg && bu && ad && xsd, "mxm_mlp_fwd_epilogue: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32),
               "mxm_mlp_fwd_epilogue: need T >= 1, N %% 128 == 0, r in {16, 32}");
  MX_CHECK_ARG((qh == nullptr) == (sh == nullptr), "mxm_mlp_fwd_epilogue: qh and sh go together");
  const int nt = (int)(N / 128);
  MX_CHECK_ARG(col_groups >= 1 && nt % col_groups == 0, "mxm_mlp_fwd_epilogue: col_groups must divide N/128");
  MX_CHECK_ARG(col_groups == 1 || xsd_part, "mxm_mlp_fwd_epilogue: partial buffer needed for col_groups > 1");
  const int64_t tpad = (T + 127) / 128 * 128;
  dim3 grid((unsigned)(tpad / 64), (unsigned)col_groups);
  cudaStream_t st = (cudaStream_t)stream;
  const int tpg = nt / col_groups;
  bf16* direct = col_groups == 1 ? (bf16*)xsd : nullptr;
#define FWD_ARGS                                                                                         \
  (const bf16*)gu, (const bf16*)xs, (const bf16*)bg, (const bf16*)bu, (const bf16*)ad, (uint8_t*)qh,    \
      (uint8_t*)sh, (float*)xsd_part, direct, (int)T, (int)N, s_g, s_u, tpg, qh != nullptr
  if (r == 16)
    k_mlp_fwd<16, 128><<<grid, 128, 0, st>>>(FWD_ARGS);
  else
    k_mlp_fwd<32, 128><<<grid, 128, 0, st>>>(FWD_ARGS);
  mx_note_launch();
#undef FWD_ARGS
  if (int e = mx_launch_status("mlp fwd epilogue")) return e;
  if (col_groups > 1) {
    const int64_t n = T * r;
    k_sum_parts<<<grid_for(n, 256), 256, 0, st>>>((const float*)xsd_part, col_groups, n, n, 1.0f, 1.0f, nullptr,
                                                  (bf16*)xsd, 0, 0);
    mx_note_launch();
    if (int e = mx_launch_status("mlp fwd xsd sum")) return e;
  }
  return MXM_OK;
}

// Backward partition (reference _bwd_grid, scripts/fused_mlp.py:218-232): the fewest partial bytes
// with at least `min_ctas` CTAs per SM.
extern "C" int mxm_mlp_bwd_partitions(int64_t T, int64_t N, int r, int* super_block, int* col_groups) {
  MX_CHECK_ARG(T >= 1 && N >= 128 && N % 128 == 0 && (r == 16 || r == 32) && super_block && col_groups,
               "mxm_mlp_bwd_partitions: bad args");
  const int BN = 32;
  const int64_t tpad = (T + 127) / 128 * 128;
  const int nt = (int)(N / BN);
  const int64_t want = 4 * (int64_t)mxm_num_sms();
  int64_t best = -1;
  int bsb = 128, bcg = nt;
  for (int ncg = 1; ncg <= nt; ++ncg) {
    if (nt % ncg) continue;
    for (int64_t sb = 128; sb <= tpad; sb += 128) {
      const int64_t nsb = (tpad + sb - 1) / sb;
      if (nsb * ncg < want && !(sb == 128 && ncg == nt)) continue;
      const int64_t cost = nsb * N * r * 3 * 4 + (int64_t)ncg * T * 3 * r * 4;
      if (best < 0 || cost < best) {
        best = cost;
        bsb = (int)sb;
        bcg = ncg;
      }
    }
  }
  *super_block = bsb;
  *col_groups = bcg;
  return MXM_OK;
}

extern "C" int mxm_mlp_bwd_epilogue(const void* gu, const void* xs, const void* dhm, const void* dxd, const void* bg,
                                    const void* bu, const void* ad, int64_t T, int64_t N, int r, float s_g, float s_u,
                                    void* q, void* s, void* dxa_part, void* dbg_part, void* dbu_part,
                                    void* dad_part, int super_block, int col_groups, void* stream) {
  MX_CHECK_ARG(gu && xs && dhm && dxd && bg && bu && ad && dxa_part && dbg_part && dbu_part && dad_part,
               "mxm_mlp_bwd_epilogue: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32),
               "mxm_mlp_bwd_epilogue: need T >= 1, N %% 128 == 0, r in {16, 32}");
  MX_CHECK_ARG((q == nullptr) == (s == nullptr), "mxm_mlp_bwd_epilogue: q and s go together");
  const int BN = 32;
  const int nt = (int)(N / BN);
  MX_CHECK_ARG(col_groups >= 1 && nt % col_groups == 0 && super_block >= 64 && super_block % 64 == 0,
               "mxm_mlp_bwd_epilogue: bad partition (%d, %d)", super_block, col_groups);
  const int64_t tpad = (T + 127) / 128 * 128;
  const int nsb = (int)((tpad + super_block - 1) / super_block);
  dim3 grid((unsigned)nsb, (unsigned)col_groups);
  const size_t smem = 4 * 3 * (size_t)r * BN * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
  const int tpg = nt / col_groups;
#define BWD_ARGS                                                                                          \
  (const bf16*)gu, (const bf16*)xs, (const bf16*)dhm, (const bf16*)dxd, (const bf16*)bg, (const bf16*)bu, \
      (const bf16*)ad, (uint8_t*)q, (uint8_t*)s, (float*)dxa_part, (float*)dbg_part, (float*)dbu_part,    \
      (float*)dad_part, (int)T, (int)tpad, (int)N, s_g, s_u, super_block, tpg, q != nullptr
  if (r == 16) {
    cudaFuncSetAttribute(k_mlp_bwd<16, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_mlp_bwd<16, 32><<<grid, 128, smem, st>>>(BWD_ARGS);
    mx_note_launch();
  } else {
    cudaFuncSetAttribute(k_mlp_bwd<32, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_mlp_bwd<32, 32><<<grid, 128, smem, st>>>(BWD_ARGS);
    mx_note_launch();
  }
#undef BWD_ARGS
  return mx_launch_status("mlp bwd epilogue");
}

extern "C" int mxm_mlp_bwd_reduce(const void* dxa_part, const void* dbg_part, const void* dbu_part,
                                  const void* dad_part, int64_t T, int64_t N, int r, float s_g, float s_u,
                                  int super_block, int col_groups, void* dxa, void* xsd, void* dBg, void* dBu,
                                  void* dAd, void* stream) {
  MX_CHECK_ARG(dxa_part && dbg_part && dbu_part && dad_part && dxa && xsd && dBg && dBu && dAd,
               "mxm_mlp_bwd_reduce: null pointer");
  const int64_t tpad = (T + 127) / 128 * 128;
  const int nsb = (int)((tpad + super_block - 1) / super_block);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nd = T * 3 * r;
  k_reduce_dxa<<<grid_for(nd, 256), 256, 0, st>>>((const float*)dxa_part, col_groups, (int)T, r, s_g, s_u, (bf16*)dxa,
                                                  (bf16*)xsd);
  mx_note_launch();
  const int64_t nb = N * r;
  k_sum_parts<<<grid_for(nb, 256), 256, 0, st>>>((const float*)dbg_part, nsb, nb, nb, s_g, 1.f, (float*)dBg, nullptr,
                                                 0, 0);
  mx_note_launch();
  k_sum_parts<<<grid_for(nb, 256), 256, 0, st>>>((const float*)dbu_part, nsb, nb, nb, s_u, 1.f, (float*)dBu, nullptr,
                                                 0, 0);
  mx_note_launch();
  k_sum_parts<<<grid_for(nb, 256), 256, 0, st>>>((const float*)dad_part, nsb, nb, nb, 1.f, 1.f, (float*)dAd, nullptr,
                                                 0, 0);
  mx_note_launch();
  return mx_launch_status("mlp bwd reduce");
}

extern "C" int mxm_rowdot(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post,
                          void* out, int64_t ldo, void* stream) {
  MX_CHECK_ARG(A && B && out, "mxm_rowdot: null pointer");
  MX_CHECK_ARG(T >= 1 && K >= 32 && K % 32 == 0 && (n == 16 || n == 32 || n == 64) && lda % 8 == 0 && ldo % 2 == 0,
               "mxm_rowdot: need K %% 32 == 0, n in {16, 32, 64}, lda %% 8 == 0");
  MX_CHECK_ARG(mx_aligned(A, 16) && mx_aligned(B, 16) && mx_aligned(out, 4), "mxm_rowdot: alignment");
  const unsigned grid = (unsigned)((T + 63) / 64);
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 16)
    k_rowdot<16><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)B, (int)T, (int)K, post, (bf16*)out, ldo);
  else if (n == 32)
    k_rowdot<32><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)B, (int)T, (int)K, post, (bf16*)out, ldo);
  else
    k_rowdot<64><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)B, (int)T, (int)K, post, (bf16*)out, ldo);
  mx_note_launch();
  return mx_launch_status("rowdot");
}

extern "C" int mxm_coldot_chunks(int64_t T, int64_t K, int* rows_per_chunk, int* chunks) {
  MX_CHECK_ARG(T >= 1 && K >= 64 && rows_per_chunk && chunks, "mxm_coldot_chunks: bad args");
  const int64_t ctas_k = (K + 63) / 64;
  const int64_t want = 4 * (int64_t)mxm_num_sms();
  int64_t nch = (want + ctas_k - 1) / ctas_k;
  int64_t rpc = (T + nch - 1) / nch;
  rpc = (rpc + 15) / 16 * 16;
  if (rpc < 256) rpc = 256;
  *rows_per_chunk = (int)rpc;
  *chunks = (int)((T + rpc - 1) / rpc);
  return MXM_OK;
}

// out = bf16( bf16(sum_t A[t,k] E[t,j]) * post ), written [K, n] or transposed [n, K].
extern "C" int mxm_coldot(const void* A, int64_t lda, const void* E, int64_t lde, int64_t T, int64_t K, int n,
                          float post, int transpose_out, void* part, int rows_per_chunk, int chunks, void* out,
                          void* stream) {
  MX_CHECK_ARG(A && E && part && out, "mxm_coldot: null pointer");
  MX_CHECK_ARG(T >= 1 && K % 64 == 0 && (n == 16 || n == 32 || n == 64) && rows_per_chunk % 16 == 0 &&
                   (int64_t)rows_per_chunk * chunks >= T,
               "mxm_coldot: bad shape or chunking");
  dim3 grid((unsigned)(K / 64), (unsigned)chunks);
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 16)
    k_coldot<16><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)E, lde, (int)T, (int)K, rows_per_chunk,
                                       (float*)part);
  else if (n == 32)
    k_coldot<32><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)E, lde, (int)T, (int)K, rows_per_chunk,
                                       (float*)part);
  else
    k_coldot<64><<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)E, lde, (int)T, (int)K, rows_per_chunk,
                                       (float*)part);
  mx_note_launch();
  if (int e = mx_launch_status("coldot")) return e;
  const int64_t nn = K * n;
  k_sum_parts<<<grid_for(nn, 256), 256, 0, st>>>((const float*)part, chunks, nn, nn, 1.f, post, nullptr, (bf16*)out,
                                                 transpose_out ? K : 0, transpose_out ? n : 0);
  mx_note_launch();
  return mx_launch_status("coldot sum");
}
