// The memory-bound passes of the fused SwiGLU-LoRA MLP (reference scripts/fused_mlp.py) on sm_100a.
//
//   k_mlp_fwd   -- the forward epilogue (reference _fwd_kernel, scripts/fused_mlp.py:81-109):
//                  reads gu = [x W_gate^T | x W_up^T] once, adds the LoRA-B terms, SwiGLU, writes h as
//                  MXFP8 (codes + blocked scales) for the down GEMM and xS_down = h A_down^T.
//   k_mlp_bwd_tc / k_mlp_bwd<32>
//               -- the backward epilogue (reference _bwd_kernel, scripts/fused_mlp.py:112-175):
//                  recomputes g, u, h from gu, dh = dh_mx + dxd A_down, SwiGLU backward, writes
//                  [dg | du] as MXFP8 for the dx GEMM, and the LoRA gradient pieces dB_gate, dB_up,
//                  dA_down (summed over rows) and dxa_gate, dxa_up, xS_down (summed over columns).
//                  Rank 16 (k_mlp_bwd_tc) runs every rank-r product as tcgen05 MMAs into TMEM; rank 32
//                  keeps the warp-level form.
//   k_rowdot    -- out[T, n] = A[T, K] B[n, K]^T for the rank-n LoRA-A products (x S^T, dy B_down).
//   k_coldot    -- out[K, n] = A[T, K]^T E[T, n] for the LoRA weight gradients (dA, dB_down).
//   k_sum_*     -- fixed-order sums of the per-CTA partial buffers (deterministic, no atomics).
//
// The rank-r products run on the tensor cores (warp-level m16n8k16 bf16 MMAs, or tcgen05 MMAs in the
// rank-16 backward); the element-wise math keeps the reference's rounding points (bf16 after each fp32
// expression it rounds).
#include <algorithm>
#include <mutex>

#include "mx_epi.cuh"
#include "mx_mma.cuh"
#include "mx_runtime.h"

namespace {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------------------------------------ forward
// CTA = one 240-row block x one column group of `tpg` 64-column tiles.  Warp 15 streams, per tile,
// the g and u tiles ([240 x 64] bf16, 128-byte swizzle) and the tile's slices of B_gate, B_up
// ([64 x r]) and A_down ([r x 64], 128-byte swizzle) into a 3-stage ring with TMA.  Warps 0-14 each
// own 16 rows (four warps per scheduler to hide latency); every MMA operand comes from shared memory
// through ldmatrix, and the per-row xS_down accumulator stays in registers across the whole group.
constexpr int FWD_CONS = 15, FWD_ROWS = 16 * FWD_CONS;             // consumer warps, rows per CTA
constexpr int FWD_THREADS = 32 * (FWD_CONS + 1);                       // + one TMA producer warp
constexpr int FWD_BN = 64, FWD_ST = 3, FWD_TILE = FWD_ROWS * FWD_BN * 2;  // 30 KB per g / u tile
__host__ __device__ constexpr int fwd_btile(int R) { return FWD_BN * R * 2; }
__host__ __device__ constexpr int fwd_stage(int R) { return 2 * FWD_TILE + 3 * fwd_btile(R); }
__host__ __device__ constexpr size_t fwd_smem(int R) { return 1024 + (size_t)FWD_ST * fwd_stage(R) + 2 * FWD_ST * 8; }

template <int R>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    k_mlp_fwd(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_bg,
              const __grid_constant__ CUtensorMap tm_bu, const __grid_constant__ CUtensorMap tm_ad,
              const bf16* __restrict__ xs, uint8_t* __restrict__ qh, uint8_t* __restrict__ sh,
              float* __restrict__ xsd_part, bf16* __restrict__ xsd_out, int T, int Tpad, int N, float s_g,
              float s_u, int tpg, int write_q, int* err) {
  constexpr int KS = R / 16, BT = fwd_btile(R), STG = fwd_stage(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + FWD_ST * STG);
  uint64_t* empty = full + FWD_ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * FWD_ROWS;
  if (threadIdx.x == 0) {
    for (int i = 0; i < FWD_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], FWD_CONS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == FWD_CONS) {  // TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_gu);
      prefetch_tmap(&tm_bg);
      prefetch_tmap(&tm_bu);
      prefetch_tmap(&tm_ad);
    }
    int stage = 0;
    uint32_t phase = 0;
    for (int ct = 0; ct < tpg; ++ct) {
      const int n0 = (blockIdx.y * tpg + ct) * FWD_BN;
      if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) break;
      if (lane == 0) {
        uint8_t* dst = smem + stage * STG;
        uint64_t* fb = &full[stage];
        mbar_arrive_expect_tx(fb, STG);
        tma_load_2d(dst, &tm_gu, fb, n0, (int)row0);
        tma_load_2d(dst + FWD_TILE, &tm_gu, fb, N + n0, (int)row0);
        tma_load_2d(dst + 2 * FWD_TILE, &tm_bg, fb, 0, n0);
        tma_load_2d(dst + 2 * FWD_TILE + BT, &tm_bu, fb, 0, n0);
        tma_load_2d(dst + 2 * FWD_TILE + 2 * BT, &tm_ad, fb, n0, 0);
      }
      __syncwarp();
      if (++stage == FWD_ST) {
        stage = 0;
        phase ^= 1;
      }
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int rl = warp * 16 + g;  // row within the block
  const int64_t ra = row0 + rl, rb = ra + 8;
  const bool va = ra < T, vb = rb < T;
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

  // ldmatrix lane roles: matrix mi = lane / 8, row-in-matrix lr = lane % 8.  Per-lane shared-memory
  // offsets are fixed for the whole kernel (the swizzles make them non-affine), so they are hoisted.
  const int mi = lane >> 3, lr = lane & 7;
  const int lrow = warp * 16 + (mi & 1) * 8 + lr;
  uint32_t o_gu[FWD_BN / 16], o_b[FWD_BN / 16][KS], o_ad[FWD_BN / 16][R / 16];
#pragma unroll
  for (int p = 0; p < FWD_BN / 16; ++p) {
    // g / u tiles (128-byte rows, 128-byte swizzle): matrices (rows +0 / +8) x (n-tile 2p / 2p+1)
    o_gu[p] = swz<128>((uint32_t)lrow, (uint32_t)(2 * p + (mi >> 1)));
    // B_gate / B_up slices [64 n x r]: matrices (n-tile 2p / 2p+1) x (j 16kk / +8)
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
      o_b[p][kk] = swz<2 * R>((uint32_t)(8 * (2 * p + (mi >> 1)) + lr), (uint32_t)(2 * kk + (mi & 1)));
    // A_down slice [r x 64] (128-byte rows): matrices (j 16jp / +8) x (k-slice p: cols 16p / +8)
#pragma unroll
    for (int jp = 0; jp < R / 16; ++jp)
      o_ad[p][jp] = swz<128>((uint32_t)(16 * jp + 8 * (mi >> 1) + lr), (uint32_t)(2 * p + (mi & 1)));
  }
  const uint32_t s_ring = smem_u32(smem);
  const float2 sg2 = make_float2(s_g, s_g), su2 = make_float2(s_u, s_u);
  const QRows qr = qrows_init(ra, T, Tpad, qh, N, sh, N, t);
  int stage = 0;
  uint32_t phase = 0;
  for (int ct = 0; ct < tpg; ++ct) {
    const int n0 = (blockIdx.y * tpg + ct) * FWD_BN;
    if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
    const uint32_t sb = s_ring + (uint32_t)stage * STG;
    const uint32_t tg = sb, tu = sb + FWD_TILE, tbg = sb + 2 * FWD_TILE, tbu = tbg + BT, tad = tbu + BT;
#pragma unroll
    for (int b = 0; b < FWD_BN / 32; ++b) {
      uint32_t hp[4][2];
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const int p = 2 * b + pp;  // pair of n8 tiles (2p, 2p+1)
        uint32_t G[4], U[4];
        ldsm4(G, tg + o_gu[p]);
        ldsm4(U, tu + o_gu[p]);
        float dg0[4] = {0.f, 0.f, 0.f, 0.f}, dg1[4] = {0.f, 0.f, 0.f, 0.f};
        float du0[4] = {0.f, 0.f, 0.f, 0.f}, du1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          uint32_t BG[4], BU[4];
          ldsm4(BG, tbg + o_b[p][kk]);
          ldsm4(BU, tbu + o_b[p][kk]);
          mma16816(dg0, axg[kk], BG[0], BG[1]);
          mma16816(dg1, axg[kk], BG[2], BG[3]);
          mma16816(du0, axu[kk], BU[0], BU[1]);
          mma16816(du1, axu[kk], BU[2], BU[3]);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float* dg = q ? dg1 : dg0;
          const float* du = q ? du1 : du0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {   // h = 0: row g, h = 1: row g + 8
            const float2 gg = up2(rn2(__ffma2_rn(sg2, make_float2(dg[2 * h], dg[2 * h + 1]), up2(G[2 * q + h]))));
            const float2 uu = up2(rn2(__ffma2_rn(su2, make_float2(du[2 * h], du[2 * h + 1]), up2(U[2 * q + h]))));
            hp[2 * pp + q][h] = rn2(__fmul2_rn(__fmul2_rn(gg, sigmoid2(gg)), uu));   // h = bf16(silu(g) * u)
          }
        }
      }
      if (write_q) quant_block16p(hp, qr, n0 + 32 * b, t);
      // xS_down += h (16 x 32 block) A_down^T: two k-slices of 16 columns
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        const uint32_t a[4] = {hp[2 * mm][0], hp[2 * mm][1], hp[2 * mm + 1][0], hp[2 * mm + 1][1]};
#pragma unroll
        for (int jp = 0; jp < R / 16; ++jp) {
          uint32_t AD[4];
          ldsm4(AD, tad + o_ad[2 * b + mm][jp]);
          mma16816(accx[2 * jp], a, AD[0], AD[1]);
          mma16816(accx[2 * jp + 1], a, AD[2], AD[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == FWD_ST) {
      stage = 0;
      phase ^= 1;
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
// Persistent CTAs, one per SM, each walking a contiguous run of `per` work items (row block of
// SB = 16 x CONS rows, 32-column tile), column tile fastest.  Warp CONS streams, per item, the [SB x 32]
// bf16 tiles of g, u and dh (64-byte swizzle) plus the tile's slices of B_gate, B_up ([32 x r]) and
// A_down ([r x 32]) into a 3-stage ring with TMA, and, when the run enters a row block, the block's xs
// and dxd rows.  Consumer warps 0 .. CONS-1 each own 16 rows of the current block:
//   * dg, du, h of the tile are computed in registers, quantized, and multiplied by the B slices into
//     the per-row sums dxa_gate, dxa_up, xS_down, which stay in registers while the run stays in the
//     row block and are then stored into this CTA's slot of the fp32 partials;
//   * dg, du, h are also stored (bf16, the same swizzle) into a shared operand tile (op_full when every
//     consumer warp has stored its rows).
// Warp CONS also reduces the operand tile over the block's SB rows into the column products dB_gate^T,
// dB_up^T and dA_down (mma, xa^T from the row buffer) while the consumers go on to the next tile, and
// then releases it (op_empty): the consumers never wait on those reductions unless they run a whole
// tile ahead.  Four warps per scheduler (r = 16) hide the latency of the per-element chains.  No
// atomics: the result is deterministic.
constexpr int BWD_BN = 32, BWD_ST = 3;
// consumer warps: 16 warps in all (4 per scheduler, 128 registers) for r = 16; 12 (3 per scheduler,
// 168 registers) for r = 32, whose per-row sums and fragments need more registers.  (14 consumers
// measured slower: the fourth warp per scheduler matters more than the block height.)
__host__ __device__ constexpr int bwd_cons(int R) { return R == 16 ? 15 : 11; }
__host__ __device__ constexpr int bwd_rows(int R) { return 16 * bwd_cons(R); }   // rows per CTA
__host__ __device__ constexpr int bwd_tile(int R) { return bwd_rows(R) * BWD_BN * 2; }
__host__ __device__ constexpr int bwd_btile(int R) { return BWD_BN * R * 2; }
__host__ __device__ constexpr int bwd_stage(int R) { return 3 * bwd_tile(R) + 3 * bwd_btile(R); }
__host__ __device__ constexpr size_t bwd_rowbuf(int R) { return ((size_t)bwd_rows(R) * 3 * R * 2 + 1023) / 1024 * 1024; }
__host__ __device__ constexpr size_t bwd_smem(int R) {
  return 1024 + (size_t)BWD_ST * bwd_stage(R) + bwd_rowbuf(R) + 3 * (size_t)bwd_tile(R) +
         (2 * BWD_ST + 4) * sizeof(uint64_t);
}

template <int R>
__global__ void __launch_bounds__(32 * (bwd_cons(R) + 1), 1)
    k_mlp_bwd(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dh,
              const __grid_constant__ CUtensorMap tm_bg, const __grid_constant__ CUtensorMap tm_bu,
              const __grid_constant__ CUtensorMap tm_ad, const __grid_constant__ CUtensorMap tm_xs,
              const __grid_constant__ CUtensorMap tm_dxd, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
              float* __restrict__ dxa_part, float* __restrict__ dbg_part, float* __restrict__ dbu_part,
              float* __restrict__ dad_part, int T, int Tpad, int N, float s_g, float s_u, int per, int write_q,
              int* err) {
  constexpr int CONS = bwd_cons(R), SB = bwd_rows(R), KS = R / 16, NT = BWD_BN / 8, R3 = 3 * R;
  constexpr int TILE = bwd_tile(R), BT = bwd_btile(R), STG = bwd_stage(R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* rows_xs = smem + BWD_ST * STG;             // [SB][2r] bf16, TMA-swizzled
  uint8_t* rows_dxd = rows_xs + (size_t)SB * 4 * R;    // [SB][r]
  uint8_t* opbuf = rows_xs + bwd_rowbuf(R);            // [3][SB][32] bf16: dg | du | h, 64-byte swizzle
  uint64_t* full = reinterpret_cast<uint64_t*>(opbuf + 3 * TILE);
  uint64_t* empty = full + BWD_ST;
  uint64_t* rows_full = empty + BWD_ST;
  uint64_t* op_full = rows_full + 1;   // all consumer warps stored the tile's dg | du | h
  uint64_t* op_empty = op_full + 1;    // all column-product blocks of the tile were read
  uint64_t* rows_empty = op_empty + 1; // every consumer warp has the block's rows in registers (the producer
                                       // reloads rows_xs / rows_dxd once its own column products are done too)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = N / BWD_BN;                                   // column tiles per row block
  const int items = ((Tpad + SB - 1) / SB) * nt;               // (row block, column tile), column fastest
  const int it_lo = blockIdx.x * per, it_hi = min(it_lo + per, items);
  const int64_t N2 = 2 * (int64_t)N;
  if (threadIdx.x == 0) {
    for (int i = 0; i < BWD_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONS);
    }
    mbar_init(rows_full, 1);
    mbar_init(rows_empty, CONS);
    mbar_init(op_full, CONS);
    mbar_init(op_empty, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CONS) {  // TMA producer and column products
    if (lane == 0) {
      prefetch_tmap(&tm_gu);
      prefetch_tmap(&tm_dh);
      prefetch_tmap(&tm_bg);
      prefetch_tmap(&tm_bu);
      prefetch_tmap(&tm_ad);
    }
    const int g = lane >> 2, t = lane & 3, mi = lane >> 3, lr = lane & 7;
    const uint32_t s_xs = smem_u32(rows_xs), s_dxd = smem_u32(rows_dxd), ob = smem_u32(opbuf);
    // Column products of one stored tile: dB_gate^T = xa_gate^T dg, dB_up^T = xa_up^T du and
    // dA_down = dxd^T h, each reduced over the block's SB rows with mma (A = xa^T from the row buffer,
    // B = the operand tile, both through ldmatrix.trans; the offsets advance by 16 rows per k-step, the
    // swizzles only use row bits 0-2) and stored as the block's partial.  Three (product, 16-row block
    // of r) pairs per pass, both 16-column halves of the tile: 12 independent accumulator chains.
    auto column_products = [&](int sbi, int n0) {
      constexpr int PM = 3 * KS, BATCH = 3;
#pragma unroll
      for (int pm0 = 0; pm0 < PM; pm0 += BATCH) {
        float acc[BATCH][2][2][4] = {};
        uint32_t pa[BATCH], pb[BATCH][2];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const int prod = (pm0 + b) / KS, mt = (pm0 + b) % KS;
          const uint32_t arow = (uint32_t)((mi >> 1) * 8 + lr);
          pa[b] = prod < 2 ? s_xs + swz<4 * R>(arow, (uint32_t)(prod * 2 * KS + 2 * mt + (mi & 1)))
                           : s_dxd + swz<2 * R>(arow, (uint32_t)(2 * mt + (mi & 1)));
#pragma unroll
          for (int nh = 0; nh < 2; ++nh)
            pb[b][nh] = ob + (uint32_t)prod * TILE + swz<64>((uint32_t)((mi & 1) * 8 + lr), (uint32_t)(2 * nh + (mi >> 1)));
        }
#pragma unroll 5
        for (int kk = 0; kk < CONS; ++kk) {
#pragma unroll
          for (int b = 0; b < BATCH; ++b) {
            const int prod = (pm0 + b) / KS;
            uint32_t A[4];
            ldsm4t(A, pa[b]);
            pa[b] += prod < 2 ? 16u * 4u * R : 16u * 2u * R;
#pragma unroll
            for (int nh = 0; nh < 2; ++nh) {
              uint32_t B[4];
              ldsm4t(B, pb[b][nh]);
              pb[b][nh] += 16u * 64u;
              mma16816(acc[b][nh][0], A, B[0], B[1]);
              mma16816(acc[b][nh][1], A, B[2], B[3]);
            }
          }
        }
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const int prod = (pm0 + b) / KS, mt = (pm0 + b) % KS, j = 16 * mt + g;
#pragma unroll
          for (int nh = 0; nh < 2; ++nh)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int n = n0 + 16 * nh + 8 * h + 2 * t;
              const float* a = acc[b][nh][h];
              if (prod < 2) {   // [n_blocks, N, r]: element (n, j)
                float* P = (prod == 0 ? dbg_part : dbu_part) + ((int64_t)sbi * N + n) * R + j;
                P[0] = a[0];
                P[R] = a[1];
                P[8] = a[2];
                P[R + 8] = a[3];
              } else {          // [n_blocks, r, N]: element (j, n)
                float* P = dad_part + ((int64_t)sbi * R + j) * N + n;
                *reinterpret_cast<float2*>(P) = make_float2(a[0], a[1]);
                *reinterpret_cast<float2*>(P + 8 * (int64_t)N) = make_float2(a[2], a[3]);
              }
            }
        }
      }
    };
    // Three queues, polled in turn (lane 0 tests, the warp follows): the next row block's xs / dxd rows
    // (once the consumers have their fragments of the current block and this warp's column products of
    // the block are done), the next tile's loads (once its ring stage is free), and the column products
    // of the oldest stored tile (once every consumer warp stored it: op_full).
    const int cnt = it_hi - it_lo;
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0, tasked = 0, row_loads = 0, rows_at = 0;   // rows_at: first item of the next row block
    uint64_t t0 = mx_globaltimer();
    while (tasked < cnt) {
      bool prog = false;
      if (rows_at < cnt && tasked == rows_at) {
        const bool rdy = row_loads == 0 ||
                         __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(rows_empty, (uint32_t)((row_loads - 1) & 1)) : 0, 0);
        if (rdy) {
          const int sbr = (it_lo + rows_at) / nt;
          if (lane == 0) {
            mbar_arrive_expect_tx(rows_full, (uint32_t)(SB * 3 * R * 2));
            tma_load_2d(rows_xs, &tm_xs, rows_full, 0, sbr * SB);
            tma_load_2d(rows_dxd, &tm_dxd, rows_full, 0, sbr * SB);
          }
          __syncwarp();
          ++row_loads;
          rows_at = (sbr + 1) * nt - it_lo;
          prog = true;
        }
      }
      if (issued < cnt && __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(&empty[stage], phase ^ 1) : 0, 0)) {
        const int it = it_lo + issued;
        const int n0 = (it % nt) * BWD_BN, r0 = (it / nt) * SB;
        if (lane == 0) {
          uint8_t* dst = smem + stage * STG;
          uint64_t* fb = &full[stage];
          mbar_arrive_expect_tx(fb, STG);
          tma_load_2d(dst, &tm_gu, fb, n0, r0);
          tma_load_2d(dst + TILE, &tm_gu, fb, N + n0, r0);
          tma_load_2d(dst + 2 * TILE, &tm_dh, fb, n0, r0);
          tma_load_2d(dst + 3 * TILE, &tm_bg, fb, 0, n0);
          tma_load_2d(dst + 3 * TILE + BT, &tm_bu, fb, 0, n0);
          tma_load_2d(dst + 3 * TILE + 2 * BT, &tm_ad, fb, n0, 0);
        }
        __syncwarp();
        ++issued;
        if (++stage == BWD_ST) {
          stage = 0;
          phase ^= 1;
        }
        prog = true;
      }
      if (tasked < issued &&
          __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(op_full, (uint32_t)(tasked & 1)) : 0, 0)) {
        mbar_wait(op_full, (uint32_t)(tasked & 1), err, MX_DEV_TIMEOUT_PRODUCER);   // complete: acquire, every lane
        const int it = it_lo + tasked;
        column_products(it / nt, (it % nt) * BWD_BN);
        __syncwarp();
        if (lane == 0) mbar_arrive(op_empty);
        ++tasked;
        prog = true;
      }
      if (prog) {
        t0 = mx_globaltimer();
      } else {
        if (mx_globaltimer() - t0 > MX_WAIT_LIMIT_NS) {
          if (lane == 0) mx_set_error(err, MX_DEV_TIMEOUT_PRODUCER);
          break;
        }
        __nanosleep(64);
      }
    }
    // leave no copy in flight: wait (bounded) for the last load of every stage that was used
    for (int k = 0; k < BWD_ST && k < issued; ++k) {
      const int i = issued - 1 - k, st = i % BWD_ST;
      mbar_wait(&full[st], (uint32_t)((i / BWD_ST) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
    }
    if (row_loads > 0) mbar_wait(rows_full, (uint32_t)((row_loads - 1) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, lr = lane & 7;

  // Per-lane shared-memory offsets, fixed for the whole kernel (the swizzles make them non-affine).
  // g / u / dh tiles and the dg / du / h operand tile (64-byte rows, 64-byte swizzle): matrices
  // (rows +0 / +8) x (n-tile 2p / 2p+1)
  const int lrow = warp * 16 + (mi & 1) * 8 + lr;
  uint32_t o_tile[NT / 2];
#pragma unroll
  for (int p = 0; p < NT / 2; ++p) o_tile[p] = swz<64>((uint32_t)lrow, (uint32_t)(2 * p + (mi >> 1)));
  // B_gate / B_up slices [32 n x r]: non-transposed for the LoRA-B terms, transposed for the row sums
  uint32_t o_b[NT / 2][KS], o_bt[NT / 2][R / 16], o_a[NT / 2][KS], o_at[NT / 2][R / 16];
#pragma unroll
  for (int p = 0; p < NT / 2; ++p) {
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      o_b[p][kk] = swz<2 * R>((uint32_t)(8 * (2 * p + (mi >> 1)) + lr), (uint32_t)(2 * kk + (mi & 1)));
      o_a[p][kk] = swz<64>((uint32_t)(16 * kk + 8 * (mi & 1) + lr), (uint32_t)(2 * p + (mi >> 1)));
    }
#pragma unroll
    for (int jp = 0; jp < R / 16; ++jp) {
      o_bt[p][jp] = swz<2 * R>((uint32_t)(16 * p + 8 * (mi & 1) + lr), (uint32_t)(2 * jp + (mi >> 1)));
      o_at[p][jp] = swz<64>((uint32_t)(16 * jp + 8 * (mi >> 1) + lr), (uint32_t)(2 * p + (mi & 1)));
    }
  }
  const uint32_t s_xs = smem_u32(rows_xs), s_dxd = smem_u32(rows_dxd), s_ring = smem_u32(smem);
  const uint32_t ob = smem_u32(opbuf);
  uint32_t axg[KS][4], axu[KS][4], axd[KS][4];     // this warp's rows of xa_gate | xa_up | dxd (A fragments)
  float rg[R / 8][4], ru[R / 8][4], rx[R / 8][4];  // per-row sums over this CTA's columns of the row block
  QRows qr{};
  uint32_t rows_ph = 0;
  // this CTA's partial of the row block's per-row products [dg Bg | du Bu | h Ad^T]: one slot per CTA
  // that works on the block, in CTA order
  auto flush_rows = [&](int sbi) {
    const int slot = (int)blockIdx.x - (sbi * nt) / per;
    float* P = dxa_part + (int64_t)slot * T * R3;
    const int64_t ra = (int64_t)sbi * SB + warp * 16 + g;
#pragma unroll
    for (int jt = 0; jt < R / 8; ++jt) {
      const int c = 8 * jt + 2 * t;
      if (ra < T) {
        *reinterpret_cast<float2*>(P + ra * R3 + c) = make_float2(rg[jt][0], rg[jt][1]);
        *reinterpret_cast<float2*>(P + ra * R3 + R + c) = make_float2(ru[jt][0], ru[jt][1]);
        *reinterpret_cast<float2*>(P + ra * R3 + 2 * R + c) = make_float2(rx[jt][0], rx[jt][1]);
      }
      if (ra + 8 < T) {
        *reinterpret_cast<float2*>(P + (ra + 8) * R3 + c) = make_float2(rg[jt][2], rg[jt][3]);
        *reinterpret_cast<float2*>(P + (ra + 8) * R3 + R + c) = make_float2(ru[jt][2], ru[jt][3]);
        *reinterpret_cast<float2*>(P + (ra + 8) * R3 + 2 * R + c) = make_float2(rx[jt][2], rx[jt][3]);
      }
    }
  };

  const float2 sg2 = make_float2(s_g, s_g), su2 = make_float2(s_u, s_u);
  int stage = 0;
  uint32_t phase = 0;
  int sbi = it_lo / nt, n0 = (it_lo % nt) * BWD_BN;
  const int cnt = it_hi - it_lo;
  for (int ct = 0; ct < cnt; ++ct) {   // ct: this CTA's tile count, for the hand-off parities
    if (ct == 0 || n0 == 0) {          // entering a row block
      if (!mbar_wait(rows_full, rows_ph, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
      rows_ph ^= 1;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        ldsm4(axg[kk], s_xs + swz<4 * R>((uint32_t)lrow, (uint32_t)(2 * kk + (mi >> 1))));
        ldsm4(axu[kk], s_xs + swz<4 * R>((uint32_t)lrow, (uint32_t)(2 * KS + 2 * kk + (mi >> 1))));
        ldsm4(axd[kk], s_dxd + swz<2 * R>((uint32_t)lrow, (uint32_t)(2 * kk + (mi >> 1))));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(rows_empty);   // the block's rows are in registers now
#pragma unroll
      for (int j = 0; j < R / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) rg[j][e] = ru[j][e] = rx[j][e] = 0.f;
      qr = qrows_init((int64_t)sbi * SB + warp * 16 + g, T, Tpad, q, N2, s, N2, t);
    }
    if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
    {
      const uint32_t sb = s_ring + (uint32_t)stage * STG;
      const uint32_t tg = sb, tu = sb + TILE, th = sb + 2 * TILE;
      const uint32_t tbg = sb + 3 * TILE, tbu = tbg + BT, tad = tbu + BT;

      uint32_t dgp[NT][2], dup[NT][2], hp[NT][2];
#pragma unroll
      for (int p = 0; p < NT / 2; ++p) {
        uint32_t G[4], U[4], D[4];
        ldsm4(G, tg + o_tile[p]);
        ldsm4(U, tu + o_tile[p]);
        ldsm4(D, th + o_tile[p]);
        float dg[2][4] = {}, du[2][4] = {}, dd[2][4] = {};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          uint32_t BG[4], BU[4], AD[4];
          ldsm4(BG, tbg + o_b[p][kk]);
          ldsm4(BU, tbu + o_b[p][kk]);
          ldsm4t(AD, tad + o_a[p][kk]);   // A_down slice [r x 32 n] transposed: B[k = j][col n]
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            mma16816(dg[qq], axg[kk], BG[2 * qq], BG[2 * qq + 1]);
            mma16816(du[qq], axu[kk], BU[2 * qq], BU[2 * qq + 1]);
            mma16816(dd[qq], axd[kk], AD[2 * qq], AD[2 * qq + 1]);
          }
        }
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int i = 2 * p + qq;
#pragma unroll
          for (int h = 0; h < 2; ++h) {   // h = 0: row g, h = 1: row g + 8
            const float2 gg = up2(rn2(__ffma2_rn(sg2, make_float2(dg[qq][2 * h], dg[qq][2 * h + 1]), up2(G[2 * qq + h]))));
            const float2 uu = up2(rn2(__ffma2_rn(su2, make_float2(du[qq][2 * h], du[qq][2 * h + 1]), up2(U[2 * qq + h]))));
            const float2 sig = sigmoid2(gg);
            const float2 sl = __fmul2_rn(gg, sig);                                 // silu(g)
            hp[i][h] = rn2(__fmul2_rn(sl, uu));                                     // h = bf16(silu * u)
            const float2 dh = up2(rn2(add_bf16x2_f32(D[2 * qq + h], make_float2(dd[qq][2 * h], dd[qq][2 * h + 1]))));
            dup[i][h] = rn2(__fmul2_rn(dh, sl));                                    // du = bf16(dh * silu)
            const float2 om = __ffma2_rn(sig, make_float2(-1.f, -1.f), make_float2(1.f, 1.f));  // 1 - sig
            const float2 f = __ffma2_rn(gg, om, make_float2(1.f, 1.f));             // g (1 - sig) + 1
            dgp[i][h] = rn2(__fmul2_rn(__fmul2_rn(__fmul2_rn(dh, uu), sig), f));    // dg
          }
        }
      }
      if (write_q) {
        quant_block16p(dgp, qr, n0, t);
        quant_block16p(dup, qr, (int64_t)N + n0, t);
      }
      // per-row products (sums over columns): [dg Bg | du Bu | h Ad^T]
#pragma unroll
      for (int mm = 0; mm < NT / 2; ++mm) {
        const uint32_t adg[4] = {dgp[2 * mm][0], dgp[2 * mm][1], dgp[2 * mm + 1][0], dgp[2 * mm + 1][1]};
        const uint32_t adu[4] = {dup[2 * mm][0], dup[2 * mm][1], dup[2 * mm + 1][0], dup[2 * mm + 1][1]};
        const uint32_t ah[4] = {hp[2 * mm][0], hp[2 * mm][1], hp[2 * mm + 1][0], hp[2 * mm + 1][1]};
#pragma unroll
        for (int jp = 0; jp < R / 16; ++jp) {
          uint32_t BG[4], BU[4], AD[4];
          ldsm4t(BG, tbg + o_bt[mm][jp]);   // B[k = n][col j] = B_gate[n][j]
          ldsm4t(BU, tbu + o_bt[mm][jp]);
          ldsm4(AD, tad + o_at[mm][jp]);    // B[k = n][col j] = A_down[j][n]
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            mma16816(rg[2 * jp + h2], adg, BG[2 * h2], BG[2 * h2 + 1]);
            mma16816(ru[2 * jp + h2], adu, BU[2 * h2], BU[2 * h2 + 1]);
            mma16816(rx[2 * jp + h2], ah, AD[2 * h2], AD[2 * h2 + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      // dg | du | h of this warp's rows into the operand tile, once the previous tile's blocks were read
      if (ct > 0 && !mbar_wait(op_empty, (uint32_t)((ct - 1) & 1), err, MX_DEV_TIMEOUT_EPILOGUE)) break;
#pragma unroll
      for (int p = 0; p < NT / 2; ++p) {
        stsm4(ob + o_tile[p], dgp[2 * p][0], dgp[2 * p][1], dgp[2 * p + 1][0], dgp[2 * p + 1][1]);
        stsm4(ob + TILE + o_tile[p], dup[2 * p][0], dup[2 * p][1], dup[2 * p + 1][0], dup[2 * p + 1][1]);
        stsm4(ob + 2 * TILE + o_tile[p], hp[2 * p][0], hp[2 * p][1], hp[2 * p + 1][0], hp[2 * p + 1][1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(op_full);
    }
    if (++stage == BWD_ST) {
      stage = 0;
      phase ^= 1;
    }
    const bool last = ct + 1 == cnt;
    if ((n0 += BWD_BN) == N || last) {   // leaving the row block
      flush_rows(sbi);
      n0 = 0;
      ++sbi;
    }
  }
}

// ------------------------------------------------------------------------------------------------ backward, r = 16
// The backward epilogue with every rank-16 product on the 5th-generation tensor cores (tcgen05.mma
// kind::f16, fp32 accumulators in TMEM) and the element-wise work on rows held by threads.  Work item =
// (row block of 256 rows, 32-column tile), column tile fastest; each CTA walks a contiguous run of `per`
// items.  Warp 17 streams per item the [256 x 32] bf16 tiles of g, u and dh (64-byte rows, 64-byte
// swizzle) and the tile's slices of B_gate, B_up ([32 n x 16], 32-byte swizzle) and A_down ([16 x 32 n],
// 64-byte swizzle) into a 3-stage ring, and per row block its xa_gate, xa_up and dxd rows (three
// [256 x 16] buffers, 32-byte swizzle).  Two warps issue the MMAs (one elected lane each, descriptors
// computed once; a small MMA costs ~50 cycles of issue, so the two streams go out side by side):
//   * warp 18: the LoRA terms xa_gate B_gate^T, xa_up B_up^T and dxd A_down of the tile (2 halves of 128
//     rows x 3 x 32 TMEM columns; only dxd A_down when gu already holds g | u), one item ahead of the
//     element-wise warps;
//   * warp 16, once those warps stored the tile's dg | du | h (bf16, [256 x 32] each, the g tile's layout) in
//     shared memory: the per-row products [dg B_gate | du B_up | h A_down^T], accumulated in TMEM over the
//     run's tiles of the row block (2 halves x 48 columns; B_gate / B_up slices read as MN-major B), and
//     the column products [dg | du | h]^T [xa_gate | xa_up | dxd] over the block's 256 rows: one M = 128,
//     N = 48 MMA per 16 rows with the three 32-column tiles as MN-major A (M atoms 16 KB apart; the
//     fourth atom reads the row buffers and lands in result rows 96-127, which nobody reads) and the three
//     row buffers as MN-major B (N atoms 8 KB apart).  The diagonal 32 x 16 blocks of the 128 x 48 result
//     are dB_gate^T, dB_up^T and dA_down^T of the tile; two result buffers alternate.
// Warps 0-15: warp w holds block rows 128 h + 32 q + lane (h = (w / 4) % 2, q = w % 4: its TMEM lane
// quarter) and columns 16 c .. 16 c + 15 (c = w / 8) of the tile; warps w and w + 8 form a pair that
// shares rows.  Each thread reads its LoRA terms from TMEM and g, u, dh from shared memory, computes
// dg, du and h with the reference's rounding points, and quantizes dg and du: the two threads of a row
// exchange their half-block abs-maxima through shared memory, and the codes leave through shared memory
// as one TMA store per warp.  The warps then store the operand tiles and drain the finished products into
// the fp32 partial buffers (warps 0-2: the previous tile's column products; all: the per-row products
// when the run leaves a row block).  Every wait is bounded, and the two warps of a pair leave together;
// no atomics, so the result is deterministic.
constexpr int BT_ROWS = 256, BT_BN = 32, BT_ST = 3, BT_CONS = 16, BT_THREADS = 32 * (BT_CONS + 3);
constexpr int BT_W_PROD = BT_CONS, BT_W_TMA = BT_CONS + 1, BT_W_REC = BT_CONS + 2;   // warp roles
constexpr int BT_TILE = BT_ROWS * BT_BN * 2;           // 16 KB: [256 x 32] bf16
constexpr int BT_SLICE = 32 * 16 * 2;                  // 1 KB: [32 x 16] or [16 x 32] bf16
constexpr int BT_STAGE = 3 * BT_TILE + 3 * BT_SLICE;   // g | u | dh | bg | bu | ad
constexpr int BT_RB = BT_ROWS * 16 * 2;                // 8 KB: one [256 x 16] row buffer
constexpr int BT_NBARS = 2 * BT_ST + 12;
constexpr size_t BT_SMEM = 1024 + (size_t)BT_ST * BT_STAGE + 3 * BT_TILE + 3 * BT_RB + BT_NBARS * 8 + 16;
static_assert(BT_SMEM <= 232448, "backward epilogue: shared memory");
static_assert(BT_STAGE % 1024 == 0 && BT_RB % 1024 == 0, "backward epilogue: swizzle alignment");
// TMEM columns: LoRA terms (2 halves x [g | u | dh] x 32), per-row products (2 halves x 48), column
// products (2 buffers x 48)
constexpr uint32_t BT_REC = 0, BT_ROWC = 192, BT_COLC = 288, BT_TMEM_COLS = 512;

// GL: gu already holds g and u with their LoRA terms (the fused gate|up kernel writes them so): the LoRA-term
// MMAs and adds of g and u are skipped, only dxd A_down is computed.
template <bool GL>
__global__ void __launch_bounds__(BT_THREADS, 1)
    k_mlp_bwd_tc(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dh,
                 const __grid_constant__ CUtensorMap tm_bg, const __grid_constant__ CUtensorMap tm_bu,
                 const __grid_constant__ CUtensorMap tm_ad, const __grid_constant__ CUtensorMap tm_xs,
                 const __grid_constant__ CUtensorMap tm_dxd, const __grid_constant__ CUtensorMap tm_q,
                 uint8_t* __restrict__ s, float* __restrict__ dxa_part, float* __restrict__ dbg_part,
                 float* __restrict__ dbu_part, float* __restrict__ dad_part, int T, int Tpad, int N, float s_g,
                 float s_u, int per, int write_q, int* err) {
  constexpr int R = 16, R3 = 3 * R;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* opbuf = smem + BT_ST * BT_STAGE;   // dg | du | h tiles
  uint8_t* rowbuf = opbuf + 3 * BT_TILE;      // xa_gate | xa_up | dxd rows of the block
  uint64_t* full = reinterpret_cast<uint64_t*>(rowbuf + 3 * BT_RB);   // [BT_ST] TMA bytes of a stage
  uint64_t* empty = full + BT_ST;             // [BT_ST] 16 element-wise warps + the commit of the tile's products
  uint64_t* rows_full = empty + BT_ST;        // TMA bytes of a block's row buffers
  uint64_t* rows_empty = rows_full + 1;       // commit after the block's last products
  uint64_t* lora_full = rows_full + 2;        // commit after a tile's LoRA-term MMAs
  uint64_t* lora_empty = rows_full + 3;       // 16 element-wise warps read the LoRA terms
  uint64_t* op_full = rows_full + 4;          // 16 element-wise warps stored dg | du | h
  uint64_t* op_empty = rows_full + 5;         // commit after the tile's products
  uint64_t* colp_full = rows_full + 6;        // [2] commit after a tile's column products
  uint64_t* colp_empty = rows_full + 8;       // [2] warps 0-2 drained them
  uint64_t* row_full = rows_full + 10;        // commit after a block's last per-row products
  uint64_t* row_empty = rows_full + 11;       // 16 element-wise warps drained them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rows_full + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = N / BT_BN;
  const int items = ((Tpad + BT_ROWS - 1) / BT_ROWS) * nt;
  const int it_lo = blockIdx.x * per, it_hi = min(it_lo + per, items), cnt = max(it_hi - it_lo, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < BT_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], BT_CONS + 1);
    }
    mbar_init(rows_full, 1);
    mbar_init(rows_empty, 1);
    mbar_init(lora_full, 1);
    mbar_init(lora_empty, BT_CONS);
    mbar_init(op_full, BT_CONS);
    mbar_init(op_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&colp_full[i], 1);
      mbar_init(&colp_empty[i], 3);
    }
    mbar_init(row_full, 1);
    mbar_init(row_empty, BT_CONS);
    fence_barrier_init();
  }
  if (warp == BT_W_PROD) tmem_alloc(tmem_slot, BT_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s_ring = smem_u32(smem), s_op = smem_u32(opbuf), s_rows = smem_u32(rowbuf);

  if (warp == BT_W_TMA) {   // TMA producer: the ring, and the row buffers when a row block starts
    if (lane == 0) {
      prefetch_tmap(&tm_gu);
      prefetch_tmap(&tm_dh);
      prefetch_tmap(&tm_bg);
      prefetch_tmap(&tm_bu);
      prefetch_tmap(&tm_ad);
      prefetch_tmap(&tm_xs);
      prefetch_tmap(&tm_dxd);
    }
    // two queues polled in turn (lane 0 tests, the warp follows): the next row block's rows (once the
    // previous block's products are done: rows_empty) and the next tile (once its stage is free)
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0, row_loads = 0, rows_at = 0;   // rows_at: local index of the next row block's first tile
    uint64_t t0 = mx_globaltimer();
    while (issued < cnt || rows_at < cnt) {
      bool prog = false;
      if (rows_at < cnt &&
          (row_loads == 0 ||
           __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(rows_empty, (uint32_t)((row_loads - 1) & 1)) : 0, 0))) {
        const int sbr = (it_lo + rows_at) / nt;
        if (lane == 0) {
          mbar_arrive_expect_tx(rows_full, 3 * BT_RB);
          tma_load_2d(rowbuf, &tm_xs, rows_full, 0, sbr * BT_ROWS);
          tma_load_2d(rowbuf + BT_RB, &tm_xs, rows_full, R, sbr * BT_ROWS);
          tma_load_2d(rowbuf + 2 * BT_RB, &tm_dxd, rows_full, 0, sbr * BT_ROWS);
        }
        __syncwarp();
        ++row_loads;
        rows_at = (sbr + 1) * nt - it_lo;
        prog = true;
      }
      if (issued < cnt && __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(&empty[stage], phase ^ 1) : 0, 0)) {
        const int it = it_lo + issued;
        const int n0 = (it % nt) * BT_BN, r0 = (it / nt) * BT_ROWS;
        if (lane == 0) {
          uint8_t* dst = smem + stage * BT_STAGE;
          uint64_t* fb = &full[stage];
          mbar_arrive_expect_tx(fb, BT_STAGE);
          tma_load_2d(dst, &tm_gu, fb, n0, r0);
          tma_load_2d(dst + BT_TILE, &tm_gu, fb, N + n0, r0);
          tma_load_2d(dst + 2 * BT_TILE, &tm_dh, fb, n0, r0);
          tma_load_2d(dst + 3 * BT_TILE, &tm_bg, fb, 0, n0);
          tma_load_2d(dst + 3 * BT_TILE + BT_SLICE, &tm_bu, fb, 0, n0);
          tma_load_2d(dst + 3 * BT_TILE + 2 * BT_SLICE, &tm_ad, fb, n0, 0);
        }
        __syncwarp();
        ++issued;
        if (++stage == BT_ST) {
          stage = 0;
          phase ^= 1;
        }
        prog = true;
      }
      if (prog) {
        t0 = mx_globaltimer();
      } else {
        if (mx_globaltimer() - t0 > MX_WAIT_LIMIT_NS) {
          if (lane == 0) mx_set_error(err, MX_DEV_TIMEOUT_PRODUCER);
          break;
        }
        __nanosleep(64);
      }
    }
    // leave no copy in flight: wait (bounded) for the last load of every stage that was used
    for (int k = 0; k < BT_ST && k < issued; ++k) {
      const int i = issued - 1 - k, st = i % BT_ST;
      mbar_wait(&full[st], (uint32_t)((i / BT_ST) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
    }
    if (row_loads > 0) mbar_wait(rows_full, (uint32_t)((row_loads - 1) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
  } else if (warp == BT_W_REC) {   // LoRA-term MMAs: the whole warp waits, lane 0 issues and commits
    // descriptors of stage 0 / row half 0; the start-address field (address / 16) takes plain offsets
    constexpr uint32_t ID_REC = f16_idesc(128, 32, false, false);      // B = B_gate / B_up slice [32 n][16 k]
    constexpr uint32_t ID_REC_AD = f16_idesc(128, 32, false, true);    // B = A_down slice [16 k][32 n]
    const uint32_t sl0 = s_ring + 3 * BT_TILE;                         // bg | bu | ad slices of stage 0
    const uint64_t a_xg = make_sdesc(s_rows, 0, 256, 6), a_xu = make_sdesc(s_rows + BT_RB, 0, 256, 6);
    const uint64_t a_xd = make_sdesc(s_rows + 2 * BT_RB, 0, 256, 6);
    const uint64_t b_g = make_sdesc(sl0, 0, 256, 6), b_u = make_sdesc(sl0 + BT_SLICE, 0, 256, 6);
    const uint64_t b_d = make_sdesc(sl0 + 2 * BT_SLICE, BT_SLICE, 512, 4);
    int n_rec = 0, blk = -1;
    for (int t = 0; t < cnt; ++t) {
      const int it = it_lo + t, st = t % BT_ST;
      const bool first = t == 0 || it % nt == 0;
      if (first) ++blk;
      if (first && !mbar_wait(rows_full, (uint32_t)(blk & 1), err, MX_DEV_TIMEOUT_MMA)) break;
      if (!mbar_wait(&full[st], (uint32_t)((t / BT_ST) & 1), err, MX_DEV_TIMEOUT_MMA)) break;
      if (t > 0 && !mbar_wait(lora_empty, (uint32_t)((t - 1) & 1), err, MX_DEV_TIMEOUT_MMA_TMEM)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t so = (uint64_t)((st * BT_STAGE) >> 4);
#pragma unroll
        for (int h = 0; h < 2; ++h) {   // rows 128 h .. 128 h + 127 (4 KB into each row buffer)
          const uint32_t d = tmem + BT_REC + 96 * h;
          const uint64_t ho = (uint64_t)(256 * h);
          if constexpr (!GL) {
            umma_bf16(d, a_xg + ho, b_g + so, ID_REC, 0u);
            umma_bf16(d + 32, a_xu + ho, b_u + so, ID_REC, 0u);
          }
          umma_bf16(d + 64, a_xd + ho, b_d + so, ID_REC_AD, 0u);
        }
        umma_commit(lora_full);
      }
      __syncwarp();
      ++n_rec;
    }
    if (n_rec > 0) mbar_wait(lora_full, (uint32_t)((n_rec - 1) & 1), err, MX_DEV_TIMEOUT_MMA);   // none in flight
  } else if (warp == BT_W_PROD) {   // product MMAs: the whole warp waits, lane 0 issues and commits
    constexpr uint32_t ID_ROW = f16_idesc(128, 16, false, false);      // B = A_down slice [16 n][32 k]
    constexpr uint32_t ID_ROW_MN = f16_idesc(128, 16, false, true);    // B = B_gate / B_up slice [32 k][16 n]
    constexpr uint32_t ID_COL = f16_idesc(128, 48, true, true);        // A = [dg | du | h] tiles, B = rows
    const uint32_t sl0 = s_ring + 3 * BT_TILE;
    // per-row products: A = dg / du / h tile (K-major, rows 128 h .., K step 32 bytes); B = the stage's slices
    const uint64_t a_r = make_sdesc(s_op, 0, 512, 4);
    const uint64_t b_rg = make_sdesc(sl0, BT_SLICE, 256, 6), b_ru = make_sdesc(sl0 + BT_SLICE, BT_SLICE, 256, 6);
    const uint64_t b_rd = make_sdesc(sl0 + 2 * BT_SLICE, 0, 512, 4);
    // column products: A = the three tiles as MN-major atoms 16 KB apart, B = the row buffers 8 KB apart
    const uint64_t a_c = make_sdesc(s_op, BT_TILE, 512, 4), b_c = make_sdesc(s_rows, BT_RB, 256, 6);
    int n_prod = 0, blk = -1;
    for (int t = 0; t < cnt; ++t) {
      const int it = it_lo + t;
      const bool first = t == 0 || it % nt == 0;
      const bool last = t + 1 == cnt || (it + 1) % nt == 0;
      if (first) ++blk;
      if (!mbar_wait(op_full, (uint32_t)(t & 1), err, MX_DEV_TIMEOUT_MMA)) break;
      if (t >= 2 && !mbar_wait(&colp_empty[t & 1], (uint32_t)(((t - 2) >> 1) & 1), err, MX_DEV_TIMEOUT_MMA_TMEM))
        break;
      if (first && blk > 0 && !mbar_wait(row_empty, (uint32_t)((blk - 1) & 1), err, MX_DEV_TIMEOUT_MMA_TMEM)) break;
      tc_fence_after();
      if (lane == 0) {
        const int st = t % BT_ST;
        const uint64_t so = (uint64_t)((st * BT_STAGE) >> 4);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t d = tmem + BT_ROWC + 48 * h;
#pragma unroll
          for (int k = 0; k < 2; ++k) {   // K = the tile's 32 columns, 16 per MMA
            const uint32_t acc = (first && k == 0) ? 0u : 1u;
            const uint64_t ao = (uint64_t)(512 * h + 2 * k);   // 8 KB per row half, 32 bytes per K step
            umma_bf16(d, a_r + ao, b_rg + so + 32 * k, ID_ROW_MN, acc);
            umma_bf16(d + 16, a_r + ao + BT_TILE / 16, b_ru + so + 32 * k, ID_ROW_MN, acc);
            umma_bf16(d + 32, a_r + ao + 2 * BT_TILE / 16, b_rd + so + 2 * k, ID_ROW, acc);
          }
        }
        const uint32_t dc = tmem + BT_COLC + 48 * (uint32_t)(t & 1);
#pragma unroll
        for (int k = 0; k < BT_ROWS / 16; ++k)   // K = the block's 256 rows, 16 per MMA (1 KB of A, 512 B of B)
          umma_bf16(dc, a_c + 64 * k, b_c + 32 * k, ID_COL, k > 0 ? 1u : 0u);
        umma_commit(op_empty);
        umma_commit(&empty[st]);
        umma_commit(&colp_full[t & 1]);
        if (last) {
          umma_commit(row_full);
          umma_commit(rows_empty);
        }
      }
      __syncwarp();
      ++n_prod;
    }
    if (n_prod > 0) mbar_wait(op_empty, (uint32_t)((n_prod - 1) & 1), err, MX_DEV_TIMEOUT_MMA);   // none in flight
  } else {   // element-wise warps 0-15
    const int c = warp >> 3, hq = warp & 7, half = hq >> 2, qw = hq & 3;
    const int r0w = half * 128 + qw * 32;                 // first block row of the pair (warps hq, hq + 8)
    const int rl = r0w + lane;                            // this thread's block row
    const uint32_t pid = 1u + (uint32_t)hq;               // the pair's named barrier
    const uint32_t lb = (uint32_t)(qw * 32) << 16;        // TMEM lane quarter
    const uint32_t trec = tmem + lb + BT_REC + 96 * half + 16 * c, trow = tmem + lb + BT_ROWC + 48 * half;
    const uint32_t o_row = (uint32_t)rl * 64, sw = (uint32_t)((rl >> 1) & 3);   // 64-byte rows, 64-byte swizzle
    const float2 sg2 = make_float2(s_g, s_g), su2 = make_float2(s_u, s_u);
    const int64_t N2 = 2 * (int64_t)N;
    const uint64_t pol = l2_evict_first();
    // column products of local tile tt (warps 0-2, TMEM lane quarters 0-2: dg, du, h columns)
    auto drain_col = [&](int tt, int64_t sbt, int64_t nt0) -> bool {
      const int b = tt & 1;
      if (!mbar_wait(&colp_full[b], (uint32_t)((tt >> 1) & 1), err, MX_DEV_TIMEOUT_EPILOGUE)) return false;
      tc_fence_after();
      uint32_t v[16];
      tmem_ld16(tmem + lb + BT_COLC + 48 * b + 16 * warp, v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&colp_empty[b]);
      const int64_t n = nt0 + lane;
      if (warp < 2) {   // [n_blocks, N, r]: element (n, j)
        uint4* P = reinterpret_cast<uint4*>((warp == 0 ? dbg_part : dbu_part) + (sbt * N + n) * R);
#pragma unroll
        for (int k = 0; k < 4; ++k) P[k] = make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      } else {          // [n_blocks, r, N]: element (j, n)
        float* P = dad_part + sbt * R * N + n;
#pragma unroll
        for (int j = 0; j < R; ++j) P[(int64_t)j * N] = __uint_as_float(v[j]);
      }
      return true;
    };
    int stage = 0;
    uint32_t phase = 0;
    int blk = -1;
    bool ok = true;
    // the item's row block and first column, stepped per tile (no divisions in the loop), and this row's
    // scale-byte offset up to the column block (the scale buffer is far below 2^31 bytes)
    int sbi = it_lo / nt, n0 = (it_lo % nt) * BT_BN;
    int row = 0, srow = 0;
    for (int t = 0; t < cnt; ++t) {
      const bool last = t + 1 == cnt || n0 + BT_BN == N;
      if (t == 0 || n0 == 0) {
        ++blk;
        row = sbi * BT_ROWS + rl;
        srow = (int)mx_scale_offset(row < Tpad ? row : 0, 0, N2);
      }
      const bool good = ok && mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE) &&
                        mbar_wait(lora_full, (uint32_t)(t & 1), err, MX_DEV_TIMEOUT_EPILOGUE);
      if (bar_any(pid, 64, !good)) {   // both warps of the pair leave together
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = s_ring + (uint32_t)stage * BT_STAGE;
      uint32_t pg[8], pu[8], ph[8];   // dg, du, h of the thread's 16 columns, bf16 pairs
#pragma unroll
      for (int k = 0; k < 2; ++k) {   // 8 columns at a time: 16 c + 8 k ..
        uint32_t lg[8], lu[8], ld[8], G[4], U[4], D[4];
        if constexpr (!GL) {
          tmem_ld8(trec + 8 * k, lg);
          tmem_ld8(trec + 32 + 8 * k, lu);
        }
        tmem_ld8(trec + 64 + 8 * k, ld);
        const uint32_t a = sb + o_row + (((uint32_t)(2 * c + k) ^ sw) << 4);
        lds128(a, G);
        lds128(a + BT_TILE, U);
        lds128(a + 2 * BT_TILE, D);
        tmem_ld_wait();
        if (k == 1) {   // the LoRA terms are in registers: the next tile's may overwrite them
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(lora_empty);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 gg = up2(G[e]), uu = up2(U[e]);
          if constexpr (!GL) {   // g = bf16(gu_gate + s_g xa_g B_gate^T), u likewise
            gg = up2(rn2(__ffma2_rn(sg2, make_float2(__uint_as_float(lg[2 * e]), __uint_as_float(lg[2 * e + 1])), gg)));
            uu = up2(rn2(__ffma2_rn(su2, make_float2(__uint_as_float(lu[2 * e]), __uint_as_float(lu[2 * e + 1])), uu)));
          }
          const float2 sig = sigmoid2(gg);
          const float2 sl = __fmul2_rn(gg, sig);                                 // silu(g)
          ph[4 * k + e] = rn2(__fmul2_rn(sl, uu));                                // h = bf16(silu * u)
          const float2 dh = up2(rn2(add_bf16x2_f32(D[e], make_float2(__uint_as_float(ld[2 * e]), __uint_as_float(ld[2 * e + 1])))));
          pu[4 * k + e] = rn2(__fmul2_rn(dh, sl));                                // du = bf16(dh * silu)
          const float2 om = __ffma2_rn(sig, make_float2(-1.f, -1.f), make_float2(1.f, 1.f));   // 1 - sig
          const float2 f = __ffma2_rn(gg, om, make_float2(1.f, 1.f));             // g (1 - sig) + 1
          pg[4 * k + e] = rn2(__fmul2_rn(__fmul2_rn(__fmul2_rn(dh, uu), sig), f));   // dg
        }
      }
      // (1) both warps of the pair have read the stage's rows r0w .. r0w + 31: from here on the pair's u rows
      // carry the abs-max exchange and its g rows the staged codes
      bar_sync(pid, 64);
      const uint32_t xch = sb + BT_TILE + (uint32_t)r0w * 64 + (uint32_t)lane * 8;   // 8 bytes per row
      uint32_t amx = 0;   // abs-max of this thread's 16 columns: dg (low half) | du (high half), signs cleared
      if (write_q) {
        uint32_t mg = amax_xs_bf16x2(amax_xs_bf16x2(pg[0], pg[1]), amax_xs_bf16x2(pg[2], pg[3]));
        mg = amax_xs_bf16x2(mg, amax_xs_bf16x2(amax_xs_bf16x2(pg[4], pg[5]), amax_xs_bf16x2(pg[6], pg[7])));
        uint32_t mu = amax_xs_bf16x2(amax_xs_bf16x2(pu[0], pu[1]), amax_xs_bf16x2(pu[2], pu[3]));
        mu = amax_xs_bf16x2(mu, amax_xs_bf16x2(amax_xs_bf16x2(pu[4], pu[5]), amax_xs_bf16x2(pu[6], pu[7])));
        // each half of mg / mu is a column-parity maximum: fold them, (dg | du) in one bf16x2
        amx = amax_xs_bf16x2(__byte_perm(mg, mu, 0x5410), __byte_perm(mg, mu, 0x7632)) & 0x7FFF7FFFu;
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(xch + 4 * c), "r"(amx) : "memory");
      }
      bar_sync(pid, 64);   // (2)
      if (write_q) {
        uint32_t oth;
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(oth) : "r"(xch + 4 * (1 - c)) : "memory");
        const uint32_t mm = max_bf16x2(amx, oth);   // the rows' 32-column abs-maxima (NaN propagates)
        const uint32_t eg = mx_e8m0_of_amax(bf16_lo(mm)), eu = mx_e8m0_of_amax(bf16_hi(mm));
        const uint16_t rg = (uint16_t)(__float_as_uint(mx_e8m0_rcp(eg)) >> 16);
        const uint16_t ru = (uint16_t)(__float_as_uint(mx_e8m0_rcp(eu)) >> 16);
        uint32_t wg[4], wu[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 g0 = scale_bf16x2(pg[2 * k], rg), g1 = scale_bf16x2(pg[2 * k + 1], rg);
          const float2 u0 = scale_bf16x2(pu[2 * k], ru), u1 = scale_bf16x2(pu[2 * k + 1], ru);
          wg[k] = e4m3x2_sat(g0.x, g0.y) | (e4m3x2_sat(g1.x, g1.y) << 16);
          wu[k] = e4m3x2_sat(u0.x, u0.y) | (e4m3x2_sat(u1.x, u1.y) << 16);
        }
        // the warp's [32 rows][dg | du][16] code box, in the pair's g rows (1 KB per warp)
        const uint32_t box = sb + (uint32_t)r0w * 64 + (uint32_t)c * 1024;
        sts128(box + (uint32_t)lane * 32, wg);
        sts128(box + (uint32_t)lane * 32 + 16, wu);
        fence_proxy_async();
        __syncwarp();
        const int64_t z = (int64_t)sbi * BT_ROWS + r0w;
        if (lane == 0 && z < T) {   // rows >= T of the box are clipped by the store
          tma_store_3d_hint(&tm_q, smem + (box - s_ring), n0 + 16 * c, 0, (int)z, pol);
          bulk_commit();
        }
        // the scale bytes: dg's by the thread of column half 0, du's by the other
        if (row < Tpad)
          stg8_if_hint(s + srow + (((c == 0 ? n0 : N + n0) >> 7) << 9) + ((n0 >> 5) & 3), c == 0 ? eg : eu, true, pol);
      }
      // dg | du | h into the operand tiles, once the previous tile's products have read them
      if (t > 0 && !mbar_wait(op_empty, (uint32_t)((t - 1) & 1), err, MX_DEV_TIMEOUT_EPILOGUE)) ok = false;
      if (ok) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint32_t a = s_op + o_row + (((uint32_t)(2 * c + k) ^ sw) << 4);
          sts128(a, pg + 4 * k);
          sts128(a + BT_TILE, pu + 4 * k);
          sts128(a + 2 * BT_TILE, ph + 4 * k);
        }
        fence_proxy_async();   // read next by the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(op_full);
      }
      if (ok && warp < 3 && t > 0 && !drain_col(t - 1, n0 ? sbi : sbi - 1, n0 ? n0 - BT_BN : N - BT_BN)) ok = false;
      if (ok && last) {   // leaving the row block: its per-row products into this CTA's slot
        if (!mbar_wait(row_full, (uint32_t)(blk & 1), err, MX_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
        } else {
          tc_fence_after();
          uint32_t v0[16], v1[16];   // column half 0: dg B_gate and h A_down^T; half 1: du B_up
          tmem_ld16(trow + (c == 0 ? 0 : 16), v0);
          if (c == 0) tmem_ld16(trow + 32, v1);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(row_empty);
          if (row < T) {
            const int slot = (int)blockIdx.x - (sbi * nt) / per;
            uint4* P = reinterpret_cast<uint4*>(dxa_part + ((int64_t)slot * T + row) * R3) + (c == 0 ? 0 : 4);
#pragma unroll
            for (int k = 0; k < 4; ++k) P[k] = make_uint4(v0[4 * k], v0[4 * k + 1], v0[4 * k + 2], v0[4 * k + 3]);
            if (c == 0) {
#pragma unroll
              for (int k = 0; k < 4; ++k) P[8 + k] = make_uint4(v1[4 * k], v1[4 * k + 1], v1[4 * k + 2], v1[4 * k + 3]);
            }
          }
        }
      }
      // the stage is free once the code store has read its g rows
      if (write_q && lane == 0) bulk_wait_read0();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == BT_ST) {
        stage = 0;
        phase ^= 1;
      }
      if ((n0 += BT_BN) == N) {
        n0 = 0;
        ++sbi;
      }
    }
    if (ok && warp < 3 && cnt > 0) drain_col(cnt - 1, n0 ? sbi : sbi - 1, n0 ? n0 - BT_BN : N - BT_BN);
    if (write_q && lane == 0) bulk_wait0();   // the code stores are complete
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == BT_W_PROD) tmem_dealloc(tmem, BT_TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------ skinny
// E4M3 bytes that are NaN (S.1111.111) -> the canonical 0x7F, four codes per word.
MX_DEV uint32_t nan_canon4(uint32_t w) {
  const uint32_t m = ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
  return w & ~m;
}

// Row-wise MXFP8 of the 8 bf16 of a 16-byte vector held by this lane, where lanes 4g .. 4g+3 hold
// one 32-element block of a row (the quantizer's algorithm, scripts/mxfp8.py:46-75): the block's
// E8M0 scale goes to `e`, the 8 E4M3 codes are returned.
MX_DEV uint2 quant8_lane(const uint4& v, uint32_t& e) {
  const uint32_t m2 = max_bf16x2(absmax_bf16x2(v.x, v.y), absmax_bf16x2(v.z, v.w));
  float m = nanmax(bf16_lo(m2), bf16_hi(m2));
  m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, 2));
  e = mx_e8m0_of_amax(m);
  const float rcp = mx_e8m0_rcp(e);
  const float2 r2 = make_float2(rcp, rcp);
  const float2 f0 = __fmul2_rn(up2(v.x), r2), f1 = __fmul2_rn(up2(v.y), r2);
  const float2 f2 = __fmul2_rn(up2(v.z), r2), f3 = __fmul2_rn(up2(v.w), r2);
  return make_uint2(nan_canon4(e4m3x2_sat(f0.x, f0.y) | (e4m3x2_sat(f1.x, f1.y) << 16)),
                    nan_canon4(e4m3x2_sat(f2.x, f2.y) | (e4m3x2_sat(f3.x, f3.y) << 16)));
}

// out[t, j] = bf16( bf16(sum_k A[t, k] B[j, k]) * post ) for j < NJ (16, 32 or 64); post == 1 skips
// the second rounding; with round_once, bf16(sum * post) (one rounding).  CTA = 16 rows; its 4 warps split K in four and their fp32 partials are summed
// through shared memory in a fixed order.  The reduction index k is permuted consistently in A and B so
// each lane loads 16 contiguous bytes per row per 32 k; a group of 32-k steps (four for n <= 32, two
// for n = 64) has all its A vectors and B fragments requested before any is used, so a group costs
// one memory latency.  With QUANT the same registers are also quantized row-wise to MXFP8
// (codes q [T, K] at row stride ldq; scales in the blocked layout of a [Tpad, scols] operand from k-block
// kb_off on), since the 4 lanes holding a row's 32 k are exactly one MX block: one read of A serves both.
// The QUANT grid covers Tpad rows.
template <int NJ, bool QUANT>
__global__ void __launch_bounds__(128) k_rowdot(const bf16* __restrict__ A, int64_t lda, const bf16* __restrict__ B,
                                                int T, int K, float post, int round_once, bf16* __restrict__ out,
                                                int64_t ldo, uint8_t* __restrict__ q, int64_t ldq,
                                                uint8_t* __restrict__ s, int64_t scols, int kb_off) {
  __shared__ float red[4][16][NJ + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t r0 = (int64_t)blockIdx.x * 16;
  const int64_t ra = r0 + g, rb = ra + 8;
  const bool va = ra < T, vb = rb < T;
  float acc[NJ / 8][4];
#pragma unroll
  for (int j = 0; j < NJ / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  const int kq = K / 4;  // this warp's quarter of K (K % 128 == 0)
  const int kb = warp * kq, ke = kb + kq;
  const bf16* pa = A + ra * lda + 8 * t;
  const bf16* pb = A + rb * lda + 8 * t;
  const bf16* pB = B + (int64_t)g * K + 8 * t;   // row 8 jt + g of B at + 8 jt K
  auto step = [&](const uint4& xa, const uint4& xb, const uint4 (&bb)[NJ / 8], int k0) {
    if (QUANT) {
      uint32_t ea, eb;
      const uint2 ca = quant8_lane(xa, ea), cb = quant8_lane(xb, eb);
      if (va) *reinterpret_cast<uint2*>(q + ra * ldq + k0 + 8 * t) = ca;
      if (vb) *reinterpret_cast<uint2*>(q + rb * ldq + k0 + 8 * t) = cb;
      if (t == 0) {
        s[mx_scale_offset(ra, kb_off + (k0 >> 5), scols)] = (uint8_t)ea;
        s[mx_scale_offset(rb, kb_off + (k0 >> 5), scols)] = (uint8_t)eb;
      }
    }
    // fragment k slots (2t, 2t+1 | 2t+8, 2t+9) <- actual k (8t, 8t+1 | 8t+2, 8t+3), then (8t+4.. | 8t+6..)
    const uint32_t a0[4] = {xa.x, xb.x, xa.y, xb.y};
    const uint32_t a1[4] = {xa.z, xb.z, xa.w, xb.w};
#pragma unroll
    for (int jt = 0; jt < NJ / 8; ++jt) {
      mma16816(acc[jt], a0, bb[jt].x, bb[jt].y);
      mma16816(acc[jt], a1, bb[jt].z, bb[jt].w);
    }
  };
  // GS 32-k steps per group: all of a group's A vectors and B fragments are requested before any is used
  constexpr int GS = NJ <= 32 ? 4 : 2;
  int k0 = kb;
  for (; k0 + 32 * GS <= ke; k0 += 32 * GS) {
    uint4 xa[GS], xb[GS], bb[GS][NJ / 8];
#pragma unroll
    for (int u = 0; u < GS; ++u) {
      xa[u] = va ? __ldg(reinterpret_cast<const uint4*>(pa + k0 + 32 * u)) : z;
      xb[u] = vb ? __ldg(reinterpret_cast<const uint4*>(pb + k0 + 32 * u)) : z;
#pragma unroll
      for (int jt = 0; jt < NJ / 8; ++jt)
        bb[u][jt] = __ldg(reinterpret_cast<const uint4*>(pB + (int64_t)8 * jt * K + k0 + 32 * u));
    }
#pragma unroll
    for (int u = 0; u < GS; ++u) step(xa[u], xb[u], bb[u], k0 + 32 * u);
  }
  for (; k0 < ke; k0 += 32) {
    const uint4 xa = va ? __ldg(reinterpret_cast<const uint4*>(pa + k0)) : z;
    const uint4 xb = vb ? __ldg(reinterpret_cast<const uint4*>(pb + k0)) : z;
    uint4 bb[NJ / 8];
#pragma unroll
    for (int jt = 0; jt < NJ / 8; ++jt) bb[jt] = __ldg(reinterpret_cast<const uint4*>(pB + (int64_t)8 * jt * K + k0));
    step(xa, xb, bb, k0);
  }
#pragma unroll
  for (int jt = 0; jt < NJ / 8; ++jt) {
    const int c = 8 * jt + 2 * t;
    red[warp][g][c] = acc[jt][0];
    red[warp][g][c + 1] = acc[jt][1];
    red[warp][g + 8][c] = acc[jt][2];
    red[warp][g + 8][c + 1] = acc[jt][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * NJ / 2; i += 128) {
    const int rr = i / (NJ / 2), c = 2 * (i % (NJ / 2));
    float v[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float sum = (red[0][rr][c + e] + red[1][rr][c + e]) + (red[2][rr][c + e] + red[3][rr][c + e]);
      if (round_once) {
        v[e] = bf16_round_f(sum * post);
      } else {
        v[e] = bf16_round_f(sum);
        if (post != 1.0f) v[e] = bf16_round_f(v[e] * post);
      }
    }
    if (r0 + rr < T) *reinterpret_cast<uint32_t*>(out + (r0 + rr) * ldo + c) = pack_bf16x2(v[0], v[1]);
  }
}

// The same products with TMA, for B small enough to stay in shared memory (NJ x K x 2 bytes <= RD_B_MAX):
// CTA = 128-row blocks (persistent, stride gridDim.x); warp 8 streams [128 rows x 64 k] boxes of A
// (128-byte swizzle) into an RD_ST-stage ring, and during the CTA's first row block also the matching
// [NJ x 64 k] boxes of B into a buffer that then serves every later block.  Consumer warps 0-7 each own
// 16 rows for the whole K: mma A fragments by ldmatrix from the ring, B fragments from the B buffer, fp32
// sums in registers, so no cross-warp reduction.  With QUANT the warp also quantizes its rows of each
// box straight from the ring, two lanes per 32-k block (the same arithmetic as quant8_lane), each lane
// storing 16 codes so that one store instruction covers 8 rows x 64 contiguous bytes.
constexpr int RD_ROWS = 128, RD_KB = 64, RD_CONS = 8;
constexpr int RD_A_BYTES = RD_ROWS * RD_KB * 2;   // 16 KB
constexpr size_t RD_SMEM_MAX = 220 * 1024, RD_B_MAX = RD_SMEM_MAX - 1024 - 2 * RD_A_BYTES - 256;
__host__ __device__ inline int rd_stages(int64_t b_bytes) {
  const int64_t st = ((int64_t)RD_SMEM_MAX - 1024 - 256 - b_bytes) / RD_A_BYTES;
  return st > 6 ? 6 : (int)st;
}
__host__ __device__ inline size_t rd_smem(int64_t b_bytes, int st) { return 1024 + (size_t)b_bytes + (size_t)st * RD_A_BYTES + 256; }

template <int NJ, bool QUANT>
__global__ void __launch_bounds__(32 * (RD_CONS + 1), 1)
    k_rowdot_tma(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int T, int K,
                 int nrb, int stages, float post, int round_once, bf16* __restrict__ out, int64_t ldo,
                 uint8_t* __restrict__ q, int64_t ldq, uint8_t* __restrict__ s, int64_t scols, int kb_off, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int nkb = K / RD_KB;
  uint8_t* sB = smem;                                            // [nkb][NJ rows x 128 B]
  uint8_t* sA = sB + (size_t)nkb * NJ * 128;                     // [stages][128 rows x 128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(sA + (size_t)stages * RD_A_BYTES);
  uint64_t* empty = full + stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], RD_CONS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == RD_CONS) {   // TMA producer
    int stage = 0, issued = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int rb = blockIdx.x, first = 1; rb < nrb && ok; rb += gridDim.x, first = 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], RD_A_BYTES + (first ? NJ * 128 : 0));
          tma_load_2d(sA + (size_t)stage * RD_A_BYTES, &tm_a, &full[stage], kb * RD_KB, rb * RD_ROWS);
          if (first) tma_load_2d(sB + (size_t)kb * NJ * 128, &tm_b, &full[stage], kb * RD_KB, 0);
        }
        __syncwarp();
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    for (int k = 0; k < stages && k < issued; ++k) {   // no copy left in flight
      const int i = issued - 1 - k;
      mbar_wait(&full[i % stages], (uint32_t)((i / stages) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3, mi = lane >> 3, lr = lane & 7;
  // ldmatrix offsets within a box: A rows 16 warp + 8 (mi & 1) + lr, k-chunk 2 kk + (mi >> 1);
  // B rows (n) 8 (2 jp + (mi >> 1)) + lr, k-chunk 2 kk + (mi & 1)
  const uint32_t arow = (uint32_t)(warp * 16 + (mi & 1) * 8 + lr);
  const uint32_t s_a = smem_u32(sA), s_b = smem_u32(sB);
  int stage = 0;
  uint32_t phase = 0;
  // MXFP8 store targets: lanes 4i .. 4i+3 hold row 8 pass + i of the warp's 16, (block 0 | 1) x
  // (16-element half 0 | 1) of each 64-element k box
  const uint32_t qblk = (uint32_t)((lane >> 1) & 1), qhalf = (uint32_t)(lane & 1);
  for (int rb = blockIdx.x; rb < nrb; rb += gridDim.x) {
    float acc[NJ / 8][4];
#pragma unroll
    for (int j = 0; j < NJ / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // per row block: the two rows' code pointers, store predicates and scale offsets up to the k block
    // (stepped per k box below, no 64-bit arithmetic in the loop)
    uint8_t* qrow[2];
    int64_t srow[2];
    bool qlive[2];
    if (QUANT) {
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int64_t rg_ = (int64_t)rb * RD_ROWS + warp * 16 + 8 * pass + (lane >> 2);
        qlive[pass] = rg_ < T;
        qrow[pass] = q + (qlive[pass] ? rg_ : 0) * ldq + 32 * qblk + 16 * qhalf;
        srow[pass] = mx_scale_offset(rg_, 0, scols);
      }
    }
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      const uint32_t ab = s_a + (uint32_t)stage * RD_A_BYTES, bb = s_b + (uint32_t)kb * NJ * 128;
#pragma unroll
      for (int kk = 0; kk < RD_KB / 16; ++kk) {
        uint32_t A[4];
        ldsm4(A, ab + swz<128>(arow, (uint32_t)(2 * kk + (mi >> 1))));
#pragma unroll
        for (int jp = 0; jp < NJ / 16; ++jp) {
          uint32_t B[4];
          ldsm4(B, bb + swz<128>((uint32_t)(8 * (2 * jp + (mi >> 1)) + lr), (uint32_t)(2 * kk + (mi & 1))));
          mma16816(acc[2 * jp], A, B[0], B[1]);
          mma16816(acc[2 * jp + 1], A, B[2], B[3]);
        }
      }
      if (QUANT) {
        // two passes of 8 rows: lanes 4i .. 4i+3 hold row 8 pass + i of the warp's 16 -- (block 0 | 1) x
        // (16-element half 0 | 1) -- so each store instruction writes 8 rows x 64 contiguous bytes
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const uint32_t row = (uint32_t)(warp * 16 + 8 * pass + (lane >> 2));
          uint32_t v[8];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t a = ab + swz<128>(row, 4 * qblk + 2 * qhalf + (uint32_t)c);
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v[4 * c]), "=r"(v[4 * c + 1]), "=r"(v[4 * c + 2]), "=r"(v[4 * c + 3]) : "r"(a));
          }
          const uint32_t m4 = max_bf16x2(max_bf16x2(absmax_bf16x2(v[0], v[1]), absmax_bf16x2(v[2], v[3])),
                                         max_bf16x2(absmax_bf16x2(v[4], v[5]), absmax_bf16x2(v[6], v[7])));
          float m = nanmax(bf16_lo(m4), bf16_hi(m4));
          m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, 1));   // the other half of the 32-k block
          const uint32_t e = mx_e8m0_of_amax(m);
          const float rcp = mx_e8m0_rcp(e);
          const float2 r2 = make_float2(rcp, rcp);
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 x0 = __fmul2_rn(up2(v[2 * i]), r2), x1 = __fmul2_rn(up2(v[2 * i + 1]), r2);
            w[i] = nan_canon4(e4m3x2_sat(x0.x, x0.y) | (e4m3x2_sat(x1.x, x1.y) << 16));
          }
          stg128_if(qrow[pass] + kb * RD_KB, w[0], w[1], w[2], w[3], qlive[pass]);
          // the row's two scale bytes (k-blocks 2 kb, 2 kb + 1: adjacent in the blocked layout)
          const uint32_t e1 = __shfl_xor_sync(0xffffffffu, e, 2);
          const int kba = kb_off + 2 * kb;
          if ((lane & 3) == 0)
            *reinterpret_cast<uint16_t*>(s + srow[pass] + ((kba >> 2) << 9) + (kba & 3)) = (uint16_t)(e | (e1 << 8));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
    const int64_t r0 = (int64_t)rb * RD_ROWS + warp * 16 + g;
#pragma unroll
    for (int jt = 0; jt < NJ / 8; ++jt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float sum = acc[jt][2 * h + e];
          if (round_once) {
            v[e] = bf16_round_f(sum * post);
          } else {
            v[e] = bf16_round_f(sum);
            if (post != 1.0f) v[e] = bf16_round_f(v[e] * post);
          }
        }
        const int64_t row = r0 + 8 * h;
        if (row < T) *reinterpret_cast<uint32_t*>(out + row * ldo + 8 * jt + 2 * t) = pack_bf16x2(v[0], v[1]);
      }
    }
  }
}

// Launches the TMA row-product kernel when B fits in shared memory and the code rows allow 16-byte
// stores; returns -1 (nothing launched) otherwise, so the caller can fall back to k_rowdot.
// rowdot_tma's answer when the request does not fit the TMA kernel (B too large, K or a stride or a pointer
// not aligned for TMA): the caller runs k_rowdot.  Never an MXM status; a real failure returns its status.
constexpr int RD_NOT_APPLICABLE = 1;

int rowdot_tma(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post, int round_once,
               void* out, int64_t ldo, uint8_t* q, int64_t ldq, uint8_t* s, int64_t scols, int kb_off,
               cudaStream_t st) {
  const int64_t b_bytes = (int64_t)n * K * 2;
  if (b_bytes > (int64_t)RD_B_MAX || K % RD_KB != 0 || T >= (1ll << 31)) return RD_NOT_APPLICABLE;
  if (!mx_aligned(A, 16) || lda % 8 != 0 || !mx_aligned(B, 16)) return RD_NOT_APPLICABLE;
  if (q && (ldq % 16 != 0 || !mx_aligned(q, 16) || !mx_aligned(s, 2) || kb_off % 2 != 0)) return RD_NOT_APPLICABLE;
  CUtensorMap ta, tb;
  if (int e = mx_make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, (uint64_t)K, (uint64_t)T, (uint64_t)(lda * 2),
                              RD_KB, RD_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = mx_make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, (uint64_t)K, (uint64_t)n, (uint64_t)(K * 2),
                              RD_KB, (uint32_t)n, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  const int stages = rd_stages(b_bytes);
  const size_t smem = rd_smem(b_bytes, stages);
  const int nrb = (int)((T + RD_ROWS - 1) / RD_ROWS);
  const int grid = std::min(nrb, mxm_num_sms());
  auto go = [&](auto kern) -> int {
    cudaError_t e = mx_smem_attr((const void*)kern, smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "rowdot tma: set smem");
    kern<<<grid, 32 * (RD_CONS + 1), smem, st>>>(ta, tb, (int)T, (int)K, nrb, stages, post, round_once, (bf16*)out,
                                                  ldo, q, ldq, s, scols, kb_off, mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("rowdot tma");
  };
  if (q) return n == 16 ? go(k_rowdot_tma<16, true>) : (n == 32 ? go(k_rowdot_tma<32, true>) : go(k_rowdot_tma<64, true>));
  return n == 16 ? go(k_rowdot_tma<16, false>) : (n == 32 ? go(k_rowdot_tma<32, false>) : go(k_rowdot_tma<64, false>));
}

// part[chunk, k, j] = sum over the chunk's rows t of A[t, k] E[t, j]   (k < K, j < NJ)
// CTA = 64 columns k of one row chunk: warp 4 streams [64 rows x 64 k] tiles of A (128-byte swizzle)
// and the matching [64 rows x NJ] rows of E into a 5-stage ring with TMA; warps 0-3 each own 16
// columns and accumulate D[k x j] = A^T E with m16n8k16 MMAs whose operands come from ldmatrix.trans
// (A^T and E^T are the transposes of the stored tiles).  Rows past T read as zero.
constexpr int CD_ST = 4, CD_ROWS = 64, CD_COLS = 64;   // 4 stages: 4 CTAs per SM at n = 32, 5 at n = 16
__host__ __device__ constexpr int cd_stage(int NJ) { return CD_ROWS * CD_COLS * 2 + CD_ROWS * NJ * 2; }
__host__ __device__ constexpr size_t cd_smem(int NJ) { return 1024 + (size_t)CD_ST * cd_stage(NJ) + 2 * CD_ST * 8; }

template <int NJ>
__global__ void __launch_bounds__(160) k_coldot(const __grid_constant__ CUtensorMap tm_a,
                                                const __grid_constant__ CUtensorMap tm_e, int K, int rows_per_chunk,
                                                int T, float* __restrict__ part, int* err) {
  constexpr int STG = cd_stage(NJ), AT = CD_ROWS * CD_COLS * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + CD_ST * STG);
  uint64_t* empty = full + CD_ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = blockIdx.x * CD_COLS;
  const int r0 = blockIdx.y * rows_per_chunk, r1 = min(r0 + rows_per_chunk, T);
  const int nsteps = r1 > r0 ? (r1 - r0 + CD_ROWS - 1) / CD_ROWS : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < CD_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 4) {  // TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_e);
    }
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    for (int i = 0; i < nsteps; ++i) {
      if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) break;
      if (lane == 0) {
        uint8_t* dst = smem + stage * STG;
        mbar_arrive_expect_tx(&full[stage], STG);
        tma_load_2d(dst, &tm_a, &full[stage], kc, r0 + i * CD_ROWS);
        tma_load_2d(dst + AT, &tm_e, &full[stage], 0, r0 + i * CD_ROWS);
      }
      __syncwarp();
      ++issued;
      if (++stage == CD_ST) {
        stage = 0;
        phase ^= 1;
      }
    }
    for (int k = 0; k < CD_ST && k < issued; ++k) {  // leave no copy in flight
      const int i = issued - 1 - k;
      mbar_wait(&full[i % CD_ST], (uint32_t)((i / CD_ST) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3, mi = lane >> 3, lr = lane & 7;
  float acc[NJ / 8][4];
#pragma unroll
  for (int j = 0; j < NJ / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  // A^T fragment (m = k: 16 warp columns, kdim = 16 rows): matrix mi = (k half mi & 1, row half mi >> 1)
  // E^T as the B operand (kdim = rows, n = j): matrix mi = (row half mi & 1, j half mi >> 1)
  uint32_t o_a[4], o_e[4][NJ / 16];
#pragma unroll
  for (int s4 = 0; s4 < 4; ++s4) {
    o_a[s4] = swz<128>((uint32_t)(16 * s4 + (mi >> 1) * 8 + lr), (uint32_t)(2 * warp + (mi & 1)));
#pragma unroll
    for (int jp = 0; jp < NJ / 16; ++jp)
      o_e[s4][jp] = AT + swz<2 * NJ>((uint32_t)(16 * s4 + (mi & 1) * 8 + lr), (uint32_t)(2 * jp + (mi >> 1)));
  }
  const uint32_t s_ring = smem_u32(smem);
  int stage = 0;
  uint32_t phase = 0;
  for (int i = 0; i < nsteps; ++i) {
    if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
    const uint32_t sb = s_ring + (uint32_t)stage * STG;
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      uint32_t a[4];
      ldsm4t(a, sb + o_a[s4]);
#pragma unroll
      for (int jp = 0; jp < NJ / 16; ++jp) {
        uint32_t e[4];
        ldsm4t(e, sb + o_e[s4][jp]);
        mma16816(acc[2 * jp], a, e[0], e[1]);
        mma16816(acc[2 * jp + 1], a, e[2], e[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == CD_ST) {
      stage = 0;
      phase ^= 1;
    }
  }
  float* P = part + (int64_t)blockIdx.y * K * NJ;
  const int k = kc + 16 * warp + g;
#pragma unroll
  for (int jt = 0; jt < NJ / 8; ++jt) {
    const int j = 8 * jt + 2 * t;
    *reinterpret_cast<float2*>(P + (int64_t)k * NJ + j) = make_float2(acc[jt][0], acc[jt][1]);
    *reinterpret_cast<float2*>(P + (int64_t)(k + 8) * NJ + j) = make_float2(acc[jt][2], acc[jt][3]);
  }
}

// out = bf16(x + bf16(y + scale * xa B^T)) for x, y [T, N] bf16, xa [T, R] (row stride ldxa), B [N, R]:
// the residual add with the rank-R LoRA term of o_proj / out_proj computed in registers (reference
// _res_lora_kernel, scripts/mxfp8.py:266-282).  Warp = 16 rows x 64 columns: xa and B fragments from
// 4-byte loads, R/16 x 8 mma.sync, then the two roundings per element on the accumulator fragment.
template <int R>
__global__ void __launch_bounds__(128) k_res_lora(const bf16* __restrict__ x, const bf16* __restrict__ y,
                                                  const bf16* __restrict__ xa, int64_t ldxa,
                                                  const bf16* __restrict__ B, int T, int N, float scale,
                                                  bf16* __restrict__ out) {
  constexpr int KS = R / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t ra = (int64_t)blockIdx.x * 64 + warp * 16 + g, rb = ra + 8;
  const int c0 = blockIdx.y * 64;
  const bool va = ra < T, vb = rb < T;
  uint32_t a[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const bf16* pa = xa + ra * ldxa + 16 * kk + 2 * t;
    const bf16* pb = xa + rb * ldxa + 16 * kk + 2 * t;
    a[kk][0] = va ? ld32(pa) : 0u;
    a[kk][1] = vb ? ld32(pb) : 0u;
    a[kk][2] = va ? ld32(pa + 8) : 0u;
    a[kk][3] = vb ? ld32(pb + 8) : 0u;
  }
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    const bf16* pB = B + (int64_t)(c0 + 8 * i + g) * R + 2 * t;   // B operand: (k = j, n = column)
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) mma16816(acc[i], a[kk], ld32g(pB + 16 * kk), ld32g(pB + 16 * kk + 8));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = c0 + 8 * i + 2 * t;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = h ? rb : ra;
      if (!(h ? vb : va)) continue;
      const int64_t off = row * N + c;
      const float2 yv = up2(ld32g(y + off)), xv = up2(ld32g(x + off));
      const float2 tv = up2(rn2(make_float2(__fmaf_rn(scale, acc[i][2 * h], yv.x), __fmaf_rn(scale, acc[i][2 * h + 1], yv.y))));
      *reinterpret_cast<uint32_t*>(out + off) = rn2(make_float2(xv.x + tv.x, xv.y + tv.y));
    }
  }
}

// out[i] = scale * sum_{p < nparts} src[p * stride + i]   (fixed order); bf16 or fp32 output,
// optionally transposed: element i = (a, b) of an [A, B] matrix written at out[b * A + a].  With
// `round_out` the value is rounded as for the bf16 output (bf16(bf16(v) * post)) and stored as fp32.
__global__ void k_sum_parts(const float* __restrict__ src, int nparts, int64_t n, int64_t stride, float scale,
                            float post, float* __restrict__ out_f, bf16* __restrict__ out_h, int64_t tr_a,
                            int64_t tr_b, int round_out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    // partials added in order; eight loads are issued before their adds (latency, not order, changes)
    float v = 0.f;
    int p = 0;
    for (; p + 8 <= nparts; p += 8) {
      float x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) x[u] = __ldg(src + (int64_t)(p + u) * stride + i);
#pragma unroll
      for (int u = 0; u < 8; ++u) v += x[u];
    }
    for (; p < nparts; ++p) v += __ldg(src + (int64_t)p * stride + i);
    v *= scale;
    int64_t o = i;
    if (tr_a > 0) o = (i % tr_b) * tr_a + i / tr_b;
    if (out_h || round_out) {
      v = bf16_round_f(v);
      if (post != 1.0f) v = bf16_round_f(v * post);
    }
    if (out_h)
      out_h[o] = __float2bfloat16_rn(v);
    else
      out_f[o] = v;
  }
}

// The per-step bf16 forms of the six LoRA matrices (the reference's _MLP.forward casts,
// scripts/fused_mlp.py:272-276, and the transposed / scaled copies its backward makes, :282,311,331),
// one launch: out = S [2r, H] | bg [N, r] | bu [N, r] | ad [r, N] | bd [H, r] | bds [H, r] | bdT [r, H] |
// ST [H, 2r] with S = [Ag; Au], bds = bf16(bd * s_d).  Sources are fp32 (src_f32) or bf16, contiguous.
struct LoraSrc {
  const void* p[6];  // Ag, Au, Bg, Bu, Ad, Bd
};
// blockIdx.y = output segment (0 S, 1 bg, 2 bu, 3 ad, 4 bd, 5 bds, 6 bdT, 7 ST).  The six straight
// segments move four values per thread when r % 4 == 0 (every segment then starts on a 4-element
// boundary); the two transposes one value per thread, writes coalesced.
__global__ void k_lora_prep(LoraSrc src, int src_f32, int H, int N, int r, float s_d, bf16* __restrict__ out) {
  const int seg = blockIdx.y;
  const int64_t rH = (int64_t)r * H, nB = (int64_t)N * r, nD = (int64_t)H * r;
  const int64_t starts[9] = {0, 2 * rH, 2 * rH + nB, 2 * rH + 2 * nB, 2 * rH + 3 * nB, 2 * rH + 3 * nB + nD,
                             2 * rH + 3 * nB + 2 * nD, 2 * rH + 3 * nB + 3 * nD, 4 * rH + 3 * nB + 3 * nD};
  int64_t off = starts[0], len = starts[1];
#pragma unroll
  for (int k = 1; k < 8; ++k)
    if (seg == k) {
      off = starts[k];
      len = starts[k + 1] - starts[k];
    }
  auto ld = [&](int w, int64_t i) -> float {
    return src_f32 ? reinterpret_cast<const float*>(src.p[w])[i]
                   : __bfloat162float(reinterpret_cast<const bf16*>(src.p[w])[i]);
  };
  auto value = [&](int64_t i) -> float {   // straight segments
    switch (seg) {
      case 0: return i < rH ? ld(0, i) : ld(1, i - rH);
      case 1: return ld(2, i);
      case 2: return ld(3, i);
      case 3: return ld(4, i);
      case 4: return ld(5, i);
      default: return bf16_round_f(bf16_round_f(ld(5, i)) * s_d);
    }
  };
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (int64_t)gridDim.x * blockDim.x;
  bf16* o = out + off;
  if (seg < 6 && (r & 3) == 0) {
    for (int64_t i = 4 * tid; i < len; i += 4 * nth) {
      uint2 w;
      w.x = pack_bf16x2(value(i), value(i + 1));
      w.y = pack_bf16x2(value(i + 2), value(i + 3));
      *reinterpret_cast<uint2*>(o + i) = w;
    }
  } else if (seg < 6) {
    for (int64_t i = tid; i < len; i += nth) o[i] = __float2bfloat16_rn(value(i));
  } else if (seg == 6) {   // bdT [r, H]: (j, h) <- Bd [H, r] (h, j)
    for (int64_t e = tid; e < len; e += nth) {
      const int64_t j = e / H, h = e % H;
      o[e] = __float2bfloat16_rn(ld(5, h * r + j));
    }
  } else {                 // ST [H, 2r]: (h, j) <- S [2r, H] (j, h)
    for (int64_t e = tid; e < len; e += nth) {
      const int64_t h = e / (2 * r), j = e % (2 * r);
      o[e] = __float2bfloat16_rn(j < r ? ld(0, j * H + h) : ld(1, (j - r) * H + h));
    }
  }
}

// Up to three independent fp32 partial sums in one launch (blockIdx.y = job), 4 floats per thread:
// out[i] = scale * sum_{p < nparts} src[p * stride + i], the same fixed order as k_sum_parts.
struct SumJob {
  const float4* src;
  float4* out;
  float scale;
};
struct SumJobs {
  SumJob j[3];
};
MX_DEV void sum_parts4_body(const SumJob& jb, int nparts, int64_t n4, int64_t stride4) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    // partials in order, 16 loads in flight: even parts into v, odd parts into w, then v + w
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f), w = v;
    const float4* p = jb.src + i;
    int k = 0;
    for (; k + 16 <= nparts; k += 16) {
      float4 x[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) x[u] = __ldg(p + (int64_t)(k + u) * stride4);
#pragma unroll
      for (int u = 0; u < 16; u += 2) {
        v.x += x[u].x; v.y += x[u].y; v.z += x[u].z; v.w += x[u].w;
        w.x += x[u + 1].x; w.y += x[u + 1].y; w.z += x[u + 1].z; w.w += x[u + 1].w;
      }
    }
    for (; k < nparts; ++k) {
      const float4 x = __ldg(p + (int64_t)k * stride4);
      if (k & 1) {
        w.x += x.x; w.y += x.y; w.z += x.z; w.w += x.w;
      } else {
        v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
      }
    }
    jb.out[i] = make_float4((v.x + w.x) * jb.scale, (v.y + w.y) * jb.scale, (v.z + w.z) * jb.scale,
                            (v.w + w.w) * jb.scale);
  }
}

// dxa partials [slots, T, 3R] -> dxa bf16 [T, 2R] (gate part x s_g, up part x s_u) and xS_down bf16 [T, R].
// Row block sbi (rows sb * sbi ..) was worked on by CTAs c_lo .. c_hi of the backward epilogue, whose
// partials sit in slots 0 .. c_hi - c_lo; they are added in slot order.  Four values per thread.
template <int R>
MX_DEV void reduce_dxa_body(const float* __restrict__ src, int sb, int nt, int per, int T, float s_g, float s_u,
                            bf16* __restrict__ dxa, bf16* __restrict__ xsd) {
  constexpr int Q = 3 * R / 4;   // float4s per row
  const int64_t n = (int64_t)T * Q;
  const int64_t stride = (int64_t)T * Q;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / Q;
    const int c = 4 * (int)(i - row * Q);
    const int sbi = (int)(row / sb);
    const int nparts = ((sbi + 1) * nt - 1) / per - (sbi * nt) / per + 1;
    float4 v = __ldg(s4 + i);
    for (int p = 1; p < nparts; ++p) {
      const float4 x = __ldg(s4 + p * stride + i);
      v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
    }
    const float sc = c < R ? s_g : (c < 2 * R ? s_u : 1.f);
    uint2 o;
    o.x = pack_bf16x2(v.x * sc, v.y * sc);
    o.y = pack_bf16x2(v.z * sc, v.w * sc);
    if (c < 2 * R)
      *reinterpret_cast<uint2*>(dxa + row * 2 * R + c) = o;
    else
      *reinterpret_cast<uint2*>(xsd + row * R + c - 2 * R) = o;
  }
}

// The backward's fixed-order reductions in one launch: grid rows 0-2 sum the column-product partials
// (dB_gate, dB_up, dA_down), row 3 the per-row partials into dxa / xS_down.
template <int R>
__global__ void __launch_bounds__(256) k_bwd_reduce(SumJobs jobs, int nparts, int64_t n4, const float* __restrict__ dsrc,
                                                    int sb, int nt, int per, int T, float s_g, float s_u,
                                                    bf16* __restrict__ dxa, bf16* __restrict__ xsd) {
  if (blockIdx.y < 3) {
    const SumJob jb = blockIdx.y == 0 ? jobs.j[0] : (blockIdx.y == 1 ? jobs.j[1] : jobs.j[2]);   // by value
    sum_parts4_body(jb, nparts, n4, n4);
  } else
    reduce_dxa_body<R>(dsrc, sb, nt, per, T, s_g, s_u, dxa, xsd);
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
  // one CTA per SM: the fewest column groups that still fill every SM twice
  const int64_t nrb = ((T + 127) / 128 * 128 + FWD_ROWS - 1) / FWD_ROWS;
  const int nt = (int)(N / FWD_BN);
  int cs = nt;
  for (int d = 1; d <= nt; ++d)
    if (nt % d == 0 && nrb * d >= 2 * (int64_t)mxm_num_sms()) {
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
  const int nt = (int)(N / FWD_BN);
  MX_CHECK_ARG(col_groups >= 1 && nt % col_groups == 0, "mxm_mlp_fwd_epilogue: col_groups must divide N/64");
  MX_CHECK_ARG(col_groups == 1 || xsd_part, "mxm_mlp_fwd_epilogue: partial buffer needed for col_groups > 1");
  MX_CHECK_ARG(mx_aligned(gu, 16) && mx_aligned(bg, 16) && mx_aligned(bu, 16) && mx_aligned(ad, 16),
               "mxm_mlp_fwd_epilogue: gu / bg / bu / ad must be 16-byte aligned");
  CUtensorMap tm, tbg, tbu, tad;
  if (int e = mx_make_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gu, (uint64_t)(2 * N), (uint64_t)T,
                              (uint64_t)(4 * N), FWD_BN, FWD_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = mx_make_tmap_2d(&tbg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bg, (uint64_t)r, (uint64_t)N,
                              (uint64_t)(2 * r), r, FWD_BN, r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tbu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bu, (uint64_t)r, (uint64_t)N,
                              (uint64_t)(2 * r), r, FWD_BN, r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tad, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ad, (uint64_t)N, (uint64_t)r,
                              (uint64_t)(2 * N), FWD_BN, r, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  const int Tpad = (int)((T + 127) / 128 * 128);  // rows of the blocked scale layout: every one gets its scales
  dim3 grid((unsigned)((Tpad + FWD_ROWS - 1) / FWD_ROWS), (unsigned)col_groups);
  cudaStream_t st = (cudaStream_t)stream;
  const int tpg = nt / col_groups;
  bf16* direct = col_groups == 1 ? (bf16*)xsd : nullptr;
  const size_t smem = fwd_smem(r);
  auto go = [&](auto kern) -> int {
    cudaError_t e = mx_smem_attr((const void*)kern, smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "mlp fwd epilogue: set smem");
    kern<<<grid, FWD_THREADS, smem, st>>>(tm, tbg, tbu, tad, (const bf16*)xs, (uint8_t*)qh, (uint8_t*)sh,
                                          (float*)xsd_part, direct, (int)T, Tpad, (int)N, s_g, s_u, tpg,
                                          qh != nullptr, mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("mlp fwd epilogue");
  };
  if (int e = (r == 16 ? go(k_mlp_fwd<16>) : go(k_mlp_fwd<32>))) return e;
  if (col_groups > 1) {
    const int64_t n = T * r;
    k_sum_parts<<<grid_for(n, 256), 256, 0, st>>>((const float*)xsd_part, col_groups, n, n, 1.0f, 1.0f, nullptr,
                                                  (bf16*)xsd, 0, 0, 0);
    mx_note_launch();
    if (int e = mx_launch_status("mlp fwd xsd sum")) return e;
  }
  return MXM_OK;
}

// Backward partition.  Work items are (row block of SB = 16 x consumer-warps rows, 32-column tile), the
// column tile fastest; each CTA (one per SM) takes a contiguous run of `per` items, so every SM gets the
// same number of tiles whatever T is, and a row block is shared by at most ceil(nt / per) + 1 CTAs, each
// writing its per-row sums into its own slot of dxa_part.  The reference's _bwd_grid
// (scripts/fused_mlp.py:218-232) splits the columns into groups for the same reason: enough CTAs for the
// GPU, at the cost of [T, 3r] fp32 partials per extra group.
namespace {
struct BwdPlan {
  int sb, nt, nsb, items, per, grid, slots;
};
BwdPlan bwd_plan(int64_t T, int64_t N, int r) {
  BwdPlan p;
  p.sb = r == 16 ? BT_ROWS : bwd_rows(32);
  const int64_t tpad = (T + 127) / 128 * 128;
  p.nsb = (int)((tpad + p.sb - 1) / p.sb);
  p.nt = (int)(N / BWD_BN);
  p.items = p.nsb * p.nt;
  const int nsm = mxm_num_sms();
  p.per = (p.items + nsm - 1) / nsm;
  p.grid = (p.items + p.per - 1) / p.per;
  p.slots = 1;
  for (int b = 0; b < p.nsb; ++b)
    p.slots = std::max(p.slots, ((b + 1) * p.nt - 1) / p.per - (b * p.nt) / p.per + 1);
  return p;
}
}  // namespace

extern "C" int mxm_mlp_bwd_partitions(int64_t T, int64_t N, int r, int* super_block, int* col_groups) {
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32) && super_block &&
                   col_groups,
               "mxm_mlp_bwd_partitions: bad args");
  const BwdPlan p = bwd_plan(T, N, r);
  *super_block = p.sb;
  *col_groups = p.slots;
  return MXM_OK;
}

extern "C" int mxm_mlp_bwd_epilogue(const void* gu, const void* xs, const void* dhm, const void* dxd, const void* bg,
                                    const void* bu, const void* ad, int64_t T, int64_t N, int r, float s_g, float s_u,
                                    int gu_lora, void* q, void* s, void* dxa_part, void* dbg_part, void* dbu_part,
                                    void* dad_part, int super_block, int col_groups, void* stream) {
  MX_CHECK_ARG(gu && xs && dhm && dxd && bg && bu && ad && dxa_part && dbg_part && dbu_part && dad_part,
               "mxm_mlp_bwd_epilogue: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32),
               "mxm_mlp_bwd_epilogue: need T >= 1, N %% 128 == 0, r in {16, 32}");
  MX_CHECK_ARG((q == nullptr) == (s == nullptr), "mxm_mlp_bwd_epilogue: q and s go together");
  MX_CHECK_ARG(gu_lora == 0 || gu_lora == 1, "mxm_mlp_bwd_epilogue: gu_lora is 0 or 1");
  MX_CHECK_ARG(gu_lora == 0 || r == 16, "mxm_mlp_bwd_epilogue: gu with the LoRA terms added is a rank-16 layout");
  const BwdPlan p = bwd_plan(T, N, r);
  MX_CHECK_ARG(col_groups >= p.slots && super_block == p.sb,
               "mxm_mlp_bwd_epilogue: bad partition (%d, %d): use mxm_mlp_bwd_partitions", super_block, col_groups);
  MX_CHECK_ARG(mx_aligned(gu, 16) && mx_aligned(dhm, 16) && mx_aligned(bg, 16) && mx_aligned(bu, 16) &&
                   mx_aligned(ad, 16),
               "mxm_mlp_bwd_epilogue: gu / dhm / bg / bu / ad must be 16-byte aligned");
  CUtensorMap tgu, tdh, tbg, tbu, tad;
  if (int e = mx_make_tmap_2d(&tgu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gu, (uint64_t)(2 * N), (uint64_t)T,
                              (uint64_t)(4 * N), BWD_BN, super_block, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tdh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dhm, (uint64_t)N, (uint64_t)T,
                              (uint64_t)(2 * N), BWD_BN, super_block, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tbg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bg, (uint64_t)r, (uint64_t)N,
                              (uint64_t)(2 * r), r, BWD_BN, r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tbu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bu, (uint64_t)r, (uint64_t)N,
                              (uint64_t)(2 * r), r, BWD_BN, r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tad, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ad, (uint64_t)N, (uint64_t)r,
                              (uint64_t)(2 * N), BWD_BN, r, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  CUtensorMap txs, tdxd;
  // xs: r = 16 reads xa_gate and xa_up as two [rows x 16] boxes (32-byte rows), r = 32 as one [rows x 64] box
  if (int e = mx_make_tmap_2d(&txs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs, (uint64_t)(2 * r), (uint64_t)T,
                              (uint64_t)(4 * r), r == 16 ? r : 2 * r, super_block,
                              r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = mx_make_tmap_2d(&tdxd, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dxd, (uint64_t)r, (uint64_t)T,
                              (uint64_t)(2 * r), r, super_block, r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  const int64_t tpad = (T + 127) / 128 * 128;
  cudaStream_t st = (cudaStream_t)stream;
  if (r == 16) {
    // codes of [dg | du] as a [T][2][N] byte array: one [32 rows][2][16] box per warp and tile
    CUtensorMap tq = tgu;   // unused when q is null
    if (q) {
      MX_CHECK_ARG(mx_aligned(q, 16), "mxm_mlp_bwd_epilogue: q must be 16-byte aligned");
      const uint64_t dims[3] = {(uint64_t)N, 2, (uint64_t)T}, strides[2] = {(uint64_t)N, (uint64_t)(2 * N)};
      const uint32_t box[3] = {16, 2, 32};
      if (int e = mx_make_tmap_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_NONE))
        return e;
    }
    auto go = [&](auto kern) -> int {
      cudaError_t e = mx_smem_attr((const void*)kern, BT_SMEM);
      if (e != cudaSuccess) return mx_cuda_status(e, "mlp bwd epilogue: set smem");
      kern<<<p.grid, BT_THREADS, BT_SMEM, st>>>(tgu, tdh, tbg, tbu, tad, txs, tdxd, tq, (uint8_t*)s, (float*)dxa_part,
                                                (float*)dbg_part, (float*)dbu_part, (float*)dad_part, (int)T,
                                                (int)tpad, (int)N, s_g, s_u, p.per, q != nullptr, mx_dev_error_ptr());
      mx_note_launch();
      return mx_launch_status("mlp bwd epilogue");
    };
    return gu_lora ? go(k_mlp_bwd_tc<true>) : go(k_mlp_bwd_tc<false>);
  }
  const size_t smem = bwd_smem(r);
  cudaError_t e = mx_smem_attr((const void*)k_mlp_bwd<32>, smem);
  if (e != cudaSuccess) return mx_cuda_status(e, "mlp bwd epilogue: set smem");
  k_mlp_bwd<32><<<p.grid, 32 * (bwd_cons(32) + 1), smem, st>>>(
      tgu, tdh, tbg, tbu, tad, txs, tdxd, (uint8_t*)q, (uint8_t*)s, (float*)dxa_part, (float*)dbg_part,
      (float*)dbu_part, (float*)dad_part, (int)T, (int)tpad, (int)N, s_g, s_u, p.per, q != nullptr,
      mx_dev_error_ptr());
  mx_note_launch();
  return mx_launch_status("mlp bwd epilogue");
}

extern "C" int mxm_mlp_bwd_reduce(const void* dxa_part, const void* dbg_part, const void* dbu_part,
                                  const void* dad_part, int64_t T, int64_t N, int r, float s_g, float s_u,
                                  int super_block, int col_groups, void* dxa, void* xsd, void* dBg, void* dBu,
                                  void* dAd, void* stream) {
  MX_CHECK_ARG(dxa_part && dbg_part && dbu_part && dad_part && dxa && xsd && dBg && dBu && dAd,
               "mxm_mlp_bwd_reduce: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32),
               "mxm_mlp_bwd_reduce: need T >= 1, N %% 128 == 0, r in {16, 32}");
  const BwdPlan p = bwd_plan(T, N, r);
  MX_CHECK_ARG(col_groups >= p.slots && super_block == p.sb,
               "mxm_mlp_bwd_reduce: bad partition (%d, %d): use mxm_mlp_bwd_partitions", super_block, col_groups);
  const int nsb = p.nsb;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nd = T * 3 * r / 4;
  const int64_t nb4 = N * r / 4;  // N % 128 == 0
  SumJobs jobs;
  jobs.j[0] = {(const float4*)dbg_part, (float4*)dBg, s_g};
  jobs.j[1] = {(const float4*)dbu_part, (float4*)dBu, s_u};
  jobs.j[2] = {(const float4*)dad_part, (float4*)dAd, 1.f};
  const int gx = std::max(grid_for(nd, 256), (int)std::min<int64_t>((nb4 + 255) / 256, (int64_t)mxm_num_sms() * 8));
  if (r == 16)
    k_bwd_reduce<16><<<dim3((unsigned)gx, 4u), 256, 0, st>>>(jobs, nsb, nb4, (const float*)dxa_part, p.sb, p.nt, p.per,
                                                             (int)T, s_g, s_u, (bf16*)dxa, (bf16*)xsd);
  else
    k_bwd_reduce<32><<<dim3((unsigned)gx, 4u), 256, 0, st>>>(jobs, nsb, nb4, (const float*)dxa_part, p.sb, p.nt, p.per,
                                                             (int)T, s_g, s_u, (bf16*)dxa, (bf16*)xsd);
  mx_note_launch();
  return mx_launch_status("mlp bwd reduce");
}

extern "C" int mxm_rowdot(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post,
                          void* out, int64_t ldo, void* stream) {
  MX_CHECK_ARG(A && B && out, "mxm_rowdot: null pointer");
  MX_CHECK_ARG(T >= 1 && K >= 128 && K % 128 == 0 && (n == 16 || n == 32 || n == 64) && lda % 8 == 0 && ldo % 2 == 0,
               "mxm_rowdot: need K %% 128 == 0, n in {16, 32, 64}, lda %% 8 == 0");
  MX_CHECK_ARG(mx_aligned(A, 16) && mx_aligned(B, 16) && mx_aligned(out, 4), "mxm_rowdot: alignment");
  cudaStream_t st = (cudaStream_t)stream;
  const int e = rowdot_tma(A, lda, B, T, K, n, post, 0, out, ldo, nullptr, 0, nullptr, K, 0, st);
  if (e != RD_NOT_APPLICABLE) return e;
  const unsigned grid = (unsigned)((T + 15) / 16);
  auto go = [&](auto kern) {
    kern<<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)B, (int)T, (int)K, post, 0, (bf16*)out, ldo, nullptr,
                               0, nullptr, K, 0);
  };
  if (n == 16)
    go(k_rowdot<16, false>);
  else if (n == 32)
    go(k_rowdot<32, false>);
  else
    go(k_rowdot<64, false>);
  mx_note_launch();
  return mx_launch_status("rowdot");
}

extern "C" int mxm_lora_prep(const void* Ag, const void* Au, const void* Bg, const void* Bu, const void* Ad,
                             const void* Bd, int src_fp32, int64_t H, int64_t N, int r, float s_d, void* out,
                             void* stream) {
  MX_CHECK_ARG(Ag && Au && Bg && Bu && Ad && Bd && out, "mxm_lora_prep: null pointer");
  MX_CHECK_ARG(H >= 1 && N >= 1 && r >= 1 && r <= 256 && H < (1ll << 31) && N < (1ll << 31),
               "mxm_lora_prep: bad shape");
  LoraSrc src{{Ag, Au, Bg, Bu, Ad, Bd}};
  // grid.y = the eight output segments; grid.x sized for the largest one (four values per thread)
  const int64_t largest = std::max<int64_t>(2 * (int64_t)r * H, (int64_t)N * r);
  const int gx = (int)std::min<int64_t>((largest / 4 + 255) / 256 + 1, (int64_t)mxm_num_sms() * 4);
  k_lora_prep<<<dim3((unsigned)gx, 8u), 256, 0, (cudaStream_t)stream>>>(src, src_fp32, (int)H, (int)N, r, s_d,
                                                                         (bf16*)out);
  mx_note_launch();
  return mx_launch_status("lora prep");
}

// The reference's lora_bwd in its LoRA mode (scripts/mxfp8.py:219-263) for one branch:
//   dxa_out [T, r] = bf16(scale * dy Bt^T)  (dy [T, N], Bt = B^T [r, N])      -- one rounding
//   dB_out  [N, r] = scale * dy^T xa        (fp32, fixed-order partial sums)
//   q / s (optional): row-wise MXFP8 of dy into columns col_tile_off*128 .. of a [ceil128(T), s_cols] operand,
//   from the same read of dy as dxa.
extern "C" int mxm_lora_bwd(const void* dy, int64_t ldy, int64_t T, int64_t N, const void* xa, int64_t ldxa,
                            const void* Bt, int r, float scale, void* q, int64_t ldq, void* s, int64_t s_cols,
                            int64_t col_tile_off, void* dxa_out, int64_t ld_dxa, void* dB_out, void* part,
                            int rows_per_chunk, int chunks, void* stream) {
  MX_CHECK_ARG(dy && xa && Bt && dxa_out && dB_out && part, "mxm_lora_bwd: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && N >= 128 && N % 128 == 0 && (r == 16 || r == 32 || r == 64) &&
                   ldy % 8 == 0 && ldxa % 8 == 0 && ld_dxa % 2 == 0,
               "mxm_lora_bwd: need N %% 128 == 0, r in {16, 32, 64}, ldy and ldxa multiples of 8");
  MX_CHECK_ARG(mx_aligned(dy, 16) && mx_aligned(xa, 16) && mx_aligned(Bt, 16) && mx_aligned(dxa_out, 4),
               "mxm_lora_bwd: alignment");
  MX_CHECK_ARG((q == nullptr) == (s == nullptr), "mxm_lora_bwd: q and s go together");
  if (q) {
    MX_CHECK_ARG(s_cols % 128 == 0 && col_tile_off >= 0 && col_tile_off * 128 + N <= s_cols && ldq >= s_cols &&
                     ldq % 8 == 0 && mx_aligned(q, 8),
                 "mxm_lora_bwd: quantized columns outside the %lld-column operand", (long long)s_cols);
  }
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = q ? (unsigned)((T + 127) / 128 * 8) : (unsigned)((T + 15) / 16);
  uint8_t* qc = q ? (uint8_t*)q + col_tile_off * 128 : nullptr;
  const int et = rowdot_tma(dy, ldy, Bt, T, N, r, scale, 1, dxa_out, ld_dxa, qc, ldq, (uint8_t*)s, s_cols,
                            (int)(col_tile_off * 4), st);
  if (et != RD_NOT_APPLICABLE && et != MXM_OK) return et;
  if (et == RD_NOT_APPLICABLE) {
    auto go = [&](auto kern) {
      kern<<<grid, 128, 0, st>>>((const bf16*)dy, ldy, (const bf16*)Bt, (int)T, (int)N, scale, 1, (bf16*)dxa_out,
                                 ld_dxa, qc, ldq, (uint8_t*)s, s_cols, (int)(col_tile_off * 4));
    };
    if (q) {
      if (r == 16) go(k_rowdot<16, true>);
      else if (r == 32) go(k_rowdot<32, true>);
      else go(k_rowdot<64, true>);
    } else {
      if (r == 16) go(k_rowdot<16, false>);
      else if (r == 32) go(k_rowdot<32, false>);
      else go(k_rowdot<64, false>);
    }
    mx_note_launch();
    if (int e = mx_launch_status("lora bwd rowdot")) return e;
  }
  // dB = scale * dy^T xa: the coldot with an fp32, unrounded result
  MX_CHECK_ARG(rows_per_chunk % CD_ROWS == 0 && rows_per_chunk > 0 && (int64_t)rows_per_chunk * chunks >= T,
               "mxm_lora_bwd: bad chunking");
  CUtensorMap ta, te;
  if (int e = mx_make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dy, (uint64_t)N, (uint64_t)T, (uint64_t)(ldy * 2),
                              CD_COLS, CD_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = mx_make_tmap_2d(&te, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xa, (uint64_t)r, (uint64_t)T,
                              (uint64_t)(ldxa * 2), (uint32_t)r, CD_ROWS,
                              r == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                      : (r == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)))
    return e;
  dim3 cgrid((unsigned)(N / CD_COLS), (unsigned)chunks);
  auto goc = [&](auto kern, int nj) -> int {
    const size_t smem = cd_smem(nj);
    cudaError_t e = mx_smem_attr((const void*)kern, smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "lora bwd: set smem");
    kern<<<cgrid, 160, smem, st>>>(ta, te, (int)N, rows_per_chunk, (int)T, (float*)part, mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("lora bwd coldot");
  };
  if (int e = r == 16 ? goc(k_coldot<16>, 16) : (r == 32 ? goc(k_coldot<32>, 32) : goc(k_coldot<64>, 64))) return e;
  const int64_t nn = N * r;
  k_sum_parts<<<grid_for(nn, 256), 256, 0, st>>>((const float*)part, chunks, nn, nn, scale, 1.f, (float*)dB_out,
                                                 nullptr, 0, 0, 0);
  mx_note_launch();
  return mx_launch_status("lora bwd sum");
}

// The backward of a group of MX linears that share one input (q|k|v, qkv|z, o_proj alone), one branch after
// another on the caller's stream: each branch's dy is read once by the fused rowdot (its MXFP8 codes into
// columns of the group's K-concatenated operand, and for a LoRA branch d(xa) = bf16(scale dy B)), then a
// LoRA branch's dB = scale dy^T xa by the coldot.  The branches reuse one partial-sum buffer: stream order
// finishes a branch's reduction before the next branch's coldot writes it.
extern "C" int mxm_group_lora_bwd(int64_t T, int nb, const mxm_group_branch* br, void* q, int64_t ldq, void* s,
                                  int64_t s_cols, void* part, int64_t part_bytes, void* stream) {
  MX_CHECK_ARG(br && nb >= 1 && T >= 1 && T < (1ll << 31), "mxm_group_lora_bwd: need T >= 1 and branches");
  MX_CHECK_ARG((q == nullptr) == (s == nullptr), "mxm_group_lora_bwd: q and s go together");
  int64_t cols = 0;
  for (int i = 0; i < nb; ++i) {   // validate every branch before the first launch
    const mxm_group_branch& b = br[i];
    MX_CHECK_ARG(b.dy && b.N >= 128 && b.N % 128 == 0, "mxm_group_lora_bwd: branch %d needs dy with N %% 128 == 0", i);
    if (b.xa) {
      if (!(b.r == 16 || b.r == 32 || b.r == 64)) {
        mx_set_last_error("mxm_group_lora_bwd: branch %d has LoRA rank %d (the kernels take 16, 32, 64)", i, b.r);
        return MXM_ERR_UNSUPPORTED;
      }
      MX_CHECK_ARG(b.Bt && b.dxa_out && b.dB_out, "mxm_group_lora_bwd: branch %d: null LoRA pointer", i);
      int rpc = 0, nch = 0;
      if (int e = mxm_coldot_chunks(T, b.N, &rpc, &nch)) return e;
      MX_CHECK_ARG((int64_t)nch * b.N * b.r * 4 <= part_bytes,
                   "mxm_group_lora_bwd: branch %d needs %lld bytes of partials, %lld given", i,
                   (long long)nch * b.N * b.r * 4, (long long)part_bytes);
    } else {
      MX_CHECK_ARG(q != nullptr, "mxm_group_lora_bwd: branch %d has neither a LoRA branch nor a quantization", i);
    }
    cols += b.N;
  }
  MX_CHECK_ARG(q == nullptr || cols <= s_cols, "mxm_group_lora_bwd: branches span %lld columns, operand has %lld",
               (long long)cols, (long long)s_cols);
  int64_t tile = 0;
  for (int i = 0; i < nb; ++i) {
    const mxm_group_branch& b = br[i];
    int e;
    if (b.xa) {
      int rpc = 0, nch = 0;
      mxm_coldot_chunks(T, b.N, &rpc, &nch);
      e = mxm_lora_bwd(b.dy, b.ldy, T, b.N, b.xa, b.ldxa, b.Bt, b.r, b.scale, q, ldq, s, s_cols, tile, b.dxa_out,
                       b.ld_dxa, b.dB_out, part, rpc, nch, stream);
    } else {
      e = mxm_quant_rows_into(b.dy, T, b.N, b.ldy, q, ldq, s, s_cols, tile, stream);
    }
    if (e) return e;
    tile += b.N / 128;
  }
  return MXM_OK;
}

// out = bf16(x + bf16(y + scale * xa B^T)), x / y / out [T, N] bf16 contiguous, xa [T, r] (row stride ldxa),
// B [N, r] contiguous (reference res_lora, scripts/mxfp8.py:285-296).
extern "C" int mxm_res_lora(const void* x, const void* y, const void* xa, int64_t ldxa, const void* B, int64_t T,
                            int64_t N, int r, float scale, void* out, void* stream) {
  MX_CHECK_ARG(x && y && xa && B && out, "mxm_res_lora: null pointer");
  MX_CHECK_ARG(T >= 1 && T * N < (1ll << 31) && N % 64 == 0 && (r == 16 || r == 32 || r == 64) && ldxa % 2 == 0,
               "mxm_res_lora: need N %% 64 == 0, r in {16, 32, 64}");
  MX_CHECK_ARG(mx_aligned(x, 4) && mx_aligned(y, 4) && mx_aligned(out, 4) && mx_aligned(xa, 4) && mx_aligned(B, 4),
               "mxm_res_lora: alignment");
  dim3 grid((unsigned)((T + 63) / 64), (unsigned)(N / 64));
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto kern) {
    kern<<<grid, 128, 0, st>>>((const bf16*)x, (const bf16*)y, (const bf16*)xa, ldxa, (const bf16*)B, (int)T, (int)N,
                               scale, (bf16*)out);
  };
  if (r == 16) go(k_res_lora<16>);
  else if (r == 32) go(k_res_lora<32>);
  else go(k_res_lora<64>);
  mx_note_launch();
  return mx_launch_status("res lora");
}

extern "C" int mxm_rowdot_quant(const void* A, int64_t lda, const void* B, int64_t T, int64_t K, int n, float post,
                                void* out, int64_t ldo, void* q, int64_t ldq, void* s, void* stream) {
  MX_CHECK_ARG(A && B && out && q && s, "mxm_rowdot_quant: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && K >= 128 && K % 128 == 0 && (n == 16 || n == 32 || n == 64) &&
                   lda % 8 == 0 && ldo % 2 == 0 && ldq >= K && ldq % 8 == 0,
               "mxm_rowdot_quant: need K %% 128 == 0, n in {16, 32, 64}, lda %% 8 == 0, ldq >= K, ldq %% 8 == 0");
  MX_CHECK_ARG(mx_aligned(A, 16) && mx_aligned(B, 16) && mx_aligned(out, 4) && mx_aligned(q, 8),
               "mxm_rowdot_quant: alignment");
  cudaStream_t st = (cudaStream_t)stream;
  const int e = rowdot_tma(A, lda, B, T, K, n, post, 0, out, ldo, (uint8_t*)q, ldq, (uint8_t*)s, K, 0, st);
  if (e != RD_NOT_APPLICABLE) return e;
  const unsigned grid = (unsigned)((T + 127) / 128 * 8);  // 16-row CTAs over the padded rows
  auto go = [&](auto kern) {
    kern<<<grid, 128, 0, st>>>((const bf16*)A, lda, (const bf16*)B, (int)T, (int)K, post, 0, (bf16*)out, ldo,
                               (uint8_t*)q, ldq, (uint8_t*)s, K, 0);
  };
  if (n == 16)
    go(k_rowdot<16, true>);
  else if (n == 32)
    go(k_rowdot<32, true>);
  else
    go(k_rowdot<64, true>);
  mx_note_launch();
  return mx_launch_status("rowdot quant");
}

extern "C" int mxm_coldot_chunks(int64_t T, int64_t K, int* rows_per_chunk, int* chunks) {
  MX_CHECK_ARG(T >= 1 && K >= 64 && rows_per_chunk && chunks, "mxm_coldot_chunks: bad args");
  // one wave of four CTAs per SM (the n = 32 occupancy): (K / 64) column blocks x as many row chunks of
  // a multiple of 64 rows as fit in it, so no partial second wave
  const int64_t ctas_k = (K + CD_COLS - 1) / CD_COLS;
  const int64_t want = 4 * (int64_t)mxm_num_sms();
  const int64_t nch = std::max<int64_t>(1, want / ctas_k);
  int64_t rpc = (T + nch - 1) / nch;
  rpc = (rpc + CD_ROWS - 1) / CD_ROWS * CD_ROWS;
  if (rpc < 4 * CD_ROWS) rpc = 4 * CD_ROWS;
  *rows_per_chunk = (int)rpc;
  *chunks = (int)((T + rpc - 1) / rpc);
  return MXM_OK;
}

// out = bf16( bf16(sum_t A[t,k] E[t,j]) * post ), written [K, n] or transposed [n, K], as bf16 or (out_fp32)
// as the same values in fp32.
extern "C" int mxm_coldot(const void* A, int64_t lda, const void* E, int64_t lde, int64_t T, int64_t K, int n,
                          float post, int transpose_out, void* part, int rows_per_chunk, int chunks, void* out,
                          int out_fp32, void* stream) {
  MX_CHECK_ARG(A && E && part && out, "mxm_coldot: null pointer");
  MX_CHECK_ARG(T >= 1 && T < (1ll << 31) && K % 64 == 0 && (n == 16 || n == 32 || n == 64) &&
                   rows_per_chunk % CD_ROWS == 0 && rows_per_chunk > 0 && (int64_t)rows_per_chunk * chunks >= T,
               "mxm_coldot: bad shape or chunking (rows per chunk must be a multiple of 64)");
  MX_CHECK_ARG(lda % 8 == 0 && lde % 8 == 0 && mx_aligned(A, 16) && mx_aligned(E, 16),
               "mxm_coldot: A and E need 16-byte aligned rows (strides %% 8 == 0)");
  CUtensorMap ta, te;
  if (int e = mx_make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, (uint64_t)K, (uint64_t)T,
                              (uint64_t)(lda * 2), CD_COLS, CD_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = mx_make_tmap_2d(&te, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, E, (uint64_t)n, (uint64_t)T,
                              (uint64_t)(lde * 2), (uint32_t)n, CD_ROWS,
                              n == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                      : (n == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)))
    return e;
  dim3 grid((unsigned)(K / CD_COLS), (unsigned)chunks);
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto kern, int nj) -> int {
    const size_t smem = cd_smem(nj);
    cudaError_t e = mx_smem_attr((const void*)kern, smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "coldot: set smem");
    kern<<<grid, 160, smem, st>>>(ta, te, (int)K, rows_per_chunk, (int)T, (float*)part, mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("coldot");
  };
  int e = n == 16 ? go(k_coldot<16>, 16) : (n == 32 ? go(k_coldot<32>, 32) : go(k_coldot<64>, 64));
  if (e) return e;
  const int64_t nn = K * n;
  k_sum_parts<<<grid_for(nn, 256), 256, 0, st>>>((const float*)part, chunks, nn, nn, 1.f, post,
                                                 out_fp32 ? (float*)out : nullptr, out_fp32 ? nullptr : (bf16*)out,
                                                 transpose_out ? K : 0, transpose_out ? n : 0, out_fp32 ? 1 : 0);
  mx_note_launch();
  return mx_launch_status("coldot sum");
}

// ================================================================================================ no-alloc
// An allocation-free variant of mxm_coldot for callers that cannot allocate device memory: code that
// runs inside a custom device allocator (a call back into the allocator would re-enter it), and
// services that reserve their whole memory budget up front and may not grow it afterwards.  Its
// partial sums live in one fixed array in device memory, allocated when the library is loaded and
// held by every GPU that loads the library until the process exits.
#define MXM_NOALLOC_SCRATCH_BYTES (16u << 20)  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[MXM_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device.  The array's name in host code is only a
// host-side handle, so the address is looked up once per device (with that device current) and cached.
static int noalloc_scratch(float** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (int e = mx_cuda_status(cudaGetDevice(&dev), "mxm_coldot_noalloc: cudaGetDevice")) return e;
  MX_CHECK_ARG(dev >= 0 && dev < 64, "mxm_coldot_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (int e = mx_cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "mxm_coldot_noalloc: cudaGetSymbolAddress"))
      return e;
    addr[dev] = p;
  }
  *out = static_cast<float*>(addr[dev]);
  return MXM_OK;
}

extern "C" int mxm_coldot_noalloc_chunks(int64_t T, int64_t K, int n, int num_sms, int* rows_per_chunk, int* chunks) {
  MX_CHECK_ARG(T >= 1 && K >= 64 && K % 64 == 0 && (n == 16 || n == 32 || n == 64) && num_sms >= 0 && rows_per_chunk &&
                   chunks, "mxm_coldot_noalloc_chunks: bad args");
  const int64_t per_chunk = K * n * (int64_t)sizeof(float);
  MX_CHECK_ARG(per_chunk <= (int64_t)MXM_NOALLOC_SCRATCH_BYTES,
               "mxm_coldot_noalloc: K * n = %lld needs %lld bytes of scratch per row chunk, more than the fixed "
               "%u-byte scratch (K * n must be <= %u)",
               (long long)(K * n), (long long)per_chunk, MXM_NOALLOC_SCRATCH_BYTES,
               MXM_NOALLOC_SCRATCH_BYTES / (unsigned)sizeof(float));
  // mxm_coldot's chunking (one wave of four CTAs per SM); on a B200 (148 SMs) its partials need at most
  // 4 * 148 * 64 * n * 4 bytes (9.7 MB at n = 64), inside the scratch; a device with more SMs gets fewer,
  // taller row chunks so the partials still fit
  const int64_t ctas_k = K / CD_COLS;
  const int64_t want = 4 * (int64_t)(num_sms > 0 ? num_sms : mxm_num_sms());
  const int64_t nch = std::max<int64_t>(1, want / ctas_k);
  int64_t rpc = (T + nch - 1) / nch;
  rpc = std::max<int64_t>((rpc + CD_ROWS - 1) / CD_ROWS * CD_ROWS, 4 * CD_ROWS);
  int64_t nc = (T + rpc - 1) / rpc;
  const int64_t max_chunks = (int64_t)MXM_NOALLOC_SCRATCH_BYTES / per_chunk;
  if (nc > max_chunks) {
    rpc = (T + max_chunks - 1) / max_chunks;
    rpc = (rpc + CD_ROWS - 1) / CD_ROWS * CD_ROWS;
    nc = (T + rpc - 1) / rpc;
  }
  *rows_per_chunk = (int)rpc;
  *chunks = (int)nc;
  return MXM_OK;
}

extern "C" int mxm_coldot_noalloc(const void* A, int64_t lda, const void* E, int64_t lde, int64_t T, int64_t K, int n,
                                  float post, int transpose_out, void* out, void* stream) {
  MX_CHECK_ARG(A && E && out, "mxm_coldot_noalloc: null pointer");
  MX_CHECK_ARG(T >= 1 && K >= 64 && K % 64 == 0 && (n == 16 || n == 32 || n == 64),
               "mxm_coldot_noalloc: need T >= 1, K %% 64 == 0, n in {16, 32, 64}");
  int rpc = 0, chunks = 0;
  if (int e = mxm_coldot_noalloc_chunks(T, K, n, 0, &rpc, &chunks)) return e;
  float* scratch = nullptr;
  if (int e = noalloc_scratch(&scratch)) return e;
  // every partial the reduction reads is written by k_coldot first: nothing needs clearing
  return mxm_coldot(A, lda, E, lde, T, K, n, post, transpose_out, scratch, rpc, chunks, out, 0, stream);
}
