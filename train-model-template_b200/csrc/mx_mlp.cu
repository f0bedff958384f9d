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

// ------------------------------------------------------------------------------------------------ helpers
MX_DEV float nanmax_abs(float m, float v) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(m), "f"(fabsf(v)));
  return r;
}
MX_DEV float nanmax(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// Division with the 2-ulp full-range PTX instruction (what a Triton `/` on fp32 lowers to).
MX_DEV float fdiv_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// Two floats -> two E4M3 codes (RNE, saturating: |v| <= 448 after the power-of-two block scaling,
// and +-inf saturates to +-448 exactly as the reference's clamp does).
MX_DEV uint32_t e4m3x2_sat(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

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
    for (int i = 0; i < 4; ++i) m = nanmax_abs(nanmax_abs(m, v[i][2 * h]), v[i][2 * h + 1]);
    m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const uint32_t e = mx_e8m0_rceil(__fdiv_rn(m, 448.0f));
    const float rcp = mx_e8m0_rcp(e);
    const int64_t row = row_g + 8 * h;
    if (row < T) {
      uint8_t* dst = q + row * ldq + col0 + 2 * t;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint16_t*>(dst + 8 * i) = (uint16_t)e4m3x2_sat(v[i][2 * h] * rcp, v[i][2 * h + 1] * rcp);
    }
    if (t == 0) s[mx_scale_offset(row, col0 >> 5, scols)] = (uint8_t)e;
  }
}

// exp(-g) once per element; silu = g / (e + 1) and sigmoid = 1 / (1 + e) share it
// (reference: g / (exp(-g) + 1), tl.sigmoid(g); scripts/fused_mlp.py:104,152,158).
MX_DEV float exp_neg(float g) { return __expf(-g); }

// bf16 pair (row r, cols c, c+1) of a [rows x 64] bf16 tile stored by TMA with the 128-byte swizzle
// (16-byte chunk j of row r sits at chunk j ^ (r % 8)).
MX_DEV uint32_t sw128_ld(const uint8_t* tile, int r, int c) {
  const int b = c * 2;
  return *reinterpret_cast<const uint32_t*>(tile + r * 128 + (((b >> 4) ^ (r & 7)) << 4) + (b & 15));
}
// Same for a [rows x 32] bf16 tile with 64-byte rows and the 64-byte swizzle (chunk j -> j ^ ((r / 2) % 4)).
MX_DEV uint32_t sw64_ld(const uint8_t* tile, int r, int c) {
  const int b = c * 2;
  return *reinterpret_cast<const uint32_t*>(tile + r * 64 + (((b >> 4) ^ ((r >> 1) & 3)) << 4) + (b & 15));
}

MX_DEV uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Named barrier among the consumer warps only (the producer warp does not take part).
MX_DEV void consumers_sync(int nthreads) { asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory"); }

constexpr int CONSUMERS = 8;                      // consumer warps (16 rows each: 128-row blocks)
constexpr int EPI_THREADS = 32 * (CONSUMERS + 1);  // + one TMA producer warp

// ------------------------------------------------------------------------------------------------ forward
// CTA = one 128-row block x one column group of `tpg` 64-column tiles.  Warp 8 streams the g and u
// tiles ([128 x 64] bf16 each, 128-byte swizzle) into a 3-stage ring with TMA; warps 0-7 each own 16
// rows, so the per-row xS_down accumulator stays in registers across the whole group.
constexpr int FWD_BN = 64, FWD_ST = 3, FWD_TILE = 128 * FWD_BN * 2;  // 16 KB per tensor tile
constexpr size_t FWD_SMEM = 1024 + FWD_ST * 2 * FWD_TILE + 2 * FWD_ST * sizeof(uint64_t);

template <int R>
__global__ void __launch_bounds__(EPI_THREADS, 1)
    k_mlp_fwd(const __grid_constant__ CUtensorMap tm_gu, const bf16* __restrict__ xs, const bf16* __restrict__ bg,
              const bf16* __restrict__ bu, const bf16* __restrict__ ad, uint8_t* __restrict__ qh,
              uint8_t* __restrict__ sh, float* __restrict__ xsd_part, bf16* __restrict__ xsd_out, int T, int N,
              float s_g, float s_u, int tpg, int write_q, int* err) {
  constexpr int KS = R / 16, NT = FWD_BN / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + FWD_ST * 2 * FWD_TILE);
  uint64_t* empty = full + FWD_ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * 128;
  if (threadIdx.x == 0) {
    for (int i = 0; i < FWD_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CONSUMERS) {  // TMA producer
    if (lane == 0) prefetch_tmap(&tm_gu);
    int stage = 0;
    uint32_t phase = 0;
    for (int ct = 0; ct < tpg; ++ct) {
      const int n0 = (blockIdx.y * tpg + ct) * FWD_BN;
      if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) break;
      if (lane == 0) {
        uint8_t* dst = smem + stage * 2 * FWD_TILE;
        mbar_arrive_expect_tx(&full[stage], 2 * FWD_TILE);
        tma_load_2d(dst, &tm_gu, &full[stage], n0, (int)row0);
        tma_load_2d(dst + FWD_TILE, &tm_gu, &full[stage], N + n0, (int)row0);
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

  int stage = 0;
  uint32_t phase = 0;
  for (int ct = 0; ct < tpg; ++ct) {
    const int n0 = (blockIdx.y * tpg + ct) * FWD_BN;
    if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
    const uint8_t* tg = smem + stage * 2 * FWD_TILE;
    const uint8_t* tu = tg + FWD_TILE;
    uint32_t ga[NT], gb[NT], ua[NT], ub[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int c = 8 * i + 2 * t;
      ga[i] = sw128_ld(tg, rl, c);
      gb[i] = sw128_ld(tg, rl + 8, c);
      ua[i] = sw128_ld(tu, rl, c);
      ub[i] = sw128_ld(tu, rl + 8, c);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == FWD_ST) {
      stage = 0;
      phase ^= 1;
    }
    float hv[NT][4];
    uint32_t hp[NT][2];
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
        hv[i][e] = bf16_round_f(fdiv_full(gg, exp_neg(gg) + 1.0f) * uu);
      }
      hp[i][0] = pack_bf16x2(hv[i][0], hv[i][1]);
      hp[i][1] = pack_bf16x2(hv[i][2], hv[i][3]);
    }
    if (write_q) {
#pragma unroll
      for (int b = 0; b < FWD_BN / 32; ++b) {
        const float(&blk)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&hv[4 * b][0]);
        quant_block16(blk, ra, T, n0 + 32 * b, qh, N, sh, N, t);
      }
    }
#pragma unroll
    for (int m = 0; m < FWD_BN / 16; ++m) {
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
// CTA = one super-block of SB rows x one column group of `tpg` 32-column tiles.  Warp 8 streams
// [128 x 32] bf16 tiles of g, u and dh (64-byte swizzle) into a 4-stage ring with TMA, column tile
// outer, 128-row step inner.  Warps 0-7 each own 16 rows of every step:
//   * dB_gate, dB_up, dA_down (sums over rows) accumulate in registers over the super-block, then the
//     8 warps' tiles are summed in a fixed order through shared memory -> one partial per super-block;
//   * dxa_gate, dxa_up, xS_down (sums over columns) accumulate in a shared-memory [SB x 3r] buffer
//     that each warp only touches in its own rows, written once per CTA as the group's partial.
// No atomics: the result is deterministic.
constexpr int BWD_BN = 32, BWD_ST = 4, BWD_TILE = 128 * BWD_BN * 2;  // 8 KB per tensor tile

__host__ __device__ constexpr size_t bwd_smem(int R, int SB) {
  return 1024 + (size_t)BWD_ST * 3 * BWD_TILE + (size_t)SB * 3 * R * 4 + (size_t)CONSUMERS * R * BWD_BN * 4 +
         2 * BWD_ST * sizeof(uint64_t);
}

template <int R>
__global__ void __launch_bounds__(EPI_THREADS, 1)
    k_mlp_bwd(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dh,
              const bf16* __restrict__ xs, const bf16* __restrict__ dxd, const bf16* __restrict__ bg,
              const bf16* __restrict__ bu, const bf16* __restrict__ ad, uint8_t* __restrict__ q,
              uint8_t* __restrict__ s, float* __restrict__ dxa_part, float* __restrict__ dbg_part,
              float* __restrict__ dbu_part, float* __restrict__ dad_part, int T, int Tpad, int N, float s_g,
              float s_u, int SB, int tpg, int write_q, int* err) {
  constexpr int KS = R / 16, NT = BWD_BN / 8, R3 = 3 * R;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  float* acc_rows = reinterpret_cast<float*>(smem + BWD_ST * 3 * BWD_TILE);  // [SB][3R]
  float* scratch = acc_rows + (size_t)SB * R3;                                 // [CONSUMERS][R][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + CONSUMERS * R * BWD_BN);
  uint64_t* empty = full + BWD_ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sbi = blockIdx.x, cg = blockIdx.y;
  const int r_begin = sbi * SB, r_end = min(r_begin + SB, Tpad);
  const int64_t N2 = 2 * (int64_t)N;
  if (threadIdx.x == 0) {
    for (int i = 0; i < BWD_ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CONSUMERS) {  // TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_gu);
      prefetch_tmap(&tm_dh);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int ct = 0; ct < tpg && ok; ++ct) {
      const int n0 = (cg * tpg + ct) * BWD_BN;
      for (int r = r_begin; r < r_end; r += 128) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* dst = smem + stage * 3 * BWD_TILE;
          mbar_arrive_expect_tx(&full[stage], 3 * BWD_TILE);
          tma_load_2d(dst, &tm_gu, &full[stage], n0, r);
          tma_load_2d(dst + BWD_TILE, &tm_gu, &full[stage], N + n0, r);
          tma_load_2d(dst + 2 * BWD_TILE, &tm_dh, &full[stage], n0, r);
        }
        __syncwarp();
        if (++stage == BWD_ST) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int nthr = CONSUMERS * 32;
  for (int i = threadIdx.x; i < SB * R3; i += nthr) acc_rows[i] = 0.f;
  consumers_sync(nthr);

  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int ct = 0; ct < tpg && ok; ++ct) {
    const int n0 = (cg * tpg + ct) * BWD_BN;
    float aBg[KS][NT][4], aBu[KS][NT][4], aAd[KS][NT][4];
#pragma unroll
    for (int a = 0; a < KS; ++a)
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) aBg[a][i][e] = aBu[a][i][e] = aAd[a][i][e] = 0.f;
    // B fragments of this column tile (same for every row step)
    uint32_t bgf[KS][NT][2], buf_[KS][NT][2], adf[KS][NT][2];
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int nc = n0 + 8 * i;
        const bf16* pbg = bg + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
        const bf16* pbu = bu + (int64_t)(nc + g) * R + 16 * kk + 2 * t;
        bgf[kk][i][0] = ld32g(pbg);
        bgf[kk][i][1] = ld32g(pbg + 8);
        buf_[kk][i][0] = ld32g(pbu);
        buf_[kk][i][1] = ld32g(pbu + 8);
        const bf16* p0 = ad + (int64_t)(16 * kk + 2 * t) * N + nc + g;
        adf[kk][i][0] = ld16x2(p0, p0 + N);
        adf[kk][i][1] = ld16x2(p0 + 8 * (int64_t)N, p0 + 9 * (int64_t)N);
      }

    for (int r = r_begin; r < r_end; r += 128) {
      const int rl = warp * 16 + g;                 // row within the step
      const int64_t ra = r + rl, rb = ra + 8;
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
      if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      const uint8_t* tg = smem + stage * 3 * BWD_TILE;
      const uint8_t* tu = tg + BWD_TILE;
      const uint8_t* th = tg + 2 * BWD_TILE;
      uint32_t ga[NT], gb[NT], ua[NT], ub[NT], ha[NT], hb[NT];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int c = 8 * i + 2 * t;
        ga[i] = sw64_ld(tg, rl, c);
        gb[i] = sw64_ld(tg, rl + 8, c);
        ua[i] = sw64_ld(tu, rl, c);
        ub[i] = sw64_ld(tu, rl + 8, c);
        ha[i] = sw64_ld(th, rl, c);
        hb[i] = sw64_ld(th, rl + 8, c);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == BWD_ST) {
        stage = 0;
        phase ^= 1;
      }

      uint32_t dgp[NT][2], dup[NT][2], hp[NT][2];
      float dgv[NT][4], duv[NT][4];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f}, dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          mma16816(dg, axg[kk], bgf[kk][i][0], bgf[kk][i][1]);
          mma16816(du, axu[kk], buf_[kk][i][0], buf_[kk][i][1]);
          mma16816(dd, axd[kk], adf[kk][i][0], adf[kk][i][1]);
        }
        const float gin[4] = {bf16_lo(ga[i]), bf16_hi(ga[i]), bf16_lo(gb[i]), bf16_hi(gb[i])};
        const float uin[4] = {bf16_lo(ua[i]), bf16_hi(ua[i]), bf16_lo(ub[i]), bf16_hi(ub[i])};
        const float hin[4] = {bf16_lo(ha[i]), bf16_hi(ha[i]), bf16_lo(hb[i]), bf16_hi(hb[i])};
        float hvv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float gg = bf16_round_f(gin[e] + s_g * dg[e]);
          const float uu = bf16_round_f(uin[e] + s_u * du[e]);
          const float en = exp_neg(gg) + 1.0f;
          const float sl = fdiv_full(gg, en);
          const float sig = fdiv_full(1.0f, en);
          hvv[e] = bf16_round_f(sl * uu);
          const float dh = bf16_round_f(hin[e] + dd[e]);
          duv[i][e] = bf16_round_f(dh * sl);
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
        const float(&bgv)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&dgv[0][0]);
        const float(&buv)[4][4] = *reinterpret_cast<const float(*)[4][4]>(&duv[0][0]);
        quant_block16(bgv, ra, T, n0, q, N2, s, N2, t);
        quant_block16(buv, ra, T, (int64_t)N + n0, q, N2, s, N2, t);
      }
      // per-row products (sums over columns) into the shared-memory row accumulators
      float* A0 = acc_rows + (int64_t)(ra - r_begin) * R3;
      float* A1 = A0 + 8 * R3;
      const uint32_t adg[4] = {dgp[0][0], dgp[0][1], dgp[1][0], dgp[1][1]};
      const uint32_t adg2[4] = {dgp[2][0], dgp[2][1], dgp[3][0], dgp[3][1]};
      const uint32_t adu[4] = {dup[0][0], dup[0][1], dup[1][0], dup[1][1]};
      const uint32_t adu2[4] = {dup[2][0], dup[2][1], dup[3][0], dup[3][1]};
      const uint32_t ah[4] = {hp[0][0], hp[0][1], hp[1][0], hp[1][1]};
      const uint32_t ah2[4] = {hp[2][0], hp[2][1], hp[3][0], hp[3][1]};
#pragma unroll
      for (int jt = 0; jt < R / 8; ++jt) {
        const int c = 8 * jt + 2 * t;
        const int j = 8 * jt + g;
        float pg[4], pu[4], px[4];
        {
          const float2 a0 = *reinterpret_cast<const float2*>(A0 + c), a1 = *reinterpret_cast<const float2*>(A1 + c);
          pg[0] = a0.x; pg[1] = a0.y; pg[2] = a1.x; pg[3] = a1.y;
          const float2 b0 = *reinterpret_cast<const float2*>(A0 + R + c), b1 = *reinterpret_cast<const float2*>(A1 + R + c);
          pu[0] = b0.x; pu[1] = b0.y; pu[2] = b1.x; pu[3] = b1.y;
          const float2 c0 = *reinterpret_cast<const float2*>(A0 + 2 * R + c), c1 = *reinterpret_cast<const float2*>(A1 + 2 * R + c);
          px[0] = c0.x; px[1] = c0.y; px[2] = c1.x; px[3] = c1.y;
        }
        // B[k = n][col j]: (n 2t..2t+1 | 2t+8..2t+9, col j), two 16-column halves of the tile
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const int64_t nn = n0 + 16 * m + 2 * t;
          const bf16* pb = bg + nn * R + j;
          const bf16* pu_ = bu + nn * R + j;
          const bf16* pad = ad + (int64_t)j * N + nn;
          mma16816(pg, m ? adg2 : adg, ld16x2(pb, pb + R), ld16x2(pb + 8 * R, pb + 9 * R));
          mma16816(pu, m ? adu2 : adu, ld16x2(pu_, pu_ + R), ld16x2(pu_ + 8 * R, pu_ + 9 * R));
          mma16816(px, m ? ah2 : ah, ld32g(pad), ld32g(pad + 8));
        }
        *reinterpret_cast<float2*>(A0 + c) = make_float2(pg[0], pg[1]);
        *reinterpret_cast<float2*>(A1 + c) = make_float2(pg[2], pg[3]);
        *reinterpret_cast<float2*>(A0 + R + c) = make_float2(pu[0], pu[1]);
        *reinterpret_cast<float2*>(A1 + R + c) = make_float2(pu[2], pu[3]);
        *reinterpret_cast<float2*>(A0 + 2 * R + c) = make_float2(px[0], px[1]);
        *reinterpret_cast<float2*>(A1 + 2 * R + c) = make_float2(px[2], px[3]);
      }
      // column products (sums over rows): [j x n] += xa^T (j x rows) . [dg | du | h] (rows x n)
#pragma unroll
      for (int jm = 0; jm < KS; ++jm) {
        const uint32_t tg4[4] = {movtrans(axg[jm][0]), movtrans(axg[jm][2]), movtrans(axg[jm][1]), movtrans(axg[jm][3])};
        const uint32_t tu4[4] = {movtrans(axu[jm][0]), movtrans(axu[jm][2]), movtrans(axu[jm][1]), movtrans(axu[jm][3])};
        const uint32_t td4[4] = {movtrans(axd[jm][0]), movtrans(axd[jm][2]), movtrans(axd[jm][1]), movtrans(axd[jm][3])};
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          mma16816(aBg[jm][i], tg4, movtrans(dgp[i][0]), movtrans(dgp[i][1]));
          mma16816(aBu[jm][i], tu4, movtrans(dup[i][0]), movtrans(dup[i][1]));
          mma16816(aAd[jm][i], td4, movtrans(hp[i][0]), movtrans(hp[i][1]));
        }
      }
    }
    if (!ok) break;
    // fixed-order sum of the 8 warps' column products, one product at a time through `scratch`
#pragma unroll
    for (int which = 0; which < 3; ++which) {
      float* W = scratch + warp * (R * BWD_BN);
#pragma unroll
      for (int jm = 0; jm < KS; ++jm)
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          const float* a = which == 0 ? aBg[jm][i] : (which == 1 ? aBu[jm][i] : aAd[jm][i]);
          const int j0 = 16 * jm + g, nn = 8 * i + 2 * t;
          W[j0 * BWD_BN + nn] = a[0];
          W[j0 * BWD_BN + nn + 1] = a[1];
          W[(j0 + 8) * BWD_BN + nn] = a[2];
          W[(j0 + 8) * BWD_BN + nn + 1] = a[3];
        }
      consumers_sync(nthr);
      for (int idx = threadIdx.x; idx < R * BWD_BN; idx += nthr) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) v += scratch[w * R * BWD_BN + idx];
        const int j = idx / BWD_BN, n = idx % BWD_BN;
        if (which == 0)
          dbg_part[((int64_t)sbi * N + n0 + n) * R + j] = v;
        else if (which == 1)
          dbu_part[((int64_t)sbi * N + n0 + n) * R + j] = v;
        else
          dad_part[((int64_t)sbi * R + j) * N + n0 + n] = v;
      }
      consumers_sync(nthr);
    }
  }
  // the group's partial of the per-row products
  float* P = dxa_part + (int64_t)cg * T * R3;
  for (int i = threadIdx.x; i < (r_end - r_begin) * R3; i += nthr) {
    const int64_t row = r_begin + i / R3;
    if (row < T) P[row * R3 + i % R3] = acc_rows[i];
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
  // one CTA per SM: the fewest column groups that still fill every SM twice
  const int64_t nrb = (T + 127) / 128;
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
  MX_CHECK_ARG(mx_aligned(gu, 16), "mxm_mlp_fwd_epilogue: gu must be 16-byte aligned");
  CUtensorMap tm;
  if (int e = mx_make_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gu, (uint64_t)(2 * N), (uint64_t)T,
                              (uint64_t)(4 * N), FWD_BN, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  dim3 grid((unsigned)((T + 127) / 128), (unsigned)col_groups);
  cudaStream_t st = (cudaStream_t)stream;
  const int tpg = nt / col_groups;
  bf16* direct = col_groups == 1 ? (bf16*)xsd : nullptr;
  auto go = [&](auto kern) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FWD_SMEM);
    if (e != cudaSuccess) return mx_cuda_status(e, "mlp fwd epilogue: set smem");
    kern<<<grid, EPI_THREADS, FWD_SMEM, st>>>(tm, (const bf16*)xs, (const bf16*)bg, (const bf16*)bu, (const bf16*)ad,
                                              (uint8_t*)qh, (uint8_t*)sh, (float*)xsd_part, direct, (int)T, (int)N,
                                              s_g, s_u, tpg, qh != nullptr, mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("mlp fwd epilogue");
  };
  if (int e = (r == 16 ? go(k_mlp_fwd<16>) : go(k_mlp_fwd<32>))) return e;
  if (col_groups > 1) {
    const int64_t n = T * r;
    k_sum_parts<<<grid_for(n, 256), 256, 0, st>>>((const float*)xsd_part, col_groups, n, n, 1.0f, 1.0f, nullptr,
                                                  (bf16*)xsd, 0, 0);
    mx_note_launch();
    if (int e = mx_launch_status("mlp fwd xsd sum")) return e;
  }
  return MXM_OK;
}

static int bwd_super_block(int r) { return r == 16 ? 512 : 256; }

// Backward partition: super-blocks of SB rows (shared-memory row accumulators bound SB) and the
// column-group count that minimises partial-sum bytes while giving every SM at least two CTAs
// (the same trade-off as the reference's _bwd_grid, scripts/fused_mlp.py:218-232).
extern "C" int mxm_mlp_bwd_partitions(int64_t T, int64_t N, int r, int* super_block, int* col_groups) {
  MX_CHECK_ARG(T >= 1 && N >= 128 && N % 128 == 0 && (r == 16 || r == 32) && super_block && col_groups,
               "mxm_mlp_bwd_partitions: bad args");
  const int64_t tpad = (T + 127) / 128 * 128;
  int sb = bwd_super_block(r);
  while (sb > 128 && (tpad + sb - 1) / sb < 2) sb /= 2;   // small T: smaller super-blocks, more CTAs
  const int64_t nsb = (tpad + sb - 1) / sb;
  const int nt = (int)(N / BWD_BN);
  const int64_t want = 2 * (int64_t)mxm_num_sms();
  int best = nt;
  for (int ncg = 1; ncg <= nt; ++ncg)
    if (nt % ncg == 0 && nsb * ncg >= want) {
      best = ncg;
      break;
    }
  *super_block = sb;
  *col_groups = best;
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
  const int nt = (int)(N / BWD_BN);
  MX_CHECK_ARG(col_groups >= 1 && nt % col_groups == 0 && super_block >= 128 && super_block % 128 == 0 &&
                   super_block <= bwd_super_block(r),
               "mxm_mlp_bwd_epilogue: bad partition (%d, %d)", super_block, col_groups);
  MX_CHECK_ARG(mx_aligned(gu, 16) && mx_aligned(dhm, 16), "mxm_mlp_bwd_epilogue: gu / dhm must be 16-byte aligned");
  CUtensorMap tgu, tdh;
  if (int e = mx_make_tmap_2d(&tgu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gu, (uint64_t)(2 * N), (uint64_t)T,
                              (uint64_t)(4 * N), BWD_BN, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = mx_make_tmap_2d(&tdh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dhm, (uint64_t)N, (uint64_t)T,
                              (uint64_t)(2 * N), BWD_BN, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  const int64_t tpad = (T + 127) / 128 * 128;
  const int nsb = (int)((tpad + super_block - 1) / super_block);
  dim3 grid((unsigned)nsb, (unsigned)col_groups);
  const size_t smem = bwd_smem(r, super_block);
  cudaStream_t st = (cudaStream_t)stream;
  const int tpg = nt / col_groups;
  auto go = [&](auto kern) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return mx_cuda_status(e, "mlp bwd epilogue: set smem");
    kern<<<grid, EPI_THREADS, smem, st>>>(tgu, tdh, (const bf16*)xs, (const bf16*)dxd, (const bf16*)bg,
                                          (const bf16*)bu, (const bf16*)ad, (uint8_t*)q, (uint8_t*)s,
                                          (float*)dxa_part, (float*)dbg_part, (float*)dbu_part, (float*)dad_part,
                                          (int)T, (int)tpad, (int)N, s_g, s_u, super_block, tpg, q != nullptr,
                                          mx_dev_error_ptr());
    mx_note_launch();
    return mx_launch_status("mlp bwd epilogue");
  };
  return r == 16 ? go(k_mlp_bwd<16>) : go(k_mlp_bwd<32>);
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
