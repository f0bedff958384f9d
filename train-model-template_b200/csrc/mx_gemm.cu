// MXFP8 block-scaled GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M, N] (bf16) = dq(A)[M, K] . dq(B)[N, K]^T  (+ L[M, kr] . Rm[N, kr]^T),  fp32 accumulation in TMEM,
//   A, B = E4M3 codes quantized along K with E8M0 scales in the 128x4 blocked layout.
//
// This is the operation torch._scaled_mm performs with MX scales in the reference
// (scripts/fused_mlp.py:279,283,309,329); the optional rank-kr term is the LoRA add that follows two of
// them (`y.addmm_(xS_down, B_down^T, alpha=s_d)`, `dx.addmm_(dxa, S)`, scripts/fused_mlp.py:284,331).
//
// Design (one CTA per SM, persistent over 128 x 256 output tiles, 12 warps):
//   warp 0      TMA producer: A tile [128 x 128B] and B tile [256 x 128B] per stage, 128-byte swizzled,
//               plus the stage's scale blocks (512 B for A, 2 x 512 B for B) with plain bulk copies --
//               the blocked layout already is the TMEM scale layout, no transpose.  With a LoRA term it
//               also loads, once per tile, L [128 x kr] and Rm [256 x kr] bf16 (kr*2-byte swizzle).
//   warp 1      MMA issuer (one thread): per stage, tcgen05.cp of the scales into TMEM (32x128b,
//               replicated over the four lane quarters) and four tcgen05.mma.kind::mxf8f6f4.block_scale
//               (M128 N256 K32, scale-factor id = 32-column block of the stage); after the last stage of
//               a tile, kr/16 tcgen05.mma.kind::f16 (bf16 x bf16 -> the same fp32 accumulator) add the
//               LoRA term on the tensor core.  Commits free stages and publish the accumulator.
//   warp 2      TMEM allocator (512 columns: accumulator 0..255, scales 256..267).
//   warps 4-11  epilogue: warp w reads TMEM lanes 32*(w%4).. and accumulator columns 128*((w-4)/4)..
//               into registers, hands the accumulator back at once (the next tile's MMAs overlap the
//               rest), then converts to bf16 and stores 16-byte vectors.
// Every mbarrier wait is bounded (see mbar_wait): on a timeout the kernel records an error code in the
// device flag and all roles fall through to the TMEM release and exit.
#include <algorithm>
#include <mutex>

#include "mx_common.cuh"
#include "mx_epi.cuh"
#include "mx_runtime.h"

namespace {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int A_BYTES = BM * BK;  // 16 KB
constexpr int B_BYTES = BN * BK;  // 32 KB
constexpr int SFA_BYTES = 512, SFB_BYTES = 1024;
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0, SFA_COL = 256, SFB_COL = 260;
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4, EPI_THREADS = 256;

__host__ __device__ constexpr int gemm_stages(int KR) { return KR == 64 ? 3 : 4; }
__host__ __device__ constexpr int lora_bytes(int KR) { return (BM + BN) * KR * 2; }
// Without a LoRA term or with a rank-16 one the epilogue warps stage their output in 2 KB pieces (32 rows x
// 32 columns each) for TMA stores; with a larger one shared memory is full and they store from registers.
__host__ __device__ constexpr bool tma_out(int KR) { return KR <= 16; }
// columns of one staged piece: 32 (2 KB, 64-byte swizzle) without a LoRA term, 16 (1 KB, 32-byte swizzle)
// with the rank-16 one, whose LoRA tiles leave room for only half the staging
__host__ __device__ constexpr int out_cols(int KR) { return KR == 0 ? 32 : 16; }
__host__ __device__ constexpr int out_bytes(int KR) { return tma_out(KR) ? 8 * 32 * out_cols(KR) * 2 : 0; }
__host__ __device__ constexpr size_t gemm_smem(int KR) {
  return 1024 + (size_t)gemm_stages(KR) * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES) + lora_bytes(KR) +
         out_bytes(KR) + 256;
}
// UMMA shared-memory layout code for a K-major bf16 tile with kr*2-byte rows (32/64/128-byte swizzle).
__host__ __device__ constexpr uint32_t lora_layout(int KR) { return KR == 16 ? 6u : (KR == 32 ? 4u : 2u); }

// Instruction descriptor of kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t bf16_idesc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int KR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_mx_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmL, const __grid_constant__ CUtensorMap tmR,
              const __grid_constant__ CUtensorMap tmD, const uint8_t* __restrict__ sa,
              const uint8_t* __restrict__ sb, int M, int N, int K, __nv_bfloat16* __restrict__ D, int64_t ldd,
              int* err) {
  constexpr int STAGES = gemm_stages(KR);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint8_t* sL = sSFB + STAGES * SFB_BYTES;  // 1024-aligned
  uint8_t* sR = sL + BM * KR * 2;
  uint8_t* sOut = sL + lora_bytes(KR);      // [8 warps][32 rows x 64 B] (tma_out), 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + out_bytes(KR));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* lora_full = tmem_full + 2;
  uint64_t* lora_empty = tmem_full + 3;
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(tmem_full + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int KT = K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, EPI_THREADS);
    mbar_init(lora_full, 1);
    mbar_init(lora_empty, 1);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;

  if (warp == 0) {
    // whole warp waits; lane 0 issues the copies
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      if (KR) {
        prefetch_tmap(&tmL);
        prefetch_tmap(&tmR);
      }
    }
    int stage = 0;
    uint32_t phase = 0, lphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int tm = tile / num_n, tn = tile % num_n;
      if constexpr (KR > 0) {
        if (!mbar_wait(lora_empty, lphase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(lora_full, lora_bytes(KR));
          tma_load_2d(sL, &tmL, lora_full, 0, tm * BM);
          tma_load_2d(sR, &tmR, lora_full, 0, tn * BN);
        }
        __syncwarp();
        lphase ^= 1;
      }
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint64_t* fb = &full[stage];
          mbar_arrive_expect_tx(fb, A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, fb, kt * BK, tm * BM);
          tma_load_2d(sB + stage * B_BYTES, &tmB, fb, kt * BK, tn * BN);
          bulk_load(sSFA + stage * SFA_BYTES, sa + ((int64_t)tm * KT + kt) * 512, 512, fb);
          bulk_load(sSFB + stage * SFB_BYTES, sb + ((int64_t)(2 * tn) * KT + kt) * 512, 512, fb);
          bulk_load(sSFB + stage * SFB_BYTES + 512, sb + ((int64_t)(2 * tn + 1) * KT + kt) * 512, 512, fb);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // whole warp waits; lane 0 issues the scale copies, the MMAs and the commits
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0, lphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      if (!mbar_wait(tmem_empty, acc_phase ^ 1, err, MX_DEV_TIMEOUT_MMA_TMEM)) break;
      tc_fence_after();
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sfa = smem_u32(sSFA + stage * SFA_BYTES);
          const uint32_t sfb = smem_u32(sSFB + stage * SFB_BYTES);
          tmem_cp_32x128b_x4(tmem + SFA_COL, make_sdesc(sfa, 0, 128, 0));
          tmem_cp_32x128b_x4(tmem + SFB_COL, make_sdesc(sfb, 0, 128, 0));
          tmem_cp_32x128b_x4(tmem + SFB_COL + 4, make_sdesc(sfb + 512, 0, 128, 0));
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = make_sdesc(a0 + k * 32, 0, 1024, 2);
            const uint64_t bd = make_sdesc(b0 + k * 32, 0, 1024, 2);
            umma_mxf8(tmem + ACC_COL, ad, bd, mx_idesc(BM, BN, k, k), tmem + SFA_COL, tmem + SFB_COL,
                      (kt | k) != 0);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if constexpr (KR > 0) {
        // LoRA term on the tensor core: acc += L [128 x kr] . Rm [256 x kr]^T (bf16, K-major, swizzled)
        if (!mbar_wait(lora_full, lphase, err, MX_DEV_TIMEOUT_MMA)) break;
        lphase ^= 1;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t l0 = smem_u32(sL), r0 = smem_u32(sR);
#pragma unroll
          for (int k = 0; k < KR / 16; ++k) {
            const uint64_t ld = make_sdesc(l0 + k * 32, 0, 8 * KR * 2, lora_layout(KR));
            const uint64_t rd = make_sdesc(r0 + k * 32, 0, 8 * KR * 2, lora_layout(KR));
            umma_bf16(tmem + ACC_COL, ld, rd, bf16_idesc(BM, BN), 1u);
          }
          umma_commit(lora_empty);
        }
        __syncwarp();
      }
      if (lane == 0) umma_commit(tmem_full);
      __syncwarp();
      acc_phase ^= 1;
    }
  } else if (warp >= EPI_WARP0) {
    const int q = warp & 3;                    // TMEM lane quarter of this warp
    const int half = (warp - EPI_WARP0) >> 2;  // accumulator columns [128*half, 128*half + 128)
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int tm = tile / num_n, tn = tile % num_n;
      if (!mbar_wait(tmem_full, acc_phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      uint32_t r[4][32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + ACC_COL + half * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + c * 32, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(tmem_empty);  // the accumulator is free: the next tile's MMAs start now
      acc_phase ^= 1;
      if constexpr (tma_out(KR)) {
        // pieces of OC columns of this warp's 32 x 128 block: bf16 rows into the warp's buffer (2*OC-byte
        // rows, matching swizzle), then one TMA store of the [32 x OC] box (rows >= M clipped); the buffer is
        // reused once the previous store has read it
        constexpr int OC = out_cols(KR), RB = 2 * OC;
        uint8_t* buf = sOut + (warp - EPI_WARP0) * (32 * RB);
        const uint32_t sb0 = smem_u32(buf) + (uint32_t)lane * RB;
        const uint64_t pol = l2_evict_first();   // dh / y are streamed to the next kernel
#pragma unroll
        for (int pc = 0; pc < 128 / OC; ++pc) {
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < OC / 8; ++j) {
            const int col = pc * OC + 8 * j;   // of the warp's 128 columns: r[col / 32][col % 32 ..]
            const uint32_t* v = &r[col >> 5][col & 31];
            const uint32_t a = sb0 + ((uint32_t)(j ^ ((lane >> (RB == 64 ? 1 : 2)) & (RB / 16 - 1))) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                         "r"(pack_bf16x2(__uint_as_float(v[0]), __uint_as_float(v[1]))),
                         "r"(pack_bf16x2(__uint_as_float(v[2]), __uint_as_float(v[3]))),
                         "r"(pack_bf16x2(__uint_as_float(v[4]), __uint_as_float(v[5]))),
                         "r"(pack_bf16x2(__uint_as_float(v[6]), __uint_as_float(v[7])))
                         : "memory");
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d_hint(&tmD, buf, tn * BN + half * 128 + pc * OC, tm * BM + q * 32, pol);
            bulk_commit();
          }
        }
        continue;
      }
      const int64_t row = (int64_t)tm * BM + q * 32 + lane;
      if (row < M) {
        uint4* dst = reinterpret_cast<uint4*>(D + row * ldd + (int64_t)tn * BN + half * 128);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(r[c][8 * j + 0]), __uint_as_float(r[c][8 * j + 1]));
            o.y = pack_bf16x2(__uint_as_float(r[c][8 * j + 2]), __uint_as_float(r[c][8 * j + 3]));
            o.z = pack_bf16x2(__uint_as_float(r[c][8 * j + 4]), __uint_as_float(r[c][8 * j + 5]));
            o.w = pack_bf16x2(__uint_as_float(r[c][8 * j + 6]), __uint_as_float(r[c][8 * j + 7]));
            dst[4 * c + j] = o;
          }
      }
    }
    if constexpr (tma_out(KR)) {
      if (lane == 0) bulk_wait0();   // this warp's stores are complete before the CTA exits
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------
// Gate|up GEMM with the SwiGLU-LoRA forward epilogue fused in (the reference's gu GEMM and _fwd_kernel,
// scripts/fused_mlp.py:279-282 and :81-109).  A tile pairs gate columns [128 tn, +128) with the up
// columns N + 128 tn .. of the same 128 outputs, so one tcgen05 accumulator of 128 rows x 256 columns
// holds both halves of 128 (g, u) column pairs.  Two launch shapes share one body:
//   * single CTA (k_mx_gemm_glu): 128-row tiles; a B stage is two TMA boxes of W_gu rows (gate, up) and
//     its two B scale blocks are the matching ones; 3 stages of 48 KB fit beside the epilogue's buffers.
//   * CTA pair (k_mx_gemm_glu2, cluster of two, cta_group::2): 256-row tiles; CTA r stages A rows
//     [256 tm + 128 r, +128) and one half of B (r = 0: the gate rows, r = 1: the up rows), the leader
//     issues M256 N256 K32 MMAs over both CTAs' shared memory, and each CTA's TMEM receives its own 128
//     rows x [gate | up] -- the same accumulator the single-CTA epilogue reads.  Per SM a k-block moves
//     32 KB of operands instead of 48 KB and the 33 KB stages leave room for 4 of them.  The peer's TMA
//     copies complete on the leader's full barriers; the leader's commits arrive on both CTAs' barriers;
//     each epilogue warp hands the accumulator back by one remote arrival on the leader's tmem_empty.
// The 8 epilogue warps drain the accumulator (warp q|h: lanes 32q.., half h = gate / up), hand it back
// and stage the bf16 tile in shared memory (128-byte swizzle); after one named barrier each warp runs
// the forward epilogue on 16 rows x 128 pairs of the staged tile -- the LoRA-B terms with mma.sync,
// SwiGLU, the MXFP8 codes of h, and the per-row xS_down = h A_down^T accumulated in registers -- while
// the MMAs of the next tile proceed; g and u with their LoRA terms go back into the staged tile, from
// which each warp writes its 16 rows of gu for the backward (two [16 x 64] TMA stores per finished
// 64-column sub-tile, full 128-byte rows).  A CTA (pair) works through a contiguous range of tiles (column tiles fastest), so xS_down
// accumulates over the columns of a row block and is written as one fp32 partial per (row block, CTA or
// pair); a fixed-order reduction sums them.  Rank 16 only (the rank-32 slices do not fit shared memory).
constexpr int GLU_STAGING = 2 * 2 * 128 * 128;   // g | u halves, two [128 x 64] bf16 sub-tiles each
template <bool PAIR> __host__ __device__ constexpr int glu_stages() { return PAIR ? 4 : 3; }
template <bool PAIR> __host__ __device__ constexpr int glu_bstage() { return PAIR ? 128 * BK : 256 * BK; }
__host__ __device__ constexpr int glu_slices(int R) { return 2 * 128 * R * 2 + R * 128 * 2; }
template <bool PAIR> __host__ __device__ constexpr size_t glu_ring() {
  return ((size_t)glu_stages<PAIR>() * (A_BYTES + glu_bstage<PAIR>() + SFA_BYTES + SFB_BYTES) + 1023) / 1024 * 1024;
}
template <bool PAIR> __host__ __device__ constexpr size_t glu_smem(int R) {
  return 1024 + glu_ring<PAIR>() + GLU_STAGING + glu_slices(R) + 256;
}

MX_DEV void epi_sync() { asm volatile("bar.sync 1, %0;" ::"r"(EPI_THREADS) : "memory"); }

template <int R, bool PAIR>
MX_DEV void glu_body(const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmG, const CUtensorMap* tmSA,
                     const CUtensorMap* tmSB, const uint8_t* __restrict__ sa, const uint8_t* __restrict__ sb, int M,
                     int N, int K, const __nv_bfloat16* __restrict__ xs, const __nv_bfloat16* __restrict__ bg,
                     const __nv_bfloat16* __restrict__ bu, const __nv_bfloat16* __restrict__ ad, float s_g, float s_u,
                     uint8_t* __restrict__ qh, uint8_t* __restrict__ sh, float* __restrict__ xsd_part, int chunk,
                     int* err) {
  constexpr int STAGES = glu_stages<PAIR>(), B_STAGE = glu_bstage<PAIR>(), KS = R / 16;
  constexpr int TM_ROWS = PAIR ? 256 : BM;                 // rows of one tile (of the pair)
  constexpr uint32_t STAGE_TX = (PAIR ? 2u : 1u) * (A_BYTES + B_STAGE + SFA_BYTES + SFB_BYTES);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_STAGE;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint8_t* stg = smem + glu_ring<PAIR>();     // [g | u][2 sub-tiles][128 rows x 128 B], 128-byte swizzle
  uint8_t* sl = stg + GLU_STAGING;           // Bg, Bu [128 x R] (2R-byte swizzle), Ad [2][R x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sl + glu_slices(R));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(tmem_full + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;   // CTA or pair
  const int num_m = (M + TM_ROWS - 1) / TM_ROWS;
  const int num_n = N / 128;
  const int KT = K / BK;
  // Schedule: a row block's column tiles are cut into chunks of `chunk` consecutive tiles (chunk divides
  // num_n); unit u takes chunks u, u + units, u + 2 units, ... in order, so at any time the units work on
  // neighbouring chunks -- a few row blocks of A and all of W_gu stay in L2 -- and each chunk's xS_down
  // partial goes to slot (chunk index within its row block).
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int ncpr = num_n / chunk;
  const int num_chunks = num_m * ncpr;
  const int my_tiles = unit < num_chunks ? ((num_chunks - 1 - unit) / units + 1) * chunk : 0;
  auto tile_of = [&](int i, int& tm, int& tn) {
    const int c = unit + (i / chunk) * units;
    tm = c / ncpr;
    tn = (c % ncpr) * chunk + i % chunk;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    // single CTA: every epilogue thread arrives; pair: one remote arrival per epilogue warp of each CTA
    mbar_init(tmem_empty, PAIR ? 2 * (EPI_THREADS / 32) : EPI_THREADS);
    fence_barrier_init();
  }
  if (warp == 2) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_alloc(tmem_base, TMEM_COLS);
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();   // barriers and TMEM of both CTAs exist before any cross-CTA operation
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  constexpr int SFA_COL = 256, SFB_COL = 260;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(tmA);
      prefetch_tmap(tmB);
      if constexpr (PAIR) {
        prefetch_tmap(tmSA);
        prefetch_tmap(tmSB);
      }
    }
    int stage = 0, issued = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      int tm, tn;
      tile_of(i, tm, tn);
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if constexpr (PAIR) {
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            const int mb = tm * 2 + (int)rank;                     // this CTA's 128-row block of A
            if (leader) mbar_arrive_expect_tx(&full[stage], STAGE_TX);
            tma_load_2d_pair(sA + stage * A_BYTES, tmA, fb, kt * BK, mb * BM);
            tma_load_2d_pair(sB + stage * B_STAGE, tmB, fb, kt * BK, (int)rank * N + tn * 128);  // gate / up rows
            tma_load_2d_pair(sSFA + stage * SFA_BYTES, tmSA, fb, 0, 2 * (mb * KT + kt));
            tma_load_2d_pair(sSFB + stage * SFB_BYTES, tmSB, fb, 0, 2 * (tn * KT + kt));
            tma_load_2d_pair(sSFB + stage * SFB_BYTES + 512, tmSB, fb, 0, 2 * ((num_n + tn) * KT + kt));
          } else {
            uint64_t* fb = &full[stage];
            mbar_arrive_expect_tx(fb, STAGE_TX);
            tma_load_2d(sA + stage * A_BYTES, tmA, fb, kt * BK, tm * BM);
            tma_load_2d(sB + stage * B_STAGE, tmB, fb, kt * BK, tn * 128);             // gate rows
            tma_load_2d(sB + stage * B_STAGE + 128 * BK, tmB, fb, kt * BK, N + tn * 128); // up rows
            bulk_load(sSFA + stage * SFA_BYTES, sa + ((int64_t)tm * KT + kt) * 512, 512, fb);
            bulk_load(sSFB + stage * SFB_BYTES, sb + ((int64_t)tn * KT + kt) * 512, 512, fb);
            bulk_load(sSFB + stage * SFB_BYTES + 512, sb + ((int64_t)(num_n + tn) * KT + kt) * 512, 512, fb);
          }
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if constexpr (PAIR) {
      // the leader's last commits to this CTA's empty barriers have landed before the CTA may exit
      for (int k = 0; k < STAGES && k < issued; ++k) {
        const int i = issued - 1 - k;
        mbar_wait(&empty[i % STAGES], (uint32_t)((i / STAGES) & 1), err, MX_DEV_TIMEOUT_PRODUCER);
      }
    }
  } else if (warp == 1 && leader) {
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0;
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      if (!mbar_wait(tmem_empty, acc_phase ^ 1, err, MX_DEV_TIMEOUT_MMA_TMEM)) break;
      tc_fence_after();
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[stage], phase, err, MX_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sfa = smem_u32(sSFA + stage * SFA_BYTES);
          const uint32_t sfb = smem_u32(sSFB + stage * SFB_BYTES);
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_STAGE);
          if constexpr (PAIR) {
            tmem_cp_32x128b_x4_pair(tmem + SFA_COL, make_sdesc(sfa, 0, 128, 0));
            tmem_cp_32x128b_x4_pair(tmem + SFB_COL, make_sdesc(sfb, 0, 128, 0));
            tmem_cp_32x128b_x4_pair(tmem + SFB_COL + 4, make_sdesc(sfb + 512, 0, 128, 0));
          } else {
            tmem_cp_32x128b_x4(tmem + SFA_COL, make_sdesc(sfa, 0, 128, 0));
            tmem_cp_32x128b_x4(tmem + SFB_COL, make_sdesc(sfb, 0, 128, 0));
            tmem_cp_32x128b_x4(tmem + SFB_COL + 4, make_sdesc(sfb + 512, 0, 128, 0));
          }
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t adsc = make_sdesc(a0 + k * 32, 0, 1024, 2);
            const uint64_t bdsc = make_sdesc(b0 + k * 32, 0, 1024, 2);
            if constexpr (PAIR)
              umma_mxf8_pair(tmem, adsc, bdsc, mx_idesc(256, 256, k, k), tmem + SFA_COL, tmem + SFB_COL,
                             (kt | k) != 0);
            else
              umma_mxf8(tmem, adsc, bdsc, mx_idesc(BM, 256, k, k), tmem + SFA_COL, tmem + SFB_COL, (kt | k) != 0);
          }
          if constexpr (PAIR)
            umma_commit_both(&empty[stage]);
          else
            umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) {
        if constexpr (PAIR)
          umma_commit_both(tmem_full);
        else
          umma_commit(tmem_full);
      }
      __syncwarp();
      acc_phase ^= 1;
    }
    // pair: both CTAs' epilogues have released the last accumulator (their remote arrivals have landed)
    if constexpr (PAIR) mbar_wait(tmem_empty, acc_phase ^ 1, err, MX_DEV_TIMEOUT_MMA_TMEM);
  } else if (warp >= EPI_WARP0) {
    const int e = warp - EPI_WARP0;            // SwiGLU rows 16e .. 16e+15 of a tile
    const int q = warp & 3, h = e >> 2;        // drain: TMEM lanes 32q .., accumulator half h (0 gate, 1 up)
    const int g = lane >> 2, t = lane & 3, mi = lane >> 3, lr = lane & 7;
    const int et = e * 32 + lane;              // 0 .. 255
    const int64_t Tpad = (int64_t)((M + BM - 1) / BM) * BM;
    const int lrow = e * 16 + (mi & 1) * 8 + lr;
    const uint32_t tmem_empty_l = PAIR ? mapa_shared(smem_u32(tmem_empty), 0) : 0u;
    uint32_t o_gu[4], o_b[4][KS], o_ad[4][KS];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      o_gu[p] = swz<128>((uint32_t)lrow, (uint32_t)(2 * p + (mi >> 1)));
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        o_b[p][kk] = swz<2 * R>((uint32_t)(8 * (2 * p + (mi >> 1)) + lr), (uint32_t)(2 * kk + (mi & 1)));
        o_ad[p][kk] = swz<128>((uint32_t)(16 * kk + 8 * (mi >> 1) + lr), (uint32_t)(2 * p + (mi & 1)));
      }
    }
    const uint32_t s_stg = smem_u32(stg), s_bg = smem_u32(sl), s_bu = s_bg + 128 * R * 2, s_ad = s_bu + 128 * R * 2;
    const float2 sg2 = make_float2(s_g, s_g), su2 = make_float2(s_u, s_u);
    float accx[R / 8][4];
    uint32_t axg[KS][4], axu[KS][4];
    QRows qr{};
    int64_t ra = 0, rb = 0;
    auto flush = [&](int slot) {   // this chunk's partial of xS_down for this warp's rows
      float* P = xsd_part + (int64_t)slot * M * R;
#pragma unroll
      for (int jt = 0; jt < R / 8; ++jt) {
        const int c = 8 * jt + 2 * t;
        if (ra < M) *reinterpret_cast<float2*>(P + ra * R + c) = make_float2(accx[jt][0], accx[jt][1]);
        if (rb < M) *reinterpret_cast<float2*>(P + rb * R + c) = make_float2(accx[jt][2], accx[jt][3]);
      }
    };
    uint32_t acc_phase = 0;
    // tile_of stepped: the chunk (its row block and first column tile) is divided out once per chunk
    int wc = unit, wii = 0, wtm = wc / ncpr, wtn0 = (wc % ncpr) * chunk;
    for (int i = 0; i < my_tiles; ++i) {
      const int tm = wtm, tn = wtn0 + wii;
      const int64_t rowb = (int64_t)tm * TM_ROWS + rank * BM;   // this CTA's first row of the tile
      if (wii == 0) {                    // a new chunk: this warp's rows of xs, zeroed xS_down sums
        ra = rowb + e * 16 + g;
        rb = ra + 8;
        const bool va = ra < M, vb = rb < M;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const __nv_bfloat16* pa = xs + ra * (2 * R) + 16 * kk + 2 * t;
          const __nv_bfloat16* pb = xs + rb * (2 * R) + 16 * kk + 2 * t;
          axg[kk][0] = va ? ld32(pa) : 0u;
          axg[kk][1] = vb ? ld32(pb) : 0u;
          axg[kk][2] = va ? ld32(pa + 8) : 0u;
          axg[kk][3] = vb ? ld32(pb + 8) : 0u;
          axu[kk][0] = va ? ld32(pa + R) : 0u;
          axu[kk][1] = vb ? ld32(pb + R) : 0u;
          axu[kk][2] = va ? ld32(pa + R + 8) : 0u;
          axu[kk][3] = vb ? ld32(pb + R + 8) : 0u;
        }
#pragma unroll
        for (int j = 0; j < R / 8; ++j) accx[j][0] = accx[j][1] = accx[j][2] = accx[j][3] = 0.f;
        qr = qrows_init(ra, M, Tpad, qh, N, sh, N, t);
      }
      // 1. drain the accumulator, hand it back, store gu and stage the bf16 tile (a warp whose wait ran
      // out skips this and the epilogue warps give up together at the named barrier below)
      const bool acc_ok = mbar_wait(tmem_full, acc_phase, err, MX_DEV_TIMEOUT_EPILOGUE);
      if (acc_ok) {
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + h * 128;
        const int rl = q * 32 + lane;
        const uint32_t sbase = s_stg + (uint32_t)h * (2 * 128 * 128);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {   // 64 columns at a time (one staged sub-tile)
          uint32_t r[2][32];
          tmem_ld32(taddr + c2 * 64, r[0]);
          tmem_ld32(taddr + c2 * 64 + 32, r[1]);
          tmem_ld_wait();
          if (c2 == 1) {   // the MMAs of the next tile start now
            tc_fence_before();
            if constexpr (PAIR) {
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(tmem_empty_l);
            } else {
              mbar_arrive(tmem_empty);
            }
          }
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(r[c][8 * j + 0]), __uint_as_float(r[c][8 * j + 1]));
              o.y = pack_bf16x2(__uint_as_float(r[c][8 * j + 2]), __uint_as_float(r[c][8 * j + 3]));
              o.z = pack_bf16x2(__uint_as_float(r[c][8 * j + 4]), __uint_as_float(r[c][8 * j + 5]));
              o.w = pack_bf16x2(__uint_as_float(r[c][8 * j + 6]), __uint_as_float(r[c][8 * j + 7]));
              // column 64 c2 + 32 c + 8 j of the half: sub-tile c2, chunk 4 c + j
              const uint32_t a = sbase + (uint32_t)c2 * (128 * 128) + swz<128>((uint32_t)rl, (uint32_t)(4 * c + j));
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(o.x), "r"(o.y), "r"(o.z),
                           "r"(o.w) : "memory");
            }
        }
        acc_phase ^= 1;
      }
      // 2. this tile's B_gate / B_up rows and A_down columns into shared memory
      for (int k = et; k < 128 * (R / 8); k += EPI_THREADS) {
        const int n = k / (R / 8), c = k % (R / 8);
        const uint4 vg = __ldg(reinterpret_cast<const uint4*>(bg + ((int64_t)tn * 128 + n) * R + 8 * c));
        const uint4 vu = __ldg(reinterpret_cast<const uint4*>(bu + ((int64_t)tn * 128 + n) * R + 8 * c));
        const uint32_t o = swz<2 * R>((uint32_t)n, (uint32_t)c);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(s_bg + o), "r"(vg.x), "r"(vg.y), "r"(vg.z),
                     "r"(vg.w) : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(s_bu + o), "r"(vu.x), "r"(vu.y), "r"(vu.z),
                     "r"(vu.w) : "memory");
      }
      for (int k = et; k < R * 16; k += EPI_THREADS) {
        const int j = k / 16, c8 = k % 16;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(ad + (int64_t)j * N + (int64_t)tn * 128 + 8 * c8));
        const uint32_t a = s_ad + (uint32_t)(c8 >> 3) * (R * 128) + swz<128>((uint32_t)j, (uint32_t)(c8 & 7));
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
      if (bar_any(1, EPI_THREADS, !acc_ok)) break;   // the epi_sync of this tile, and the give-up decision
      // 3. the forward epilogue on rows 16e .. 16e+15, two 64-column sub-tiles.  g and u with their LoRA
      // terms (the bf16 values the SwiGLU uses, which the backward would otherwise recompute) go back into
      // the staged tile, and gu leaves from it per warp and finished sub-tile, rows >= M clipped
#pragma unroll 1
      for (int sbk = 0; sbk < 2; ++sbk) {
        const uint32_t tg = s_stg + sbk * (128 * 128), tu = tg + 2 * 128 * 128;
        const uint32_t tbg = s_bg + sbk * (64 * R * 2), tbu = s_bu + sbk * (64 * R * 2), tad = s_ad + sbk * (R * 128);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t hp[4][2];
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            const int p = 2 * b + pp;
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
            for (int qq = 0; qq < 2; ++qq) {
              const float* dgv = qq ? dg1 : dg0;
              const float* duv = qq ? du1 : du0;
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                G[2 * qq + hh] = rn2(__ffma2_rn(sg2, make_float2(dgv[2 * hh], dgv[2 * hh + 1]), up2(G[2 * qq + hh])));
                U[2 * qq + hh] = rn2(__ffma2_rn(su2, make_float2(duv[2 * hh], duv[2 * hh + 1]), up2(U[2 * qq + hh])));
                const float2 gg = up2(G[2 * qq + hh]), uu = up2(U[2 * qq + hh]);
                hp[2 * pp + qq][hh] = rn2(__fmul2_rn(__fmul2_rn(gg, sigmoid2(gg)), uu));
              }
            }
            stsm4(tg + o_gu[p], G[0], G[1], G[2], G[3]);   // g, u with the LoRA terms, in place
            stsm4(tu + o_gu[p], U[0], U[1], U[2], U[3]);
          }
          quant_block16p(hp, qr, (int64_t)tn * 128 + sbk * 64 + 32 * b, t);
#pragma unroll
          for (int mm = 0; mm < 2; ++mm) {
            const uint32_t a4[4] = {hp[2 * mm][0], hp[2 * mm][1], hp[2 * mm + 1][0], hp[2 * mm + 1][1]};
#pragma unroll
            for (int jp = 0; jp < KS; ++jp) {
              uint32_t AD[4];
              ldsm4(AD, tad + o_ad[2 * b + mm][jp]);
              mma16816(accx[2 * jp], a4, AD[0], AD[1]);
              mma16816(accx[2 * jp + 1], a4, AD[2], AD[3]);
            }
          }
        }
        // this warp's 16 rows of sub-tile sbk of g and u are final: two [16 x 64] TMA stores (gu is next
        // read by the backward), no wait on the other warps
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && rowb + 16 * e < M) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
            tma_store_2d_hint(tmG, stg + (hh * 2 + sbk) * (128 * 128) + e * (16 * 128), hh * N + tn * 128 + sbk * 64,
                              (int)(rowb + 16 * e), qr.pol);
          bulk_commit();
        }
      }
      if (lane == 0) bulk_wait_read0();   // this warp's gu stores have read the staged tile
      epi_sync();   // staged tile and slices are free for the next tile
      if (wii == chunk - 1) flush(wc % ncpr);
      if (++wii == chunk) {
        wii = 0;
        wc += units;
        wtm = wc / ncpr;
        wtn0 = (wc % ncpr) * chunk;
      }
    }
    if (lane == 0) bulk_wait0();
  }

  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();
    tc_fence_after();
    if (warp == 2) tmem_dealloc_pair(tmem, TMEM_COLS);
  } else {
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int R>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_mx_gemm_glu(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmG, const uint8_t* __restrict__ sa,
                  const uint8_t* __restrict__ sb, int M, int N, int K, const __nv_bfloat16* __restrict__ xs,
                  const __nv_bfloat16* __restrict__ bg, const __nv_bfloat16* __restrict__ bu,
                  const __nv_bfloat16* __restrict__ ad, float s_g, float s_u, uint8_t* __restrict__ qh,
                  uint8_t* __restrict__ sh, float* __restrict__ xsd_part, int chunk, int* err) {
  glu_body<R, false>(&tmA, &tmB, &tmG, nullptr, nullptr, sa, sb, M, N, K, xs, bg, bu, ad, s_g, s_u, qh, sh, xsd_part,
                     chunk, err);
}

// CTA-pair launch shape: scale blocks come in by TMA as [blocks * KT * 2, 256] byte tensors (tmSA, tmSB)
template <int R>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    k_mx_gemm_glu2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmSA,
                   const __grid_constant__ CUtensorMap tmSB, int M, int N, int K, const __nv_bfloat16* __restrict__ xs,
                   const __nv_bfloat16* __restrict__ bg, const __nv_bfloat16* __restrict__ bu,
                   const __nv_bfloat16* __restrict__ ad, float s_g, float s_u, uint8_t* __restrict__ qh,
                   uint8_t* __restrict__ sh, float* __restrict__ xsd_part, int chunk, int* err) {
  glu_body<R, true>(&tmA, &tmB, &tmG, &tmSA, &tmSB, nullptr, nullptr, M, N, K, xs, bg, bu, ad, s_g, s_u, qh, sh,
                    xsd_part, chunk, err);
}

// xsd [M, R] bf16 = the fixed-order sum over the `slots` chunk partials (chunk 0, 1, .. of each row block).
__global__ void k_glu_xsd_reduce(const float* __restrict__ part, int M, int R, int slots,
                                 __nv_bfloat16* __restrict__ xsd) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)M * R; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int c = 0; c < slots; ++c) v += part[(int64_t)c * M * R + i];
    xsd[i] = __float2bfloat16_rn(v);
  }
}

CUtensorMapSwizzle lora_swizzle(int kr) {
  return kr == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : (kr == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

int gemm_launch(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb, int64_t M,
                int64_t N, int64_t K, void* d, int64_t ldd, const void* L, int64_t ldl, const void* Rm, int kr,
                void* stream, const char* fn) {
  MX_CHECK_ARG(qa && sa && qb && sb && d, "%s: null pointer", fn);
  MX_CHECK_ARG(M >= 1 && M < (1ll << 31), "%s: M=%lld out of range", fn, (long long)M);
  MX_CHECK_ARG(N >= BN && N % BN == 0 && N < (1ll << 31), "%s: N=%lld must be a multiple of %d", fn, (long long)N, BN);
  MX_CHECK_ARG(K >= BK && K % BK == 0 && K < (1ll << 31), "%s: K=%lld must be a multiple of %d", fn, (long long)K, BK);
  MX_CHECK_ARG(lda >= K && ldb >= K && lda % 16 == 0 && ldb % 16 == 0, "%s: lda/ldb must be >= K and 16-aligned", fn);
  MX_CHECK_ARG(ldd >= N && ldd % 8 == 0 && mx_aligned(d, 16), "%s: output stride/alignment", fn);
  MX_CHECK_ARG(mx_aligned(sa, 16) && mx_aligned(sb, 16), "%s: scale buffers must be 16-byte aligned", fn);
  if (kr) {
    MX_CHECK_ARG(kr == 16 || kr == 32 || kr == 64, "%s: LoRA rank must be 16, 32 or 64", fn);
    MX_CHECK_ARG(L && Rm && ldl >= kr && ldl % 8 == 0 && mx_aligned(L, 16) && mx_aligned(Rm, 16),
                 "%s: LoRA operands must be 16-byte aligned with row stride %% 8 == 0", fn);
  }

  CUtensorMap tmA, tmB, tmL, tmR, tmD;
  if (int st = mx_make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qa, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK,
                               BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (int st = mx_make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qb, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK,
                               BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (kr) {
    if (int st = mx_make_tmap_2d(&tmL, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, L, (uint64_t)kr, (uint64_t)M,
                                 (uint64_t)ldl * 2, kr, BM, lora_swizzle(kr)))
      return st;
    if (int st = mx_make_tmap_2d(&tmR, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Rm, (uint64_t)kr, (uint64_t)N,
                                 (uint64_t)kr * 2, kr, BN, lora_swizzle(kr)))
      return st;
  } else {
    tmL = tmR = tmA;  // unused by the kernel
  }
  if (kr <= 16) {
    // the output's map for the epilogue's TMA stores ([32 x 32] boxes)
    if (int st = mx_make_tmap_2d(&tmD, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, (uint64_t)N, (uint64_t)M,
                                 (uint64_t)ldd * 2, (uint32_t)out_cols(kr), 32,
                                 kr == 0 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B))
      return st;
  } else {
    tmD = tmA;        // unused: the epilogue stores from registers
  }

  static bool attr_done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int vi = kr == 0 ? 0 : (kr == 16 ? 1 : (kr == 32 ? 2 : 3));
  const void* kfns[4] = {(const void*)k_mx_gemm<0>, (const void*)k_mx_gemm<16>, (const void*)k_mx_gemm<32>,
                         (const void*)k_mx_gemm<64>};
  const size_t smem_by[4] = {gemm_smem(0), gemm_smem(16), gemm_smem(32), gemm_smem(64)};
  if (dev >= 0 && dev < 64 && !attr_done[vi][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kfns[vi], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_by[vi]);
    if (e != cudaSuccess) return mx_cuda_status(e, "gemm: set smem");
    attr_done[vi][dev] = true;
  }
  const int num_tiles = (int)(((M + BM - 1) / BM) * (N / BN));
  const int grid = num_tiles < mxm_num_sms() ? num_tiles : mxm_num_sms();
  auto go = [&](auto kern) {
    kern<<<grid, NUM_THREADS, smem_by[vi], (cudaStream_t)stream>>>(tmA, tmB, tmL, tmR, tmD, (const uint8_t*)sa,
                                                                  (const uint8_t*)sb, (int)M, (int)N, (int)K,
                                                                  (__nv_bfloat16*)d, ldd, mx_dev_error_ptr());
  };
  if (vi == 0)
    go(k_mx_gemm<0>);
  else if (vi == 1)
    go(k_mx_gemm<16>);
  else if (vi == 2)
    go(k_mx_gemm<32>);
  else
    go(k_mx_gemm<64>);
  mx_note_launch();
  return mx_launch_status(fn);
}

}  // namespace

extern "C" int mxm_gemm(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                        int64_t M, int64_t N, int64_t K, void* d, int64_t ldd, void* stream) {
  return gemm_launch(qa, lda, sa, qb, ldb, sb, M, N, K, d, ldd, nullptr, 0, nullptr, 0, stream, "mxm_gemm");
}

extern "C" int mxm_gemm_lora(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                             int64_t M, int64_t N, int64_t K, const void* L, int64_t ldl, const void* Rm, int kr,
                             void* d, int64_t ldd, void* stream) {
  return gemm_launch(qa, lda, sa, qb, ldb, sb, M, N, K, d, ldd, L, ldl, Rm, kr, stream, "mxm_gemm_lora");
}

// ------------------------------------------------------------------------------------------------ fused gate|up
namespace {
// CTA pairs of k_mx_gemm_glu2 that can be resident at once on the current device; 0 selects the
// single-CTA kernel (no room for a cluster of two).  Queried once per device.
int glu_pairs() {
  static int pairs[64] = {};
  static bool done[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    done[dev] = true;
    const size_t smem = glu_smem<true>(16);
    int n = 0;
    cudaError_t e = cudaFuncSetAttribute(k_mx_gemm_glu2<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (unsigned)(mxm_num_sms() / 2), 1, 1);
      cfg.blockDim = dim3(NUM_THREADS, 1, 1);
      cfg.dynamicSmemBytes = smem;
      e = cudaOccupancyMaxActiveClusters(&n, k_mx_gemm_glu2<16>, &cfg);
    }
    if (e != cudaSuccess) {   // refused: clear the error and run the single-CTA kernel instead
      cudaGetLastError();
      n = 0;
    }
    pairs[dev] = n;
  }
  return pairs[dev];
}
bool glu_use_pairs(int64_t M) { return M >= 256 && glu_pairs() > 0; }
}  // namespace

extern "C" int mxm_gemm_glu_partition(int64_t M, int64_t N, int* per, int* grid, int* slots) {
  MX_CHECK_ARG(M >= 1 && N >= 128 && N % 128 == 0 && per && grid && slots, "mxm_gemm_glu_partition: bad args");
  // units: CTA pairs over 256-row tiles when they fit, otherwise single CTAs over 128-row tiles
  const bool pair = glu_use_pairs(M);
  const int64_t rows = pair ? 256 : BM, units_max = pair ? glu_pairs() : mxm_num_sms();
  const int64_t num_m = (M + rows - 1) / rows, num_n = N / 128;
  // chunk = column tiles per chunk, a divisor of num_n: the one with the least estimated time, counting the
  // busiest unit's tiles (a tile ~ rows x 256 x 2048 x 2 FLOP at ~2.4 PFLOP/s over the units) and the
  // xS_down partials (slots x M x 16 fp32, written and read back, at ~6 TB/s)
  const double t_tile = 2.0 * rows * 256 * 2048 / (2.4e15 / (double)units_max);
  int64_t best_c = 1;
  double best_t = 1e30;
  for (int64_t c = 1; c <= num_n; ++c) {
    if (num_n % c) continue;
    const int64_t chunks = num_m * (num_n / c);
    const int64_t busiest = (chunks + units_max - 1) / units_max * c;
    const double t = busiest * t_tile + (double)(num_n / c) * (double)M * 16 * 4 * 2 / 6e12;
    if (t < best_t * (1.0 - 1e-9)) {
      best_t = t;
      best_c = c;
    }
  }
  const int64_t chunks = num_m * (num_n / best_c);
  const int64_t u = chunks < units_max ? chunks : units_max;
  *per = (int)best_c;
  *grid = (int)(pair ? 2 * u : u);
  *slots = (int)(num_n / best_c);   // chunks per row block: one xS_down partial each
  return MXM_OK;
}

extern "C" int mxm_gemm_glu(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                            int64_t M, int64_t N, int64_t K, void* gu, const void* xs, const void* bg, const void* bu,
                            const void* ad, int r, float s_g, float s_u, void* qh, void* sh, void* xsd_part, void* xsd,
                            void* stream) {
  MX_CHECK_ARG(qa && sa && qb && sb && gu && xs && bg && bu && ad && qh && sh && xsd_part && xsd,
               "mxm_gemm_glu: null pointer");
  MX_CHECK_ARG(r == 16, "mxm_gemm_glu: LoRA rank %d not supported (16 only)", r);
  MX_CHECK_ARG(M >= 1 && M < (1ll << 31) && N >= 128 && N % 128 == 0 && 2 * N * M < (1ll << 31) && K >= BK &&
                   K % BK == 0 && lda >= K && ldb >= K && lda % 16 == 0 && ldb % 16 == 0,
               "mxm_gemm_glu: need N %% 128 == 0, K %% 128 == 0, 2N * M < 2^31");
  MX_CHECK_ARG(mx_aligned(gu, 16) && mx_aligned(xs, 4) && mx_aligned(bg, 16) && mx_aligned(bu, 16) &&
                   mx_aligned(ad, 16) && mx_aligned(sa, 16) && mx_aligned(sb, 16) && mx_aligned(qh, 8),
               "mxm_gemm_glu: alignment");
  int per = 0, grid = 0, slots = 0;
  if (int e = mxm_gemm_glu_partition(M, N, &per, &grid, &slots)) return e;
  const bool pair = glu_use_pairs(M);
  CUtensorMap tmA, tmB, tmG;
  if (int st = mx_make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qa, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK,
                               BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (int st = mx_make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qb, (uint64_t)K, (uint64_t)(2 * N),
                               (uint64_t)ldb, BK, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (int st = mx_make_tmap_2d(&tmG, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gu, (uint64_t)(2 * N), (uint64_t)M,
                               (uint64_t)(4 * N), 64, 16, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  cudaStream_t st = (cudaStream_t)stream;
  if (pair) {
    // scale blocks as [blocks * KT * 2, 256] byte tensors: one 512-byte block = two 256-byte rows
    const int64_t KT = K / BK;
    CUtensorMap tmSA, tmSB;
    if (int e = mx_make_tmap_2d(&tmSA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, sa, 256, (uint64_t)((M + 127) / 128 * KT * 2),
                                256, 256, 2, CU_TENSOR_MAP_SWIZZLE_NONE))
      return e;
    if (int e = mx_make_tmap_2d(&tmSB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, sb, 256, (uint64_t)(2 * N / 128 * KT * 2), 256,
                                256, 2, CU_TENSOR_MAP_SWIZZLE_NONE))
      return e;
    k_mx_gemm_glu2<16><<<grid, NUM_THREADS, glu_smem<true>(16), st>>>(
        tmA, tmB, tmG, tmSA, tmSB, (int)M, (int)N, (int)K, (const __nv_bfloat16*)xs, (const __nv_bfloat16*)bg,
        (const __nv_bfloat16*)bu, (const __nv_bfloat16*)ad, s_g, s_u, (uint8_t*)qh, (uint8_t*)sh, (float*)xsd_part, per,
        mx_dev_error_ptr());   // per: column tiles per chunk
  } else {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = glu_smem<false>(16);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_mx_gemm_glu<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return mx_cuda_status(e, "gemm glu: set smem");
      attr_done[dev] = true;
    }
    k_mx_gemm_glu<16><<<grid, NUM_THREADS, smem, st>>>(tmA, tmB, tmG, (const uint8_t*)sa, (const uint8_t*)sb, (int)M,
                                                       (int)N, (int)K, (const __nv_bfloat16*)xs,
                                                       (const __nv_bfloat16*)bg, (const __nv_bfloat16*)bu,
                                                       (const __nv_bfloat16*)ad, s_g, s_u, (uint8_t*)qh, (uint8_t*)sh,
                                                       (float*)xsd_part, per, mx_dev_error_ptr());
  }
  mx_note_launch();
  if (int e = mx_launch_status("gemm glu")) return e;
  const int64_t n = M * r;
  const int rg = (int)std::min<int64_t>((n + 255) / 256, (int64_t)mxm_num_sms() * 8);
  k_glu_xsd_reduce<<<rg, 256, 0, st>>>((const float*)xsd_part, (int)M, r, slots, (__nv_bfloat16*)xsd);
  mx_note_launch();
  return mx_launch_status("gemm glu xsd reduce");
}
