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
#include "mx_common.cuh"
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
__host__ __device__ constexpr size_t gemm_smem(int KR) {
  return 1024 + (size_t)gemm_stages(KR) * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES) + lora_bytes(KR) + 256;
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
              const uint8_t* __restrict__ sa, const uint8_t* __restrict__ sb, int M, int N, int K,
              __nv_bfloat16* __restrict__ D, int64_t ldd, int* err) {
  constexpr int STAGES = gemm_stages(KR);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint8_t* sL = sSFB + STAGES * SFB_BYTES;  // 1024-aligned
  uint8_t* sR = sL + BM * KR * 2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + lora_bytes(KR));
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
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
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

  CUtensorMap tmA, tmB, tmL, tmR;
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
    tmL = tmA;  // unused by the kernel
    tmR = tmA;
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
    kern<<<grid, NUM_THREADS, smem_by[vi], (cudaStream_t)stream>>>(tmA, tmB, tmL, tmR, (const uint8_t*)sa,
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
