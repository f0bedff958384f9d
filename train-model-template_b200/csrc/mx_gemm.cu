// MXFP8 block-scaled GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M, N] (bf16) = dq(A)[M, K] . dq(B)[N, K]^T,  fp32 accumulation in TMEM,
//   A, B = E4M3 codes quantized along K with E8M0 scales in the 128x4 blocked layout.
//
// This is the operation torch._scaled_mm performs with MX scales in the reference
// (scripts/fused_mlp.py:279,283,309,329).
//
// Design (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: A tile [128 x 128B] and B tile [256 x 128B] per stage, 128-byte
//               swizzled, plus the stage's scale blocks (512 B for A, 2 x 512 B for B) with plain
//               bulk copies -- the blocked layout already is the TMEM scale layout, no transpose.
//   warp 1      MMA issuer (one elected thread): per stage copies the scales into TMEM with
//               tcgen05.cp (32x128b, replicated over the four lane quarters) and issues four
//               tcgen05.mma.kind::mxf8f6f4.block_scale (M=128, N=256, K=32), scale-factor id = the
//               32-column block within the 128-column stage; commits free the stage.
//   warp 2      TMEM allocator (512 columns: accumulator 0..255, scales 256..267).
//   warps 4-7   epilogue: tcgen05.ld of the accumulator (warp i reads TMEM lanes 32i..32i+31),
//               bf16 conversion and 16-byte stores; then hands the accumulator back.
// Every mbarrier wait is bounded (see mbar_wait): on a timeout the kernel records an error code
// in the device flag and all roles fall through to the TMEM release and exit.
#include "mx_common.cuh"
#include "mx_runtime.h"

namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK;  // 16 KB
constexpr int B_BYTES = BN * BK;  // 32 KB
constexpr int SFA_BYTES = 512, SFB_BYTES = 1024;
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0, SFA_COL = 256, SFB_COL = 260;
constexpr int NUM_THREADS = 256;
constexpr int EPI_WARP0 = 4;

struct __align__(8) Bars {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full;
  uint64_t tmem_empty;
  uint32_t tmem_base;
};

constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES) + sizeof(Bars);

// Epilogue variants: KR == 0 stores bf16(acc); KR in {16, 32} adds a rank-KR LoRA term with the
// reference's two roundings: out = bf16( bf16(acc) + alpha * sum_j L[row, j] Rm[col, j] ), which is
// `y = _scaled_mm(...); y.addmm_(L, Rm^T, alpha=alpha)` (scripts/fused_mlp.py:283-284, :329-331).
template <int KR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_mx_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const uint8_t* __restrict__ sa, const uint8_t* __restrict__ sb, int M, int N, int K,
              __nv_bfloat16* __restrict__ D, int64_t ldd, const __nv_bfloat16* __restrict__ L, int64_t ldl,
              const __nv_bfloat16* __restrict__ Rm, float alpha, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sSFB + STAGES * SFB_BYTES);

  const int warp = threadIdx.x >> 5;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int KT = K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    mbar_init(&bars->tmem_full, 1);
    mbar_init(&bars->tmem_empty, 128);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&bars->tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    // whole warp waits; lane 0 issues the copies
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int tm = tile / num_n, tn = tile % num_n;
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&bars->empty[stage], phase ^ 1, err, MX_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint64_t* fb = &bars->full[stage];
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
    uint32_t phase = 0, acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      if (!mbar_wait(&bars->tmem_empty, acc_phase ^ 1, err, MX_DEV_TIMEOUT_MMA_TMEM)) break;
      tc_fence_after();
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&bars->full[stage], phase, err, MX_DEV_TIMEOUT_MMA)) {
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
          umma_commit(&bars->empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok && lane == 0) umma_commit(&bars->tmem_full);
      __syncwarp();
      acc_phase ^= 1;
    }
  } else if (warp >= EPI_WARP0) {
    const int q = warp - EPI_WARP0;  // TMEM lane quarter of this warp
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int tm = tile / num_n, tn = tile % num_n;
      if (!mbar_wait(&bars->tmem_full, acc_phase, err, MX_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int64_t row = (int64_t)tm * BM + q * 32 + lane;
      __nv_bfloat16* drow = D + row * ldd + (int64_t)tn * BN;
      float lr[KR > 0 ? KR : 1];
      if constexpr (KR > 0) {
#pragma unroll
        for (int j = 0; j < KR; j += 8) {
          uint4 u = row < M ? __ldg(reinterpret_cast<const uint4*>(L + row * ldl + j)) : make_uint4(0u, 0u, 0u, 0u);
          lr[j + 0] = bf16_lo(u.x); lr[j + 1] = bf16_hi(u.x);
          lr[j + 2] = bf16_lo(u.y); lr[j + 3] = bf16_hi(u.y);
          lr[j + 4] = bf16_lo(u.z); lr[j + 5] = bf16_hi(u.z);
          lr[j + 6] = bf16_lo(u.w); lr[j + 7] = bf16_hi(u.w);
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + ACC_COL + c * 32, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (KR > 0) {
          const __nv_bfloat16* rc = Rm + ((int64_t)tn * BN + c * 32) * KR;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < KR; j += 8) {
              const uint4 u = __ldg(reinterpret_cast<const uint4*>(rc + i * KR + j));
              dot = fmaf(lr[j + 0], bf16_lo(u.x), dot); dot = fmaf(lr[j + 1], bf16_hi(u.x), dot);
              dot = fmaf(lr[j + 2], bf16_lo(u.y), dot); dot = fmaf(lr[j + 3], bf16_hi(u.y), dot);
              dot = fmaf(lr[j + 4], bf16_lo(u.z), dot); dot = fmaf(lr[j + 5], bf16_hi(u.z), dot);
              dot = fmaf(lr[j + 6], bf16_lo(u.w), dot); dot = fmaf(lr[j + 7], bf16_hi(u.w), dot);
            }
            v[i] = bf16_round_f(v[i]) + alpha * dot;
          }
        }
        if (row < M) {
          uint4* dst = reinterpret_cast<uint4*>(drow + c * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 o;
            o.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            o.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            o.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            o.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            dst[j] = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->tmem_empty);
      acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
}

int gemm_launch(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                       int64_t M, int64_t N, int64_t K, void* d, int64_t ldd, const void* L, int64_t ldl,
                       const void* Rm, int kr, float alpha, void* stream, const char* fn) {
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

  CUtensorMap tmA, tmB;
  if (int st = mx_make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qa, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK,
                               BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (int st = mx_make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qb, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK,
                               BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;

  static bool attr_done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int vi = kr == 0 ? 0 : (kr == 16 ? 1 : (kr == 32 ? 2 : 3));
  const void* kfns[4] = {(const void*)k_mx_gemm<0>, (const void*)k_mx_gemm<16>, (const void*)k_mx_gemm<32>,
                         (const void*)k_mx_gemm<64>};
  const void* kfn = kfns[vi];
  if (dev >= 0 && dev < 64 && !attr_done[vi][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return mx_cuda_status(e, "gemm: set smem");
    attr_done[vi][dev] = true;
  }
  const int num_tiles = (int)(((M + BM - 1) / BM) * (N / BN));
  const int grid = num_tiles < mxm_num_sms() ? num_tiles : mxm_num_sms();
  auto args = [&](auto kern) {
    kern<<<grid, NUM_THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(
        tmA, tmB, (const uint8_t*)sa, (const uint8_t*)sb, (int)M, (int)N, (int)K, (__nv_bfloat16*)d, ldd,
        (const __nv_bfloat16*)L, ldl, (const __nv_bfloat16*)Rm, alpha, mx_dev_error_ptr());
    mx_note_launch();
  };
  if (vi == 0)
    args(k_mx_gemm<0>);
  else if (vi == 1)
    args(k_mx_gemm<16>);
  else if (vi == 2)
    args(k_mx_gemm<32>);
  else
    args(k_mx_gemm<64>);
  return mx_launch_status(fn);
}

}  // namespace

extern "C" int mxm_gemm(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                        int64_t M, int64_t N, int64_t K, void* d, int64_t ldd, void* stream) {
  return gemm_launch(qa, lda, sa, qb, ldb, sb, M, N, K, d, ldd, nullptr, 0, nullptr, 0, 1.0f, stream, "mxm_gemm");
}

extern "C" int mxm_gemm_lora(const void* qa, int64_t lda, const void* sa, const void* qb, int64_t ldb, const void* sb,
                             int64_t M, int64_t N, int64_t K, const void* L, int64_t ldl, const void* Rm, int kr,
                             float alpha, void* d, int64_t ldd, void* stream) {
  return gemm_launch(qa, lda, sa, qb, ldb, sb, M, N, K, d, ldd, L, ldl, Rm, kr, alpha, stream, "mxm_gemm_lora");
}
