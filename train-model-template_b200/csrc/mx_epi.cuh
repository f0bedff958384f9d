// Element-wise helpers shared by the memory-bound MLP epilogues (csrc/mx_mlp.cu) and the GEMM with the
// fused SwiGLU epilogue (csrc/mx_gemm.cu): packed f32x2 / bf16x2 arithmetic, the MXFP8 quantization of a
// warp tile held in mma D-fragment form, predicated stores, and the shared-memory swizzle of TMA tiles.
#pragma once
#include "mx_mma.cuh"

MX_DEV float nanmax(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// Two floats -> two E4M3 codes (RNE, saturating: |v| <= 448 after the power-of-two block scaling,
// and +-inf saturates to +-448 exactly as the reference's clamp does).
MX_DEV uint32_t e4m3x2_sat(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Predicated global stores (no branch around them).
MX_DEV void stg16_if(void* p, uint32_t v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.b16 [%0], %1;\n\t}" ::"l"(p),
               "h"((uint16_t)v), "r"((int)pred));
}
MX_DEV void stg64_if(void* p, uint32_t lo, uint32_t hi, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t@q st.global.v2.b32 [%0], {%1, %2};\n\t}" ::"l"(p),
               "r"(lo), "r"(hi), "r"((int)pred));
}
MX_DEV void stg128_if(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q st.global.v4.b32 [%0], {%1, %2, %3, %4};\n\t}" ::"l"(p),
               "r"(a), "r"(b), "r"(c), "r"(d), "r"((int)pred));
}
MX_DEV void stg8_if(void* p, uint32_t v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.b8 [%0], %1;\n\t}" ::"l"(p),
               "h"((uint16_t)v), "r"((int)pred));
}
// the same with an L2 cache policy (evict-first for streamed outputs)
MX_DEV void stg64_if_hint(void* p, uint32_t lo, uint32_t hi, bool pred, uint64_t pol) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t@q st.global.L2::cache_hint.v2.b32 [%0], {%1, %2}, %4;\n\t}"
               ::"l"(p), "r"(lo), "r"(hi), "r"((int)pred), "l"(pol));
}
MX_DEV void stg128_if_hint(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d, bool pred, uint64_t pol) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %6;\n\t}"
               ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d), "r"((int)pred), "l"(pol));
}
MX_DEV void stg8_if_hint(void* p, uint32_t v, bool pred, uint64_t pol) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.L2::cache_hint.b8 [%0], %1, %3;\n\t}"
               ::"l"(p), "h"((uint16_t)v), "r"((int)pred), "l"(pol));
}

// ---- packed helpers: two values per instruction (Blackwell f32x2 ALU ops, bf16x2 conversions)
MX_DEV float2 up2(uint32_t p) { return make_float2(bf16_lo(p), bf16_hi(p)); }
MX_DEV uint32_t rn2(float2 v) { return pack_bf16x2(v.x, v.y); }   // round both to bf16 (RNE)
MX_DEV float ex2a(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
MX_DEV float rcpa(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// sigmoid(g) = 1 / (1 + exp(-g)) for a pair (exp via ex2 of -g*log2(e))
MX_DEV float2 sigmoid2(float2 g) {
  const float2 t = __fmul2_rn(g, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  return make_float2(rcpa(ex2a(t.x) + 1.0f), rcpa(ex2a(t.y) + 1.0f));
}
MX_DEV uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("{\n\t.reg .b32 x, y;\n\tabs.bf16x2 x, %1;\n\tabs.bf16x2 y, %2;\n\tmax.NaN.bf16x2 %0, x, y;\n\t}"
      : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// max(|a|, |b|) per half with the xor of the signs as the sign (NaN if either is NaN): chains of these
// give a block's abs-max up to its sign bit, which the caller clears once.
MX_DEV uint32_t amax_xs_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// {f32(lo(p)) + c.x, f32(hi(p)) + c.y}, each rounded once: the bf16 halves feed the adds directly.
MX_DEV float2 add_bf16x2_f32(uint32_t p, float2 c) {
  float2 r;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.bf16 %0, lo, %3;\n\t"
      "add.rn.f32.bf16 %1, hi, %4;\n\t}"
      : "=f"(r.x), "=f"(r.y) : "r"(p), "f"(c.x), "f"(c.y));
  return r;
}
// {f32(lo(p)) * s, f32(hi(p)) * s} for a bf16 power of two s (exact scaling; -0 addend keeps -0 products).
MX_DEV float2 scale_bf16x2(uint32_t p, uint16_t s) {
  float2 r;
  asm("{\n\t.reg .b16 lo, hi;\n\t.reg .f32 z;\n\tmov.b32 {lo, hi}, %2;\n\tmov.b32 z, 0x80000000;\n\t"
      "fma.rn.f32.bf16 %0, lo, %3, z;\n\tfma.rn.f32.bf16 %1, hi, %3, z;\n\t}"
      : "=f"(r.x), "=f"(r.y) : "r"(p), "h"(s));
  return r;
}
MX_DEV uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Per-thread store targets of the MX output of one 16-row warp tile (rows g and g + 8), fixed for the
// whole kernel: the code row pointers (+ 2t), the scale bytes of k-block 0, and the store predicates
// (codes for rows < T; scales for rows < Tpad, written by lane t = 0 of the quad).
struct QRows {
  uint8_t* code[2];
  uint8_t* scale[2];
  bool live[2], slive[2];
  uint64_t pol;   // L2 policy of the code / scale stores (evict first: the outputs are streamed)
};
MX_DEV QRows qrows_init(int64_t row_g, int64_t T, int64_t Tpad, uint8_t* q, int64_t ldq, uint8_t* s, int64_t scols,
                        int t) {
  QRows r;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t row = row_g + 8 * h;
    r.live[h] = row < T;
    r.slive[h] = t == 0 && row < Tpad;
    r.code[h] = q ? q + (r.live[h] ? row : 0) * ldq + 2 * t : nullptr;
    r.scale[h] = s ? s + mx_scale_offset(row < Tpad ? row : 0, 0, scols) : nullptr;
  }
  r.pol = l2_evict_first();
  return r;
}

// Quad transpose of 16-bit pairs: lane t of each quad holds c[i] (the codes of columns 8i+2t, +1,
// i = 0..3) as r0 = c0 | c1 << 16, r1 = c2 | c3 << 16; afterwards it holds the codes of its own 8
// columns 8t .. 8t+7 in order (r0 = columns 8t .. 8t+3, r1 = 8t+4 .. 8t+7).  Two steps: swap the
// off-diagonal 2 x 2 blocks between lanes t and t ^ 2, then transpose each 2 x 2 block between t, t ^ 1.
MX_DEV void quad_transpose16(uint32_t& r0, uint32_t& r1, int t) {
  const bool lo = t < 2;
  const uint32_t got = __shfl_xor_sync(0xffffffffu, lo ? r1 : r0, 2);
  if (lo) r1 = got; else r0 = got;
  const uint32_t o0 = __shfl_xor_sync(0xffffffffu, r0, 1), o1 = __shfl_xor_sync(0xffffffffu, r1, 1);
  const bool even = (t & 1) == 0;
  r0 = even ? __byte_perm(r0, o0, 0x5410) : __byte_perm(o0, r0, 0x7632);
  r1 = even ? __byte_perm(r1, o1, 0x5410) : __byte_perm(o1, r1, 0x7632);
}

// Quantizes one 32-column block (columns col0 .. col0+31, col0 % 32 == 0) of a 16-row warp tile whose
// bf16 values are held packed in D-fragment form: pk[i][h] = (row g + 8h, cols 8i+2t, +1), i = 0..3
// (t = lane % 4).  Codes and the two rows' scales go to the targets of `qr`; after a quad transpose
// each lane writes 8 consecutive codes, so a quad fills the row's 32-byte sector in one store.
MX_DEV void quant_block16p(const uint32_t (&pk)[4][2], const QRows& qr, int64_t col0, int t) {
  const int64_t soff = ((col0 >> 7) << 9) + ((col0 >> 5) & 3);  // k-block col0/32 in the blocked layout
  // both rows' abs-maxes in one bf16x2 (an abs-max of bf16 values is a bf16 value): (row g | row g + 8);
  // the xorsign maxima carry a meaningless sign, cleared at the end
  const uint32_t m0 = amax_xs_bf16x2(amax_xs_bf16x2(pk[0][0], pk[1][0]), amax_xs_bf16x2(pk[2][0], pk[3][0]));
  const uint32_t m1 = amax_xs_bf16x2(amax_xs_bf16x2(pk[0][1], pk[1][1]), amax_xs_bf16x2(pk[2][1], pk[3][1]));
  uint32_t mm = amax_xs_bf16x2(__byte_perm(m0, m1, 0x5410), __byte_perm(m0, m1, 0x7632));
  mm = amax_xs_bf16x2(mm, __shfl_xor_sync(0xffffffffu, mm, 1));
  mm = amax_xs_bf16x2(mm, __shfl_xor_sync(0xffffffffu, mm, 2)) & 0x7FFF7FFFu;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t e = mx_e8m0_of_amax(h ? bf16_hi(mm) : bf16_lo(mm));
    // 2^(127 - e) (1.0, 2^-127, NaN for e = 0, 254, 255) is a bf16 value: its high half
    const uint16_t rcp = (uint16_t)(__float_as_uint(mx_e8m0_rcp(e)) >> 16);
    uint32_t c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = scale_bf16x2(pk[i][h], rcp);
      c[i] = e4m3x2_sat(v.x, v.y);
    }
    uint32_t r0 = __byte_perm(c[0], c[1], 0x5410), r1 = __byte_perm(c[2], c[3], 0x5410);
    quad_transpose16(r0, r1, t);
    stg64_if_hint(qr.code[h] + col0 + 6 * t, r0, r1, qr.live[h], qr.pol);   // code[h] points at column 2t
    stg8_if_hint(qr.scale[h] + soff, e, qr.slive[h], qr.pol);
  }
}

// The same quantization for a 32-column block held whole by one thread (pk[i] = columns 2i, 2i+1): the
// 32 codes go to code[0 .. 31] in two 16-byte stores, the E8M0 scale to *scale; the same arithmetic as
// quant_block16p, without the shuffles.
MX_DEV void quant_row32(const uint32_t (&pk)[16], uint8_t* code, uint8_t* scale, bool live, bool slive, uint64_t pol) {
  uint32_t m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = amax_xs_bf16x2(pk[2 * i], pk[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] = amax_xs_bf16x2(m[2 * i], m[2 * i + 1]);
  m[0] = amax_xs_bf16x2(amax_xs_bf16x2(m[0], m[1]), amax_xs_bf16x2(m[2], m[3]));
  const uint32_t am = amax_xs_bf16x2(m[0], __byte_perm(m[0], 0u, 0x1032)) & 0x7FFFu;  // low half, sign cleared
  const uint32_t e = mx_e8m0_of_amax(__uint_as_float(am << 16));
  const uint16_t rcp = (uint16_t)(__float_as_uint(mx_e8m0_rcp(e)) >> 16);
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float2 v0 = scale_bf16x2(pk[2 * k], rcp), v1 = scale_bf16x2(pk[2 * k + 1], rcp);
    w[k] = e4m3x2_sat(v0.x, v0.y) | (e4m3x2_sat(v1.x, v1.y) << 16);
  }
  stg128_if_hint(code, w[0], w[1], w[2], w[3], live, pol);
  stg128_if_hint(code + 16, w[4], w[5], w[6], w[7], live, pol);
  stg8_if_hint(scale, e, slive, pol);
}

// 16-byte shared-memory load / store (ordered with the surrounding barrier waits and arrivals).
MX_DEV void lds128(uint32_t a, uint32_t* r) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a)
               : "memory");
}
MX_DEV void sts128(uint32_t a, const uint32_t* v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile with RB-byte rows stored by TMA with the
// matching RB-byte swizzle (RB = 32, 64, 128): chunk bits [4, 4+b) are XORed with address bits [7, 7+b).
template <int RB>
MX_DEV uint32_t swz(uint32_t row, uint32_t chunk) {
  constexpr uint32_t SH = RB == 128 ? 0 : (RB == 64 ? 1 : 2), MK = RB / 16 - 1;
  return row * RB + ((chunk ^ ((row >> SH) & MK)) << 4);
}
template <int RB>
__host__ __device__ constexpr CUtensorMapSwizzle swz_mode() {
  return RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// Rounds a pointer into dynamic shared memory up to 1024 bytes by pointer arithmetic, so the result
// keeps the shared state space (and the compiler keeps emitting shared-memory instructions for it).
MX_DEV uint8_t* align1024(uint8_t* p) { return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u); }



