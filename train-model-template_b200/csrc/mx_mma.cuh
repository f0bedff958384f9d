// Warp-level bf16 MMA helpers (m16n8k16, fp32 accumulate) for the rank-r LoRA products that ride
// along the memory-bound MLP passes, plus the fragment shuffles they need.
//
// Fragment layouts (g = lane / 4, t = lane % 4), each .b32 register holds two bf16 (low = first):
//   A 16x16  a[0] = (row g,   k 2t..2t+1)   a[1] = (row g+8, k 2t..2t+1)
//            a[2] = (row g,   k 2t+8..+9)   a[3] = (row g+8, k 2t+8..+9)
//   B 16x8   b[0] = (k 2t..2t+1, col g)     b[1] = (k 2t+8..+9, col g)
//   D 16x8   d[0], d[1] = (row g, cols 2t, 2t+1)   d[2], d[3] = (row g+8, cols 2t, 2t+1)
// The D fragments of two adjacent 16x8 tiles, rounded to bf16 and packed, are exactly the A
// fragment of the 16x16 block they form (the usual accumulator-to-operand reuse).
#pragma once
#include "mx_common.cuh"

MX_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of the 8x8 bf16 block held in the m8n8 fragment layout (thread (g, t) holds row g,
// cols 2t..2t+1) -> thread (g, t) holds row g, cols 2t..2t+1 of the transpose.
MX_DEV uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

MX_DEV uint32_t ld32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }
MX_DEV uint32_t ld32g(const __nv_bfloat16* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
MX_DEV uint32_t ld16x2(const __nv_bfloat16* p0, const __nv_bfloat16* p1) {
  const uint32_t lo = __ldg(reinterpret_cast<const unsigned short*>(p0));
  const uint32_t hi = __ldg(reinterpret_cast<const unsigned short*>(p1));
  return lo | (hi << 16);
}
MX_DEV uint32_t ld16z(const __nv_bfloat16* p, bool valid) {
  return valid ? (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)) : 0u;
}

// ldmatrix: four 8x8 bf16 matrices from shared memory in fragment layout; lane L supplies the
// address of row (L % 8) of matrix (L / 8).  .trans delivers the transposed matrices.
MX_DEV void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
MX_DEV void ldsm4t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// stmatrix: the inverse of ldsm4 -- register i of every lane goes to matrix i in fragment layout;
// lane L supplies the address of row (L % 8) of matrix (L / 8).
MX_DEV void stsm4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
