// Shared device helpers for the sm_100a MXFP8 kernels: number formats, the E8M0
// round-up, mbarriers with bounded waits, TMA, and the tcgen05 (TMEM / UMMA) wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mxmlp.h"

#define MX_DEV __device__ __forceinline__

// ------------------------------------------------------------------------------------------------
// Device-side error flag: a bounded wait that runs out records where it gave up and the kernel
// returns instead of hanging.  Kernels get the flag's address as an argument (mx_dev_error_ptr()
// on the host); the host reads and clears it with mxm_device_error().

enum MxDevError : int {
  MX_DEV_OK = 0,
  MX_DEV_TIMEOUT_PRODUCER = 1,
  MX_DEV_TIMEOUT_MMA = 2,
  MX_DEV_TIMEOUT_EPILOGUE = 3,
  MX_DEV_TIMEOUT_MMA_TMEM = 4,
  MX_DEV_TIMEOUT_SELFTEST = 9,   // the wait of mxm_selftest_wait (nobody arrives by design)
};

MX_DEV void mx_set_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

MX_DEV uint64_t mx_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------
// Number formats.

// E8M0 scale of a block: the power of two >= descale (round toward +inf), saturating to 254,
// NaN -> 255.  One PTX instruction on sm_100a (cvt.rp.satfinite.ue8m0x2.f32).
MX_DEV uint32_t mx_e8m0_rceil(float descale) {
  uint16_t r;
  asm("cvt.rp.satfinite.ue8m0x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(descale));
  return r & 0xFFu;
}

// The same E8M0 scale computed from the block's abs-max without the division: rceil(RN(amax / 448)).
// amax is a bf16 value (the abs-max of bf16 inputs), s * 2^E with a 7-bit fraction; 448 = 1.75 * 2^8,
// so amax / 448 = (s / 1.75) * 2^(E-8) with s / 1.75 in [0.57, 1.15): it rounds up to 2^(E-8) when
// s <= 1.75 and to 2^(E-7) when s > 1.75 (fraction > 0x60), and no value is near enough to a power of
// two for the fp32 rounding of the quotient to change that.  In the bf16 bits that is
// ((bits + 0x1F) >> 7) - 8, clamped at 0 (scales below 2^-127), with +inf -> 254 and NaN -> 255 as the
// saturating cvt gives.  Checked against the division for all 32,768 non-negative bf16 values.
MX_DEV uint32_t mx_e8m0_of_amax(float amax) {
  const uint32_t b = __float_as_uint(amax) >> 16;  // bf16-exact: the low half is zero
  int e = (int)((b + 0x1Fu) >> 7) - 8;
  e = e < 0 ? 0 : e;
  e = b == 0x7F80u ? 254 : e;
  e = b > 0x7F80u ? 255 : e;
  return (uint32_t)e;
}

// Multiplier applied to the block before the E4M3 cast: 255 -> NaN, 254 -> 2^-127,
// 0 -> 1.0, else 2^(127 - e).  2^(127-e) is built from its exponent bits (exact).
MX_DEV float mx_e8m0_rcp(uint32_t e) {
  uint32_t r = (254u - e) << 23;        // 2^(127 - e) for e in 1 .. 253
  r = e == 0u ? 0x3f800000u : r;        // 1.0
  r = e == 254u ? 0x00400000u : r;      // 2^-127 (subnormal)
  r = e == 255u ? 0x7fffffffu : r;      // NaN
  return __uint_as_float(r);
}

// Two floats (already clamped to [-448, 448], or NaN) -> two E4M3 codes, RNE.
// NaN always becomes the canonical code 0x7F.
MX_DEV uint16_t mx_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  if (lo != lo) r = (uint16_t)((r & 0xFF00u) | 0x7Fu);
  if (hi != hi) r = (uint16_t)((r & 0x00FFu) | 0x7F00u);
  return r;
}

MX_DEV float mx_clamp448(float v) {
  // fminf/fmaxf would drop a NaN; the block's NaN must survive to the cast.
  return (v != v) ? v : fminf(fmaxf(v, -448.0f), 448.0f);
}

MX_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
MX_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
MX_DEV float bf16_round_f(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
MX_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// |x| maximum that propagates NaN (amax of a block is NaN when the block holds a NaN).
MX_DEV float mx_absmax_nan(float a, float b) {
  float r = fmaxf(fabsf(a), fabsf(b));
  return (a != a || b != b) ? __int_as_float(0x7fffffff) : r;
}
MX_DEV float mx_max_nan(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fffffff) : fmaxf(a, b);
}

// Offset of the scale of (row r, 32-block kb) in the blocked 128x4 layout of a [*, cols] operand.
MX_DEV __host__ int64_t mx_scale_offset(int64_t r, int64_t kb, int64_t cols) {
  return ((r >> 7) * (cols >> 7) + (kb >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (kb & 3);
}

// ------------------------------------------------------------------------------------------------
// Shared-memory addresses, mbarriers.
MX_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MX_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
MX_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
MX_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

MX_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
MX_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
MX_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Non-blocking test of the phase with the given parity (for a warp that polls more than one barrier).
MX_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up after `limit_ns` of wall
// time (globaltimer), records `err` and returns false: no wait in these kernels is unbounded.
#ifndef MX_WAIT_LIMIT_NS
#define MX_WAIT_LIMIT_NS 2000000000ull  // 2 s
#endif
MX_DEV bool mbar_wait_ns(uint64_t* bar, uint32_t parity, int* flag, int err, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = mx_globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (mx_globaltimer() - t0 > limit_ns) {
      mx_set_error(flag, err);
      return false;
    }
  }
}
MX_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* flag, int err) {
  return mbar_wait_ns(bar, parity, flag, err, MX_WAIT_LIMIT_NS);
}

// Named barrier `id` over `nthreads` threads that also ORs a predicate across them: warps that wait on
// the same mbarrier with their own clocks decide to give up together (a warp that gave up alone would
// leave the others waiting at the next named barrier).
MX_DEV bool bar_any(uint32_t id, uint32_t nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}

// Named barrier `id` over `nthreads` threads (a multiple of 32).
MX_DEV void bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this project).
MX_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
// Plain bulk copy global -> shared (both 16-byte aligned, size a multiple of 16).
MX_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// Tiled store shared -> global (bulk-group completion): x = innermost coordinate (elements), y = row.
MX_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(map), "r"(x), "r"(y), "r"(smem_u32(src)) : "memory");
}
// L2 policy for data written once and not read again soon (streamed outputs): evict first, so the lines
// of a GEMM's operands, reused across tiles, are the ones that stay in L2.
MX_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// tma_store_2d with an L2 cache policy (l2_evict_first for streamed outputs).
MX_DEV void tma_store_2d_hint(const CUtensorMap* map, const void* src, int32_t x, int32_t y, uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;"
               ::"l"(map), "r"(x), "r"(y), "r"(smem_u32(src)), "l"(pol) : "memory");
}
// The same for a 3-D box (x innermost).
MX_DEV void tma_store_3d_hint(const CUtensorMap* map, const void* src, int32_t x, int32_t y, int32_t z, uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2, %3}], [%4], %5;"
               ::"l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(src)), "l"(pol) : "memory");
}
MX_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared-memory sources of this thread's committed bulk stores have been read.
MX_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's committed bulk stores are complete.
MX_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
MX_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, copies, loads.
MX_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MX_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
MX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format, version 1).
// layout: 0 none, 2 = 128B swizzle.  lbo / sbo in bytes.
MX_DEV uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::mxf8f6f4 with E4M3 A/B, K-major A/B, UE8M0 scales.
__host__ __device__ constexpr uint32_t mx_idesc(int M, int N, uint32_t sfa_id, uint32_t sfb_id) {
  return ((sfb_id & 3u) << 4) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24) |
         ((sfa_id & 3u) << 29);
}

MX_DEV void umma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t tsfa,
                      uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb) : "memory");
}
// bf16 x bf16 -> fp32 MMA into the same kind of accumulator (kind::f16).
MX_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
MX_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 rows x 128 bits from shared memory into TMEM, replicated to all four lane quarters.
MX_DEV void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
MX_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 8 consecutive 32-bit columns -> 8 registers per thread.
MX_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
MX_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
MX_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Instruction descriptor of kind::f16 with bf16 A / B and fp32 D; a_mn / b_mn select the MN-major
// (transposed) layout of A / B in shared memory instead of K-major.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- CTA pairs (cluster of two, cta_group::2): the leader (rank 0) issues MMAs that read both CTAs'
// shared memory and write both CTAs' TMEM.  No load here is multicast.
MX_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
MX_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cta address -> the shared::cluster address of the same offset in CTA `rank` of the cluster
MX_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
MX_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// tiled TMA load into this CTA's shared memory whose completion is counted on an mbarrier of the pair
// (bar_cluster: a shared::cluster address, normally the leader's barrier)
MX_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.cta_group::2 "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
MX_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
MX_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
MX_DEV void tmem_cp_32x128b_x4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
MX_DEV void umma_mxf8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t tsfa,
                           uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb) : "memory");
}
// commit of the pair's MMAs, arriving on the barrier at the same offset in both CTAs
MX_DEV void umma_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3) : "memory");
}

MX_DEV uint32_t lane_id() { return threadIdx.x & 31u; }
MX_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\telect.sync rx|px, 0xffffffff;\n\tselp.u32 %0, 1, 0, px;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
