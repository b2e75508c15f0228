// tcgen05 (5th-generation tensor core) building blocks shared by the GEMM
// kernels: MMA issue and commit, TMEM loads, shared-memory descriptors of the
// UMMA K-major canonical layout (no swizzle) and the int8 instruction
// descriptor with M = 128.
#pragma once
#include "common.cuh"

namespace nrc {

constexpr int TC_M = 128;  // rows per MMA tile

// int32 -> f32 for |v| < 2^22 in two full-rate operations: the bits of
// 1.5 * 2^23 + v are that float exactly, and subtracting 1.5 * 2^23 is exact.
constexpr uint32_t TC_MAGIC_BITS = 0x4B400000u;
constexpr float TC_MAGIC_F = 12582912.0f;
NRC_DEV float small_i2f(uint32_t v) { return __fsub_rn(__uint_as_float(v + TC_MAGIC_BITS), TC_MAGIC_F); }
NRC_DEV float2 small_i2f2(uint32_t a, uint32_t b) {
  return __fadd2_rn(make_float2(__uint_as_float(a + TC_MAGIC_BITS), __uint_as_float(b + TC_MAGIC_BITS)),
                    make_float2(-TC_MAGIC_F, -TC_MAGIC_F));
}

NRC_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
NRC_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
NRC_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
NRC_DEV void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
NRC_DEV void tc_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
NRC_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Wait for this thread's tcgen05.ld, then pin the loaded registers behind the
// wait (empty volatile asm per register): no use of them moves above it.
template <int N>
NRC_DEV void tc_wait_ld_regs(uint32_t* r) {
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < N; i++) asm volatile("" : "+r"(r[i]));
}
NRC_DEV void tc_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
NRC_DEV void tc_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
// The same 32-bit value into 8 consecutive columns of this thread's lane.
NRC_DEV void tc_st8_fill(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
               : "memory");
}
// The same 32-bit value into 16 consecutive columns of this thread's lane.
NRC_DEV void tc_st16_fill(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
                   taddr),
               "r"(v)
               : "memory");
}
NRC_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed f32 pairs, one rounding per operation. The assembler still fuses a
// packed multiply that feeds a packed add or subtract into FFMA2, so these
// serve only where no product feeds a sum (product -> product, sum -> sum);
// a product that feeds a sum goes through the scalar __fmul_rn / __fadd_rn.
NRC_DEV uint64_t f2_bits(float2 v) { return (uint64_t)__float_as_uint(v.x) | ((uint64_t)__float_as_uint(v.y) << 32); }
NRC_DEV float2 bits_f2(uint64_t b) { return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32))); }
NRC_DEV float2 mul2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
NRC_DEV float2 add2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
NRC_DEV float2 sub2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}

// UMMA shared-memory descriptor, K-major, no swizzle: 8x16-byte core matrices,
// `lbo` = byte distance between the two 16-byte K halves, `sbo` = between
// consecutive 8-row groups; version 1 (sm_100).
NRC_DEV uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
  return a | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor: D s32, A/B signed int8, both K-major, N = ns, M = 128.
NRC_DEV uint32_t idesc_i8(int ns) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(ns >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}
NRC_DEV uint32_t canon_off(int r, int c) { return (uint32_t)((r & 7) * 16 + (r >> 3) * 256 + c * 128); }

}  // namespace nrc
