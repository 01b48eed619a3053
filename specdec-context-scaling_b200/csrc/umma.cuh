// umma.cuh -- sm_100a fifth-generation tensor core (tcgen05) building blocks:
// shared-memory matrix descriptors, instruction descriptors, MMA issue/commit,
// tensor-memory (TMEM) allocation and 32x32b loads/stores.  Encodings follow the
// PTX ISA for tcgen05 (and the field layout CUTLASS's cute/arch/mma_sm100_desc.hpp
// documents).  Only cta_group::1, kind::f16 (bf16/f16 inputs, fp32 accumulate).
#pragma once

#include <stdint.h>

#include "sd_common.cuh"

namespace sd {
namespace umma {

// ---------------------------------------------------------------- descriptors
enum Layout : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

// Shared-memory matrix descriptor: start address, leading / stride byte offsets
// (all in bytes, multiples of 16), fixed version 1, base offset 0 (1024-byte
// aligned swizzle atoms), swizzle layout.
SD_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// K-major operand in 128-byte swizzle atoms (8 rows x 128 B): rows 128 B apart,
// 8-row groups `sbo` apart.  One descriptor covers one K=16 (32-byte) slice;
// successive slices inside the 128-byte row advance the start address by 32 B.
SD_DEV uint64_t desc_kmajor_sw128(uint32_t saddr, uint32_t sbo_bytes = 1024) {
  return smem_desc(saddr, 16, sbo_bytes, kSwizzle128B);
}
// MN-major operand in 128-byte swizzle atoms (8 K-rows x 64 MN-elements of 16 bit):
// `lbo` = distance between 64-element MN groups, `sbo` = distance between 8-row K groups.
SD_DEV uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes = 1024) {
  return smem_desc(saddr, lbo_bytes, sbo_bytes, kSwizzle128B);
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
// a_bf16/b_bf16: operand type bf16 (else f16); a_mn/b_mn: MN-major operand (else K-major).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_bf16, bool b_bf16, bool a_mn, bool b_mn) {
  return (1u << 4)                                  // D format: f32
         | ((a_bf16 ? 1u : 0u) << 7)                // A format
         | ((b_bf16 ? 1u : 0u) << 10)               // B format
         | ((a_mn ? 1u : 0u) << 15)                 // A major
         | ((b_mn ? 1u : 0u) << 16)                 // B major
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------- MMA issue (one thread)
// D[tmem] (+)= A[smem] * B[smem]^T ; accumulate = false overwrites D.
SD_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t no_mask = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(no_mask), "r"(no_mask), "r"(no_mask), "r"(no_mask)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 operation this thread issued so far has completed.
SD_DEV void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- fences
SD_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SD_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------- TMEM allocation (one full warp)
SD_DEV void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
SD_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
SD_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// TMEM address: lane in bits 31..16, column in bits 15..0.
SD_DEV uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) { return base + (lane << 16) + col; }

// ---------------------------------------------------------------- TMEM <-> registers (warp-wide)
// Warp w (w % 4 == q) may only touch lanes 32q .. 32q+31.  32x32b.xN: thread t
// gets lane (32q + t), columns col .. col+N-1.
SD_DEV void tmem_ld16(uint32_t ta, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(ta));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
SD_DEV void tmem_ld8(uint32_t ta, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(ta));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
SD_DEV void tmem_st16(uint32_t ta, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          ta),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
SD_DEV void tmem_st8(uint32_t ta, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(ta),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
SD_DEV void tmem_ld4(uint32_t ta, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(ta));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
SD_DEV void tmem_st4(uint32_t ta, const float (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ta), "r"(__float_as_uint(v[0])),
               "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3]))
               : "memory");
}
// N consecutive columns (N = 4, 8, 16 or 32) of this thread's lane
template <int N>
SD_DEV void tmem_ldn(uint32_t ta, float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 16 || N == 32, "4, 8, 16 or 32 columns");
  if constexpr (N == 32) {
    tmem_ld16(ta, reinterpret_cast<float(&)[16]>(v[0]));
    tmem_ld16(ta + 16, reinterpret_cast<float(&)[16]>(v[16]));
  } else if constexpr (N == 16) {
    tmem_ld16(ta, v);
  } else if constexpr (N == 8) {
    tmem_ld8(ta, v);
  } else {
    tmem_ld4(ta, v);
  }
}
template <int N>
SD_DEV void tmem_stn(uint32_t ta, const float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 16 || N == 32, "4, 8, 16 or 32 columns");
  if constexpr (N == 32) {
    tmem_st16(ta, reinterpret_cast<const float(&)[16]>(v[0]));
    tmem_st16(ta + 16, reinterpret_cast<const float(&)[16]>(v[16]));
  } else if constexpr (N == 16) {
    tmem_st16(ta, v);
  } else if constexpr (N == 8) {
    tmem_st8(ta, v);
  } else {
    tmem_st4(ta, v);
  }
}
SD_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SD_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace umma
}  // namespace sd
