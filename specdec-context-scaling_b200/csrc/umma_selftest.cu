// umma_selftest.cu -- device self-check of the tcgen05 operand layouts the attention
// kernel relies on.  One CTA of 4 warps stages four bf16 matrices in shared memory
// in 128-byte-swizzled atoms, runs
//   D1[128 x 32] = K[128 x 128] . Q[32 x 128]^T     (A and B K-major: the QK^T shape)
//   D2[128 x 32] = V[128 x 128]^T . P[32 x 128]^T   (A MN-major, B K-major: the PV shape)
// on the tensor cores with fp32 accumulation in TMEM, and writes both to global memory.
#include "sd_common.cuh"
#include "sd_internal.h"
#include "umma.cuh"

namespace sd {

// byte offset of element (row r, col c) of a [rows][128] bf16 matrix stored as two
// [rows][64] half regions of 128-byte-swizzled rows (half region = rows * 128 B)
SD_DEV uint32_t sw128_offset(int r, int c, int rows) {
  const int half = c >> 6, chunk = (c & 63) >> 3;
  return static_cast<uint32_t>(half * rows * 128 + r * 128 + ((chunk ^ (r & 7)) << 4) + ((c & 7) << 1));
}

__global__ void __launch_bounds__(128) umma_selftest_kernel(const __nv_bfloat16* __restrict__ k,
                                                            const __nv_bfloat16* __restrict__ q,
                                                            const __nv_bfloat16* __restrict__ v,
                                                            const __nv_bfloat16* __restrict__ p, float* out1,
                                                            float* out2, int32_t* status) {
  constexpr int N = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sk = smem;             // 128 x 128 -> 32 KB
  uint8_t* sv = smem + 32768;     // 32 KB
  uint8_t* sq = smem + 65536;     // 32 x 128 -> 8 KB
  uint8_t* sp = smem + 73728;     // 8 KB
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < 128 * 128; i += 128) {
    const int r = i >> 7, c = i & 127;
    *reinterpret_cast<__nv_bfloat16*>(sk + sw128_offset(r, c, 128)) = k[i];
    *reinterpret_cast<__nv_bfloat16*>(sv + sw128_offset(r, c, 128)) = v[i];
  }
  for (int i = tid; i < N * 128; i += 128) {
    const int r = i >> 7, c = i & 127;
    *reinterpret_cast<__nv_bfloat16*>(sq + sw128_offset(r, c, N)) = q[i];
    *reinterpret_cast<__nv_bfloat16*>(sp + sw128_offset(r, c, N)) = p[i];
  }
  if (warp == 0) {
    umma::tmem_alloc(&tmem_base, 64);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor-core (async) proxy
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = tmem_base;

  if (tid == 0) {
    const uint32_t id1 = umma::idesc_f16(128, N, true, true, false, false);
    const uint32_t id2 = umma::idesc_f16(128, N, true, true, true, false);
    const uint32_t k0 = smem_u32(sk), v0 = smem_u32(sv), q0 = smem_u32(sq), p0 = smem_u32(sp);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t a = umma::desc_kmajor_sw128(k0 + (kk >> 2) * 16384 + (kk & 3) * 32);
      const uint64_t b = umma::desc_kmajor_sw128(q0 + (kk >> 2) * (N * 128) + (kk & 3) * 32);
      umma::mma_f16_ss(umma::taddr(tbase, 0, 0), a, b, id1, kk > 0);
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t a = umma::desc_mnmajor_sw128(v0 + kk * 2048, 16384);
      const uint64_t b = umma::desc_kmajor_sw128(p0 + (kk >> 2) * (N * 128) + (kk & 3) * 32);
      umma::mma_f16_ss(umma::taddr(tbase, 0, N), a, b, id2, kk > 0);
    }
    umma::commit(&done);
  }
  const bool ok = mbar_wait(&done, 0);
  if (!ok && lane == 0) raise_status(status, SPECDEC_STATUS_TIMEOUT);
  umma::fence_after_sync();
  if (ok) {
    float r1[16], r2[16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      umma::tmem_ld16(umma::taddr(tbase, 32 * warp, 16 * h), r1);
      umma::tmem_ld16(umma::taddr(tbase, 32 * warp, N + 16 * h), r2);
      umma::tmem_wait_ld();
      const int row = 32 * warp + lane;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        out1[row * N + 16 * h + c] = r1[c];
        out2[row * N + 16 * h + c] = r2[c];
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tbase, 64);
  }
}

}  // namespace sd

using namespace sd;

extern "C" int specdec_umma_selftest(const void* k, const void* q, const void* v, const void* p, float* out1,
                                     float* out2, int32_t* status, specdec_stream_t stream) {
  if (!k || !q || !v || !p || !out1 || !out2) return fail(SPECDEC_ERR_INVALID, "selftest pointers must be set");
  // 80 KB are used; the rest keeps any misread stride inside this CTA's allocation
  const int smem = 160 * 1024;
  cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  umma_selftest_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(v), static_cast<const __nv_bfloat16*>(p), out1, out2, status);
  return after_launch("umma_selftest_kernel");
}
