// sd_common.cuh -- sm_100a building blocks shared by the kernels of this library:
// mbarrier / bulk-TMA wrappers, FP8 conversions, and the page-block layout of the
// paged KV pool.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/specdec_b200.h"

#define SD_DEV __device__ __forceinline__

namespace sd {

constexpr int kPage = SPECDEC_PAGE_TOKENS;  // tokens per page
constexpr float kE4M3Max = 448.0f;           // model_self.py:300 E4M3_MAX

// ---------------------------------------------------------------- status word
SD_DEV void raise_status(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------- shared-memory addressing
SD_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
SD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
SD_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while its
// predecessor on the stream is still running.  grid_dep_wait() returns once that
// predecessor has completed and its memory is visible (a no-op for an ordinary
// launch); every read of device data another kernel produces, and every global
// write, comes after it.  grid_dep_launch() lets the successor start early; a CTA
// issues it only after its own grid_dep_wait(), so a kernel that has started can
// rely on everything before its immediate predecessor having completed.
SD_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SD_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
SD_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

SD_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
SD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
SD_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// non-blocking probe of phase `parity` (test_wait never suspends the thread)
SD_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
SD_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for phase `parity` of `bar`.  Gives up after `limit_ns` of wall time
// (~1 s by default; checked every 256 polls) and returns false; callers then raise
// SPECDEC_STATUS_TIMEOUT and leave, so a lost arrival can never hang the GPU.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;
SD_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// warp-uniform bounded wait; returns false when any lane gave up
SD_DEV bool warp_wait(uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); }

// ---------------------------------------------------------------- bulk TMA (plain per-CTA loads)
// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// src/dst 16-byte aligned, bytes a multiple of 16.
SD_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// L2 policy for data read once per call (the KV stream): its lines are the first to go,
// so the small tensors around it (queries, page tables, plans, split partials) stay in L2.
SD_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// 3-D tiled tensor load with an L2 policy; c0 is the innermost (element) coordinate and
// must be a multiple of 16 bytes / element size (callers pass 0 or 64 bf16 elements).
SD_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2,
                        uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Four rows of a 2-D tensor map in one request (tile::gather4): rows r0 .. r3 starting
// at element x (the map's box is one row high), written to dst as four consecutive
// rows; completion is counted on the mbarrier; `policy` is the L2 policy of the reads.
SD_DEV void tma_gather4(void* dst, const CUtensorMap* map, int32_t x, int32_t r0, int32_t r1, int32_t r2, int32_t r3,
                        uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}
SD_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- thread-block clusters
// Rank of this CTA in its cluster, and the cluster's CTA count / index in the grid.
SD_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
SD_DEV uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
SD_DEV uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Cluster-wide barrier: every thread of every CTA of the cluster arrives (release: its
// shared-memory writes become visible to the other CTAs) and waits (acquire).  All threads
// of the CTA execute it at the same program point.
SD_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync: arrive (release) early, wait (acquire) later.
SD_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
SD_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Address in CTA `rank`'s shared memory of the variable at this CTA's shared address `saddr`
// (distributed shared memory), and 16-byte / 4-byte loads from it.
SD_DEV uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
SD_DEV float4 dsmem_ld4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
SD_DEV float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ---------------------------------------------------------------- named barriers
SD_DEV void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- packing / conversion
SD_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (low 16 bits)
  return *reinterpret_cast<uint32_t*>(&v);
}
SD_DEV uint32_t pack_f16(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Two E4M3 codes (low byte = first element) -> f16x2 (low half = first element).
// Exact: every E4M3 value, subnormals included, is an f16 normal or zero.
SD_DEV uint32_t e4m3x2_to_f16x2(uint32_t two_codes) {
  uint32_t r;
  const uint16_t v = static_cast<uint16_t>(two_codes & 0xFFFFu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
// Round-to-nearest-even to E4M3 with saturation to +-448.  Returns the code of
// `first` in the low byte and `second` in the high byte.
SD_DEV uint32_t f32x2_to_e4m3x2(float first, float second) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(second), "f"(first));
  return r;
}
// Max of two magnitudes (>= 0 or NaN) that keeps a NaN, as torch's amax does (fmaxf drops it):
// a NaN anywhere in a V row makes the row's scale NaN, and with it every code of the row.
SD_DEV float amax_nan(float a, float b) { return (b > a || b != b) ? b : a; }
// Per-token E4M3 scale of quantize_kv_fp8: s = amax / 448 with IEEE division, 1 for an all-zero
// row; a NaN amax is passed through unchanged (the reference's division returns its NaN
// operand, the quiet NaN 0x7FC00000 of |NaN|, where the GPU's division would return its own
// canonical NaN pattern).
SD_DEV float e4m3_scale(float amax) {
  if (amax != amax) return amax;
  const float s = __fdiv_rn(amax, kE4M3Max);
  return s == 0.f ? 1.f : s;
}
SD_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
SD_DEV float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------- page-block layouts
// bf16 K (and bf16 V) page-head block: 16 tokens x D dims, stored as D/64
// half-tiles of [16 rows][128 bytes]; the 16-byte chunk j of row r is stored at
// chunk position j ^ (r & 7).  That is exactly what a TMA SWIZZLE_128B load of
// a {64, 16} box writes to a 1024-byte aligned shared buffer, so pool pages
// (one bulk copy) and contiguous tensors (tensor-map loads) give the same image.
// Byte offset of element (row r, dim d) inside the block:
SD_DEV uint32_t kblock_offset(int r, int d) {
  const int half = d >> 6;
  const int chunk = (d & 63) >> 3;
  return static_cast<uint32_t>(half * 2048 + r * 128 + ((chunk ^ (r & 7)) << 4) + ((d & 7) << 1));
}
// Byte offset of 16-byte chunk `c` (dims 8c..8c+7) of row r.
SD_DEV uint32_t kblock_chunk_offset(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * 2048 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
// E4M3 V page-head block: plain [16 tokens][D] code rows (token r, dim d at r * D + d).

}  // namespace sd
