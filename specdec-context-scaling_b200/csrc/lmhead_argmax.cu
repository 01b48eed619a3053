// lmhead_argmax.cu -- greedy next tokens straight from the hidden states: the tied LM
// head logits = x @ W^T (specdec/engine/model_self.py:857) fused with the argmax the
// SpecDec executors take over them (spec_dec.py:230-236, fast_spec_dec.py:246-249), so
// the (rows x vocab) logits are never written.
//
// Each logit is the fp32 tensor-core dot product rounded to bf16 -- the value the
// reference's bf16 GEMM stores -- and the argmax follows torch.argmax on those bf16
// values: NaN is the maximum, ties (-0 == +0 included) go to the lowest index.
//
// Work: units of (128 token rows) x (n_tile vocab rows), vocab-major, dealt round-robin
// to one persistent CTA per SM.  Per CTA (192 threads):
//   warp 4   producer: TMA loads of the unit's X tile [128 rows][64 dims] and W tile
//            [n_tile rows][64 dims] per 64-dim chunk of the hidden size (128-byte
//            swizzle, K-major) into a 4-deep ring;
//   warp 5   MMA issuer (one lane): D[128 x n_tile] (fp32, TMEM) += X . W^T with
//            tcgen05.mma kind::f16, M 128, N n_tile, K 16; two accumulators in TMEM
//            (512 columns) so a unit's epilogue overlaps the next unit's MMAs;
//   warps 0-3 epilogue: thread t owns token row t of the tile (TMEM lane t), reads its
//            n_tile logits, rounds each to bf16 and keeps the first maximum, then merges
//            it into the row's packed key with one 64-bit atomicMax:
//               key = order(bf16 value) << 32 | (0xffffffff - vocab index)
//            so the largest value and, among equal values, the lowest index wins.
// The last CTA to finish (ticket) turns the keys into indices and clears them, so the
// zeroed workspace stays reusable and the call can sit in a CUDA graph.
#include <cudaTypedefs.h>

#include "sd_common.cuh"
#include "sd_internal.h"
#include "umma.cuh"

namespace sd {

constexpr int kLmThreads = 192;
constexpr int kLmStages = 4;
constexpr int kLmXTile = 16384;                  // [128 rows][128 B]
constexpr int kLmWTileMax = 32768;               // [<= 256 rows][128 B]
constexpr int kLmStage = kLmXTile + kLmWTileMax;  // 48 KB
constexpr int kLmSmem = kLmStages * kLmStage + 1024;
constexpr int kLmMaxRows = 1 << 16;

struct LmParams {
  int32_t rows, hidden, vocab, n_tile, n_mb, units;
  unsigned long long* keys;  // [rows]
  int32_t* ticket;
  int32_t* argmax;
  float* max_value;
  int32_t* status;
};

// torch.argmax order of a bf16 value as a 16-bit unsigned key: NaN above everything,
// -0 equal to +0, otherwise the usual sign-magnitude to unsigned mapping.
SD_DEV uint32_t bf16_order_key(float logit) {
  const __nv_bfloat16 h = __float2bfloat16_rn(logit);
  uint32_t b = *reinterpret_cast<const uint16_t*>(&h);
  if ((b & 0x7F80u) == 0x7F80u && (b & 0x7Fu) != 0u) return 0xFFFFu;  // NaN
  if (b == 0x8000u) b = 0u;                                             // -0 -> +0
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}
// inverse of bf16_order_key (NaN keys give a NaN)
SD_DEV float bf16_from_key(uint32_t key) {
  if (key == 0xFFFFu) return __int_as_float(0x7FC00000);
  const uint32_t b = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
  return __uint_as_float(b << 16);
}

SD_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
SD_DEV uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__global__ void __launch_bounds__(kLmThreads, 1) lmhead_argmax_kernel(const LmParams p,
                                                                      const __grid_constant__ CUtensorMap xmap,
                                                                      const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kLmStages], empty[kLmStages], acc_full[2], acc_empty[2], fin_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort, s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kLmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(&fin_bar, 1);
    s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
  }
  if (warp == 5) {
    umma::tmem_alloc(&tmem_base, 512);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const int nk = p.hidden / 64;
  const uint32_t wbytes = static_cast<uint32_t>(p.n_tile) * 128u;

  if (warp == 4) {
    // ---- producer
    const uint64_t w_policy = l2_evict_first();  // every W tile is read by n_mb units at about the same time
    const uint64_t x_policy = l2_evict_last();   // X is read by every vocab tile
    int g = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < p.units && !stop; u += gridDim.x) {
      const int v = u / p.n_mb, m = u - v * p.n_mb;
      for (int k = 0; k < nk; ++k, ++g) {
        const int s = g % kLmStages;
        if (g >= kLmStages && !warp_wait(&empty[s], ((g / kLmStages) - 1) & 1)) {
          if (lane == 0) {
            raise_status(p.status, SPECDEC_STATUS_TIMEOUT);
            atomicExch(&s_abort, 1);
          }
          stop = true;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kLmStage;
          mbar_arrive_expect_tx(&full[s], kLmXTile + wbytes);
          tma_load_2d(st, &xmap, k * 64, m * 128, &full[s], x_policy);
          tma_load_2d(st + kLmXTile, &wmap, k * 64, v * p.n_tile, &full[s], w_policy);
        }
        __syncwarp();
      }
    }
    // let every copy land before the CTA retires (bounded)
    for (int u = max(0, g - kLmStages); u < g; ++u) (void)warp_wait(&full[u % kLmStages], (u / kLmStages) & 1);
  } else if (warp == 5) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma::idesc_f16(128, p.n_tile, true, true, false, false);
      int g = 0, ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++ui) {
        const int b = ui & 1;
        // accumulator b is free once the epilogue has read unit ui - 2
        if (ui >= 2 && !mbar_wait(&acc_empty[b], ((ui >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        umma::fence_after_sync();
        const uint32_t d = umma::taddr(tbase, 0, b * 256);
        for (int k = 0; k < nk; ++k, ++g) {
          const int s = g % kLmStages;
          if (!mbar_wait(&full[s], (g / kLmStages) & 1)) {
            ok = false;
            break;
          }
          umma::fence_after_sync();
          const uint32_t xa = smem_u32(smem + s * kLmStage), wa = xa + kLmXTile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma::mma_f16_ss(d, umma::desc_kmajor_sw128(xa + kk * 32), umma::desc_kmajor_sw128(wa + kk * 32), idesc,
                             k > 0 || kk > 0);
          umma::commit(&empty[s]);
        }
        if (!ok) break;
        umma::commit(&acc_full[b]);
      }
      if (!ok) {
        raise_status(p.status, SPECDEC_STATUS_TIMEOUT);
        atomicExch(&s_abort, 1);
      }
      umma::commit(&fin_bar);
      (void)mbar_wait(&fin_bar, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread (warp, lane) owns token row 32 warp + lane of each unit
    int ui = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++ui) {
      const int v = u / p.n_mb, m = u - v * p.n_mb;
      const int b = ui & 1;
      if (!warp_wait(&acc_full[b], (ui >> 1) & 1)) {
        if (lane == 0) {
          raise_status(p.status, SPECDEC_STATUS_TIMEOUT);
          atomicExch(&s_abort, 1);
        }
        break;
      }
      umma::fence_after_sync();
      const int row = m * 128 + warp * 32 + lane;
      const int col0 = v * p.n_tile;
      const int ncols = min(p.n_tile, p.vocab - col0);
      uint32_t best = 0;
      int best_i = 0;
#pragma unroll 1
      for (int c = 0; c < p.n_tile; c += 16) {
        float x[16];
        umma::tmem_ld16(umma::taddr(tbase, warp * 32, b * 256 + c), x);
        umma::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t key = bf16_order_key(x[i]);
          if (c + i < ncols && key > best) {
            best = key;
            best_i = col0 + c + i;
          }
        }
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (row < p.rows && best != 0)
        atomicMax(p.keys + row, (static_cast<unsigned long long>(best) << 32) |
                                    static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(best_i)));
    }
    __threadfence();  // this thread's key updates before the CTA's ticket
  }

  umma::fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tbase, 512);
  }
  // the last CTA turns the packed keys into indices and clears them for the next call
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(p.ticket, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int r = tid; r < p.rows; r += blockDim.x) {
    const unsigned long long key = __ldcg(p.keys + r);
    p.argmax[r] = key ? static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key)) : -1;
    if (p.max_value) p.max_value[r] = key ? bf16_from_key(static_cast<uint32_t>(key >> 32)) : -INFINITY;
    p.keys[r] = 0ull;
  }
  if (tid == 0) *p.ticket = 0;
}

static int encode_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_outer) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) != cudaSuccess ||
        qres != cudaDriverEntryPointSuccess)
      return fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPECDEC_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SPECDEC_OK;
}

// Vocab rows per unit: the multiple of 16 in [128, 256] whose round-robin deal over the
// grid gives the CTAs the fewest vocab rows each (so the last wave is nearly full).
static int pick_n_tile(int vocab, int n_mb, int grid) {
  int best_n = 256;
  long long best = -1;
  for (int n = 256; n >= 128; n -= 16) {
    const long long units = static_cast<long long>((vocab + n - 1) / n) * n_mb;
    const long long per_cta = (units + grid - 1) / grid * n;
    if (best < 0 || per_cta < best) {
      best = per_cta;
      best_n = n;
    }
  }
  return best_n;
}

}  // namespace sd

using namespace sd;

extern "C" size_t specdec_lmhead_workspace_bytes(int32_t rows) {
  if (rows <= 0 || rows > kLmMaxRows) return 0;
  return align_up(sizeof(unsigned long long) * static_cast<size_t>(rows), 256) + 256;
}

extern "C" int specdec_lmhead_argmax(const SpecdecLmHeadArgs* a, specdec_stream_t stream) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  if (!a->x || !a->w || !a->argmax || !a->workspace) return fail(SPECDEC_ERR_INVALID, "x, w, argmax and workspace must be set");
  if (a->rows <= 0 || a->rows > kLmMaxRows) return fail(SPECDEC_ERR_INVALID, "rows must be in 1 .. %d", kLmMaxRows);
  if (a->hidden <= 0 || a->hidden % 64) return fail(SPECDEC_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  if (a->vocab <= 0) return fail(SPECDEC_ERR_INVALID, "vocab must be positive");
  if (a->x_stride < a->hidden || (a->x_stride * 2) % 16)
    return fail(SPECDEC_ERR_INVALID, "x row stride must cover hidden and be a multiple of 8 elements");
  if ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->w)) & 15u)
    return fail(SPECDEC_ERR_INVALID, "x and w must be 16-byte aligned");
  if (a->workspace_bytes < specdec_lmhead_workspace_bytes(a->rows))
    return fail(SPECDEC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required", a->workspace_bytes,
                specdec_lmhead_workspace_bytes(a->rows));
  if (reinterpret_cast<uintptr_t>(a->workspace) & 255u) return fail(SPECDEC_ERR_INVALID, "workspace must be 256-byte aligned");
  const int sms = (a->num_sms > 0 && a->num_sms < device_sm_count()) ? a->num_sms : device_sm_count();
  LmParams p;
  p.rows = a->rows;
  p.hidden = a->hidden;
  p.vocab = a->vocab;
  p.n_mb = (a->rows + 127) / 128;
  p.n_tile = pick_n_tile(a->vocab, p.n_mb, sms);
  p.units = ((a->vocab + p.n_tile - 1) / p.n_tile) * p.n_mb;
  p.keys = static_cast<unsigned long long*>(a->workspace);
  p.ticket = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(a->workspace) +
                                        align_up(sizeof(unsigned long long) * static_cast<size_t>(a->rows), 256));
  p.argmax = a->argmax;
  p.max_value = a->max_value;
  p.status = a->status;
  CUtensorMap xmap, wmap;
  if (int rc = encode_2d(&xmap, a->x, static_cast<uint64_t>(a->hidden), static_cast<uint64_t>(a->rows),
                         static_cast<uint64_t>(a->x_stride) * 2, 64, 128))
    return rc;
  if (int rc = encode_2d(&wmap, a->w, static_cast<uint64_t>(a->hidden), static_cast<uint64_t>(a->vocab),
                         static_cast<uint64_t>(a->hidden) * 2, 64, static_cast<uint32_t>(p.n_tile)))
    return rc;
  static bool attr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!attr[dev]) {
    cudaFuncSetAttribute(lmhead_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLmSmem);
    attr[dev] = true;
  }
  const int grid = std::min(sms, p.units);
  lmhead_argmax_kernel<<<grid, kLmThreads, kLmSmem, reinterpret_cast<cudaStream_t>(stream)>>>(p, xmap, wmap);
  return after_launch("lmhead_argmax_kernel");
}
