// append_kv.cu -- write new K/V tokens into the paged pool; V is optionally
// quantised to E4M3 on the way in.
//
// Quantisation is the reference's V-only scheme, quantize_kv_fp8(v, GROUP_V=128)
// (specdec/engine/model_self.py:304-314): per token and KV head,
//     m = max |v|  (fp32),  s = m / 448  (IEEE division),  s = 1 if s == 0,
//     code = e4m3_rne(v / s)  (IEEE division per element).
// torch's float8_e4m3fn cast rounds to nearest even and turns |x| >= 464 into
// NaN, while cvt.rn.satfinite clamps to 448; |v / s| <= 448 * (1 + 2^-23), so
// the two agree on every input this computation can produce.  This TU is built
// without fast-math so the divisions stay correctly rounded.
//
// One warp per (sequence, new token, KV head); lanes own 4 (D=128) or 2 (D=64)
// consecutive dims.  The K row and a bf16 V row go to the swizzled page-block
// order; E4M3 codes go to plain [16 tokens][D] rows of the page block.
#include "sd_common.cuh"
#include "sd_internal.h"

namespace sd {

struct AppendParams {
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  int64_t st, sh;
  const int32_t* row0;
  const int32_t* n_new;
  const int32_t* pos0;
  int32_t* len_out;
  int32_t B, max_new;
  uint8_t* k_pool;
  uint8_t* v_pool;
  float* v_scale;
  const int32_t* page_table;
  int32_t num_pages, KV, max_pages;
  int32_t* status;
};

template <int D, bool VF8>
__global__ void __launch_bounds__(256) append_kernel(const AppendParams p) {
  constexpr int PER = D / 32;  // dims per lane
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int per_seq = p.max_new * p.KV;
  const int b = warp_global / per_seq;
  if (b >= p.B) return;
  const int rem = warp_global - b * per_seq;
  const int i = rem / p.KV;
  const int h = rem - i * p.KV;
  const int n = p.n_new[b];
  if (n < 0 || n > p.max_new) {
    if (i == 0 && h == 0 && lane == 0) raise_status(p.status, SPECDEC_STATUS_BAD_LENGTH);
    return;
  }
  const int pos_start = p.pos0[b];
  if (i == 0 && h == 0 && lane == 0 && p.len_out) p.len_out[b] = pos_start + n;
  if (i >= n) return;
  const int pos = pos_start + i;
  const int blk = pos / kPage, slot = pos - blk * kPage;
  if (pos < 0 || blk >= p.max_pages) {
    if (lane == 0) raise_status(p.status, SPECDEC_STATUS_PAGE_OVERFLOW);
    return;
  }
  const int page = p.page_table[static_cast<int64_t>(b) * p.max_pages + blk];
  if (page < 0 || page >= p.num_pages) {
    if (lane == 0) raise_status(p.status, SPECDEC_STATUS_BAD_PAGE);
    return;
  }
  const int64_t ph = static_cast<int64_t>(page) * p.KV + h;
  const int64_t src = static_cast<int64_t>(p.row0[b] + i) * p.st + static_cast<int64_t>(h) * p.sh;
  const int d0 = lane * PER;

  // ---- K: bf16 copy into the swizzled block
  {
    uint8_t* kblk = p.k_pool + ph * (D * 32);
    if (PER == 4) {
      const uint2 kv = *reinterpret_cast<const uint2*>(p.k_new + src + d0);
      *reinterpret_cast<uint2*>(kblk + kblock_offset(slot, d0)) = kv;
    } else {
      const uint32_t kv = *reinterpret_cast<const uint32_t*>(p.k_new + src + d0);
      *reinterpret_cast<uint32_t*>(kblk + kblock_offset(slot, d0)) = kv;
    }
  }
  // ---- V
  if (!VF8) {
    uint8_t* vblk = p.v_pool + ph * (D * 32);
    if (PER == 4) {
      const uint2 vv = *reinterpret_cast<const uint2*>(p.v_new + src + d0);
      *reinterpret_cast<uint2*>(vblk + kblock_offset(slot, d0)) = vv;
    } else {
      const uint32_t vv = *reinterpret_cast<const uint32_t*>(p.v_new + src + d0);
      *reinterpret_cast<uint32_t*>(vblk + kblock_offset(slot, d0)) = vv;
    }
  } else {
    float x[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = __bfloat162float(p.v_new[src + d0 + e]);
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) m = fmaxf(m, fabsf(x[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = __fdiv_rn(m, kE4M3Max);
    if (s == 0.f) s = 1.f;
    // natural [16 tokens][D] code rows: each lane writes its 4 codes as one word
    uint8_t* vrow = p.v_pool + ph * (D * 16) + slot * D;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < PER; e += 2) {
      const uint32_t two = f32x2_to_e4m3x2(__fdiv_rn(x[e], s), __fdiv_rn(x[e + 1], s));
      word |= two << (8 * e);
    }
    *reinterpret_cast<uint32_t*>(vrow + d0) = word;
    if (lane == 0) p.v_scale[ph * kPage + slot] = s;
  }
}

}  // namespace sd

using namespace sd;

extern "C" int specdec_append_kv(const SpecdecAppendArgs* a, specdec_stream_t stream) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  if (!a->k_new || !a->v_new || !a->row0 || !a->n_new || !a->pos0)
    return fail(SPECDEC_ERR_INVALID, "k_new, v_new, row0, n_new and pos0 must be set");
  if (!a->k_pool || !a->v_pool || !a->page_table) return fail(SPECDEC_ERR_INVALID, "pool pointers must be set");
  if (a->num_seqs <= 0 || a->max_new <= 0 || a->num_kv_heads <= 0)
    return fail(SPECDEC_ERR_INVALID, "num_seqs, max_new and num_kv_heads must be positive");
  if (a->head_dim != 64 && a->head_dim != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  const bool vf8 = a->v_dtype == SPECDEC_E4M3;
  if (!vf8 && a->v_dtype != SPECDEC_BF16) return fail(SPECDEC_ERR_UNSUPPORTED, "v_dtype must be BF16 or E4M3");
  if (vf8 && a->head_dim != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "E4M3 V needs head_dim 128");
  if (vf8 && !a->v_scale) return fail(SPECDEC_ERR_INVALID, "E4M3 V needs v_scale");
  if ((a->stride_tok | a->stride_head) & 3)
    return fail(SPECDEC_ERR_INVALID, "strides must be multiples of 4 elements (8-byte vectors)");
  if ((reinterpret_cast<uintptr_t>(a->k_new) | reinterpret_cast<uintptr_t>(a->v_new)) & 7u)
    return fail(SPECDEC_ERR_INVALID, "k_new and v_new must be 8-byte aligned");
  AppendParams p;
  p.k_new = static_cast<const __nv_bfloat16*>(a->k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(a->v_new);
  p.st = a->stride_tok;
  p.sh = a->stride_head;
  p.row0 = a->row0;
  p.n_new = a->n_new;
  p.pos0 = a->pos0;
  p.len_out = a->len_out;
  p.B = a->num_seqs;
  p.max_new = a->max_new;
  p.k_pool = static_cast<uint8_t*>(a->k_pool);
  p.v_pool = static_cast<uint8_t*>(a->v_pool);
  p.v_scale = a->v_scale;
  p.page_table = a->page_table;
  p.num_pages = a->num_pages;
  p.KV = a->num_kv_heads;
  p.max_pages = a->max_pages_per_seq;
  p.status = a->status;
  const int64_t warps = static_cast<int64_t>(p.B) * p.max_new * p.KV;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return fail(SPECDEC_ERR_INVALID, "append batch too large");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a->head_dim == 128) {
    if (vf8)
      append_kernel<128, true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    else
      append_kernel<128, false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  } else {
    append_kernel<64, false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  }
  return after_launch("append_kernel");
}
