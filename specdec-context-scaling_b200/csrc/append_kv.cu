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
  grid_dep_wait();  // launched programmatically: k/v and the lengths may be the preceding work's output
  grid_dep_launch();
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
  // the new K / V row is read while the page id is looked up (two independent round trips)
  const int64_t src = static_cast<int64_t>(p.row0[b] + i) * p.st + static_cast<int64_t>(h) * p.sh;
  const int d0 = lane * PER;
  uint2 k4 = make_uint2(0u, 0u), v4 = make_uint2(0u, 0u);
  if (PER == 4) {
    k4 = *reinterpret_cast<const uint2*>(p.k_new + src + d0);
    v4 = *reinterpret_cast<const uint2*>(p.v_new + src + d0);
  } else {
    k4.x = *reinterpret_cast<const uint32_t*>(p.k_new + src + d0);
    v4.x = *reinterpret_cast<const uint32_t*>(p.v_new + src + d0);
  }
  const int page = p.page_table[static_cast<int64_t>(b) * p.max_pages + blk];
  if (page < 0 || page >= p.num_pages) {
    if (lane == 0) raise_status(p.status, SPECDEC_STATUS_BAD_PAGE);
    return;
  }
  const int64_t ph = static_cast<int64_t>(page) * p.KV + h;

  // ---- K: bf16 copy into the swizzled block
  {
    uint8_t* kblk = p.k_pool + ph * (D * 32);
    if (PER == 4) {
      *reinterpret_cast<uint2*>(kblk + kblock_offset(slot, d0)) = k4;
    } else {
      *reinterpret_cast<uint32_t*>(kblk + kblock_offset(slot, d0)) = k4.x;
    }
  }
  // ---- V
  if (!VF8) {
    uint8_t* vblk = p.v_pool + ph * (D * 32);
    if (PER == 4) {
      *reinterpret_cast<uint2*>(vblk + kblock_offset(slot, d0)) = v4;
    } else {
      *reinterpret_cast<uint32_t*>(vblk + kblock_offset(slot, d0)) = v4.x;
    }
  } else {
    float x[PER];
    const __nv_bfloat16* vh = reinterpret_cast<const __nv_bfloat16*>(&v4);
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = __bfloat162float(vh[e]);
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) m = amax_nan(m, fabsf(x[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = amax_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = e4m3_scale(m);
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

// ---------------------------------------------------------------- fused RoPE + append
// One launch after the fused QKV projection of a step (rows x (H + 2 KV) x D bf16):
// warps 0 .. rows*H-1 rotate one query head row each into q_out (rows, H, D);
// the following warps take one (sequence, new token, KV head) each, rotate its K
// row, and append K and V (E4M3-quantised when the pool is) like append_kernel.
// Rotation: y = bf16(bf16(x cos) + bf16(rotate_half(x) sin)), cos/sin (rows, D)
// at each packed row's position.  Lane l holds dims PER*l ..; the rotate-half
// partner of those dims is held by lane l ^ 16.
struct RopeAppendParams {
  const __nv_bfloat16* qkv;
  int64_t qkv_st;
  const __nv_bfloat16* cs;
  const __nv_bfloat16* sn;
  __nv_bfloat16* q_out;
  int32_t rows, H;
  AppendParams a;
};

template <int PER>
SD_DEV void rope_lane(const __nv_bfloat16* src, const __nv_bfloat16* cs, const __nv_bfloat16* sn, int lane,
                      float (&y)[PER]) {
  const int d0 = lane * PER;
  float x[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) x[e] = __bfloat162float(src[d0 + e]);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const float rot = lane < 16 ? -other : other;
    const float a = __bfloat162float(__float2bfloat16_rn(x[e] * __bfloat162float(cs[d0 + e])));
    const float c = __bfloat162float(__float2bfloat16_rn(rot * __bfloat162float(sn[d0 + e])));
    y[e] = __bfloat162float(__float2bfloat16_rn(a + c));
  }
}

template <int D, bool VF8>
__global__ void __launch_bounds__(256) rope_append_kernel(const RopeAppendParams rp) {
  constexpr int PER = D / 32;
  grid_dep_wait();  // launched programmatically: qkv is the preceding work's output
  grid_dep_launch();
  const AppendParams& p = rp.a;
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nq = rp.rows * rp.H;
  if (warp_global < nq) {
    const int r = warp_global / rp.H, h = warp_global - r * rp.H;
    float y[PER];
    rope_lane<PER>(rp.qkv + static_cast<int64_t>(r) * rp.qkv_st + static_cast<int64_t>(h) * D,
                   rp.cs + static_cast<int64_t>(r) * D, rp.sn + static_cast<int64_t>(r) * D, lane, y);
    __nv_bfloat16* dst = rp.q_out + (static_cast<int64_t>(r) * rp.H + h) * D + lane * PER;
#pragma unroll
    for (int e = 0; e < PER; ++e) dst[e] = __float2bfloat16_rn(y[e]);
    return;
  }
  const int w = warp_global - nq;
  const int per_seq = p.max_new * p.KV;
  const int b = w / per_seq;
  if (b >= p.B) return;
  const int rem = w - b * per_seq;
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
  const int row = p.row0[b] + i;
  const __nv_bfloat16* src = rp.qkv + static_cast<int64_t>(row) * rp.qkv_st;
  const int d0 = lane * PER;
  // K: rotated, then the swizzled block
  {
    float y[PER];
    rope_lane<PER>(src + static_cast<int64_t>(rp.H + h) * D, rp.cs + static_cast<int64_t>(row) * D,
                   rp.sn + static_cast<int64_t>(row) * D, lane, y);
    uint8_t* kblk = p.k_pool + ph * (D * 32);
    if (PER == 4) {
      uint2 kv;
      kv.x = pack_bf16(y[0], y[1]);
      kv.y = pack_bf16(y[2 % PER], y[3 % PER]);
      *reinterpret_cast<uint2*>(kblk + kblock_offset(slot, d0)) = kv;
    } else {
      *reinterpret_cast<uint32_t*>(kblk + kblock_offset(slot, d0)) = pack_bf16(y[0], y[1]);
    }
  }
  // V: as append_kernel
  const __nv_bfloat16* vsrc = src + static_cast<int64_t>(rp.H + p.KV + h) * D;
  if (!VF8) {
    uint8_t* vblk = p.v_pool + ph * (D * 32);
    if (PER == 4) {
      const uint2 vv = *reinterpret_cast<const uint2*>(vsrc + d0);
      *reinterpret_cast<uint2*>(vblk + kblock_offset(slot, d0)) = vv;
    } else {
      const uint32_t vv = *reinterpret_cast<const uint32_t*>(vsrc + d0);
      *reinterpret_cast<uint32_t*>(vblk + kblock_offset(slot, d0)) = vv;
    }
  } else {
    float x[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = __bfloat162float(vsrc[d0 + e]);
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) m = amax_nan(m, fabsf(x[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = amax_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = e4m3_scale(m);
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

// validation and parameters shared by the append entry points; `need_src`: the
// k_new / v_new rows and strides are read (plain append)
static int fill_append(const SpecdecAppendArgs* a, bool need_src, AppendParams& p) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  if ((need_src && (!a->k_new || !a->v_new)) || !a->row0 || !a->n_new || !a->pos0)
    return fail(SPECDEC_ERR_INVALID, "k_new, v_new, row0, n_new and pos0 must be set");
  if (!a->k_pool || !a->v_pool || !a->page_table) return fail(SPECDEC_ERR_INVALID, "pool pointers must be set");
  if (a->num_seqs <= 0 || a->max_new <= 0 || a->num_kv_heads <= 0)
    return fail(SPECDEC_ERR_INVALID, "num_seqs, max_new and num_kv_heads must be positive");
  if (a->head_dim != 64 && a->head_dim != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  const bool vf8 = a->v_dtype == SPECDEC_E4M3;
  if (!vf8 && a->v_dtype != SPECDEC_BF16) return fail(SPECDEC_ERR_UNSUPPORTED, "v_dtype must be BF16 or E4M3");
  if (vf8 && a->head_dim != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "E4M3 V needs head_dim 128");
  if (vf8 && !a->v_scale) return fail(SPECDEC_ERR_INVALID, "E4M3 V needs v_scale");
  if (need_src) {
    if ((a->stride_tok | a->stride_head) & 3)
      return fail(SPECDEC_ERR_INVALID, "strides must be multiples of 4 elements (8-byte vectors)");
    if ((reinterpret_cast<uintptr_t>(a->k_new) | reinterpret_cast<uintptr_t>(a->v_new)) & 7u)
      return fail(SPECDEC_ERR_INVALID, "k_new and v_new must be 8-byte aligned");
  }
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
  return SPECDEC_OK;
}

extern "C" int specdec_append_kv(const SpecdecAppendArgs* a, specdec_stream_t stream) {
  AppendParams p;
  if (int rc = fill_append(a, true, p)) return rc;
  const bool vf8 = a->v_dtype == SPECDEC_E4M3;
  const int64_t warps = static_cast<int64_t>(p.B) * p.max_new * p.KV;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return fail(SPECDEC_ERR_INVALID, "append batch too large");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto* kern = a->head_dim == 128 ? (vf8 ? append_kernel<128, true> : append_kernel<128, false>)
                                  : append_kernel<64, false>;
  return launch_pdl("append_kernel", kern, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, p);
}

extern "C" int specdec_rope_append(const SpecdecRopeAppendArgs* a, specdec_stream_t stream) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  RopeAppendParams rp;
  if (int rc = fill_append(&a->kv, false, rp.a)) return rc;
  if (!a->qkv || !a->cos || !a->sin || !a->q_out) return fail(SPECDEC_ERR_INVALID, "qkv, cos, sin and q_out must be set");
  if (a->rows < 0 || a->num_q_heads <= 0) return fail(SPECDEC_ERR_INVALID, "rows >= 0 and num_q_heads > 0 required");
  const int D = a->kv.head_dim;
  if (a->qkv_row_stride < static_cast<int64_t>(a->num_q_heads + 2 * a->kv.num_kv_heads) * D)
    return fail(SPECDEC_ERR_INVALID, "qkv rows must hold H + 2 KV heads of head_dim values");
  if ((a->qkv_row_stride & 3) || (reinterpret_cast<uintptr_t>(a->qkv) & 7u))
    return fail(SPECDEC_ERR_INVALID, "qkv must be 8-byte aligned with a row stride of 4-element multiples");
  rp.qkv = static_cast<const __nv_bfloat16*>(a->qkv);
  rp.qkv_st = a->qkv_row_stride;
  rp.cs = static_cast<const __nv_bfloat16*>(a->cos);
  rp.sn = static_cast<const __nv_bfloat16*>(a->sin);
  rp.q_out = static_cast<__nv_bfloat16*>(a->q_out);
  rp.rows = a->rows;
  rp.H = a->num_q_heads;
  const bool vf8 = a->kv.v_dtype == SPECDEC_E4M3;
  const int64_t warps = static_cast<int64_t>(rp.rows) * rp.H + static_cast<int64_t>(rp.a.B) * rp.a.max_new * rp.a.KV;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return fail(SPECDEC_ERR_INVALID, "batch too large");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto* kern = D == 128 ? (vf8 ? rope_append_kernel<128, true> : rope_append_kernel<128, false>)
                        : rope_append_kernel<64, false>;
  return launch_pdl("rope_append_kernel", kern, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, rp);
}
