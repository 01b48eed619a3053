// elementwise.cu -- RMSNorm, rotate-half RoPE and SwiGLU with the rounding of
// the eager engine formulas (specdec/kernels/reference.py:14-31):
//   rmsnorm: y = w * dtype(x * rsqrt(mean(x^2) + eps))   (fp32 statistics)
//   rope   : y = dtype(dtype(x * cos) + dtype(rotate_half(x) * sin))
//   swiglu : y = dtype(dtype(silu(g)) * u)
// bf16 rows are read and written with 16-byte vectors where the row allows it.
#include <math.h>

#include "sd_common.cuh"
#include "sd_internal.h"

namespace sd {

template <typename T>
SD_DEV float to_f(T v);
template <>
SD_DEV float to_f<float>(float v) {
  return v;
}
template <>
SD_DEV float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
SD_DEV T from_f(float v);
template <>
SD_DEV float from_f<float>(float v) {
  return v;
}
template <>
SD_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
// value rounded to T and widened back (models a torch op that stores in T)
template <typename T>
SD_DEV float round_to(float v) {
  return to_f<T>(from_f<T>(v));
}

// torch's CPU rsqrt: 1 / sqrt(x), both steps correctly rounded (rsqrtf is approximate)
SD_DEV float inv_sqrt_rn(float x) { return __fdiv_rn(1.f, __fsqrt_rn(x)); }

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                      T* __restrict__ y, int hidden, float eps) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * hidden;
  T* yr = y + row * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = to_f<T>(xr[i]);
    ss += v * v;
  }
  __shared__ float s_part[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  __shared__ float s_inv;
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < (blockDim.x >> 5); ++k) t += s_part[k];
    s_inv = inv_sqrt_rn(t / static_cast<float>(hidden) + eps);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float n = round_to<T>(to_f<T>(xr[i]) * inv);
    yr[i] = from_f<T>(to_f<T>(w[i]) * n);
  }
}

// bf16 rows of hidden % 8 == 0 (<= 4096): one warp per row, 16-byte vectors kept in
// registers between the sum of squares (fp32) and the scaling; no block-level sync.
template <int CH>
__global__ void __launch_bounds__(256) rmsnorm_warp_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           __nv_bfloat16* __restrict__ y, int64_t rows, int hidden,
                                                           float eps) {
  grid_dep_wait();  // launched programmatically: x is the preceding work's output
  grid_dep_launch();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nch = hidden / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * hidden);
  uint4 v[CH];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
      v[i] = xr[c];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(e[k]);
        ss += f * f;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = inv_sqrt_rn(ss / static_cast<float>(hidden) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * hidden);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
      const uint4 wv = wr[c];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float n = round_to<__nv_bfloat16>(__bfloat162float(e[k]) * inv);
        oe[k] = __float2bfloat16_rn(__bfloat162float(we[k]) * n);
      }
      yr[c] = o;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const T* __restrict__ x, int64_t sb, int64_t sh, int64_t ss,
                                                   const T* __restrict__ cs, const T* __restrict__ sn,
                                                   T* __restrict__ y, int H, int S, int D, int64_t n) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  const int d = static_cast<int>(idx % D);
  int64_t t = idx / D;
  const int s = static_cast<int>(t % S);
  t /= S;
  const int h = static_cast<int>(t % H);
  const int64_t b = t / H;
  const T* xr = x + b * sb + h * sh + s * ss;
  const int half = D / 2;
  const float xv = to_f<T>(xr[d]);
  const float rot = d < half ? -to_f<T>(xr[d + half]) : to_f<T>(xr[d - half]);
  // one rounding per torch op (x * cos, rotate_half(x) * sin, their sum): explicit IEEE
  // products and sum, so no fused multiply-add merges them for fp32
  const float a = round_to<T>(__fmul_rn(xv, to_f<T>(cs[s * D + d])));
  const float c = round_to<T>(__fmul_rn(rot, to_f<T>(sn[s * D + d])));
  y[idx] = from_f<T>(__fadd_rn(a, c));
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u,
                                                     T* __restrict__ y, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gv = to_f<T>(g[i]);
    const float silu = round_to<T>(gv / (1.f + expf(-gv)));
    y[i] = from_f<T>(silu * to_f<T>(u[i]));
  }
}

// SwiGLU of a fused gate|up projection: row r of `gu` holds gate (inter values) then
// up (inter values); 8 values per thread with 16-byte vectors (inter % 8 == 0).
__global__ void __launch_bounds__(256) swiglu_packed_kernel(const __nv_bfloat16* __restrict__ gu,
                                                            __nv_bfloat16* __restrict__ y, int64_t rows,
                                                            int64_t inter) {
  grid_dep_wait();  // launched programmatically: gu is the preceding work's output
  grid_dep_launch();
  const int64_t n8 = rows * (inter / 8);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / (inter / 8), c = (i - r * (inter / 8)) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 2 * inter + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter + c);
    const __nv_bfloat16* g8 = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* u8 = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 ov;
    __nv_bfloat16* o8 = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // silu with the hardware exp2 and reciprocal (relative error ~1e-6 before the bf16
      // rounding of the reference formula dtype(silu(g)) * u)
      const float g = __bfloat162float(g8[e]);
      const float silu = round_to<__nv_bfloat16>(g * __frcp_rn(1.f + __expf(-g)));
      o8[e] = __float2bfloat16_rn(silu * __bfloat162float(u8[e]));
    }
    *reinterpret_cast<uint4*>(y + r * inter + c) = ov;
  }
}

}  // namespace sd

using namespace sd;

extern "C" int specdec_swiglu_packed(const void* gate_up, void* out, int64_t rows, int64_t inter,
                                     specdec_stream_t stream) {
  if (!gate_up || !out) return fail(SPECDEC_ERR_INVALID, "tensors must be CUDA");
  if (rows < 0 || inter <= 0 || inter % 8 != 0) return fail(SPECDEC_ERR_INVALID, "rows >= 0 and inter % 8 == 0 required");
  if ((reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(SPECDEC_ERR_INVALID, "gate_up and out must be 16-byte aligned");
  const int64_t n8 = rows * (inter / 8);
  if (n8 == 0) return SPECDEC_OK;
  int64_t blocks = (n8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return launch_pdl("swiglu_packed_kernel", swiglu_packed_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                    reinterpret_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(gate_up),
                    static_cast<__nv_bfloat16*>(out), rows, inter);
}

extern "C" int specdec_rmsnorm(const void* x, const void* weight, void* out, int32_t dtype, int64_t rows,
                               int32_t hidden, float eps, specdec_stream_t stream) {
  if (!x || !weight || !out) return fail(SPECDEC_ERR_INVALID, "x must be CUDA");
  if (hidden <= 0) return fail(SPECDEC_ERR_INVALID, "empty hidden size");
  if (rows == 0) return SPECDEC_OK;
  if (rows < 0 || rows > 0x7fffffff) return fail(SPECDEC_ERR_INVALID, "row count out of range");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = dtype == SPECDEC_BF16 && hidden % 8 == 0 && hidden <= 4096 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight) |
                     reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  if (vec) {
    const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
    const int ch = (hidden / 8 + 31) / 32;  // 16-byte chunks per lane
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    const auto* wb = static_cast<const __nv_bfloat16*>(weight);
    auto* yb = static_cast<__nv_bfloat16*>(out);
    auto* kern = ch <= 1 ? rmsnorm_warp_kernel<1>
                 : ch <= 2 ? rmsnorm_warp_kernel<2>
                 : ch <= 4 ? rmsnorm_warp_kernel<4>
                 : ch <= 8 ? rmsnorm_warp_kernel<8>
                           : rmsnorm_warp_kernel<16>;
    return launch_pdl("rmsnorm_warp_kernel", kern, dim3(blocks), dim3(256), 0, st, xb, wb, yb, rows, hidden, eps);
  }
  if (dtype == SPECDEC_F32)
    rmsnorm_kernel<float><<<static_cast<unsigned>(rows), 256, 0, st>>>(
        static_cast<const float*>(x), static_cast<const float*>(weight), static_cast<float*>(out), hidden, eps);
  else if (dtype == SPECDEC_BF16)
    rmsnorm_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(out), hidden, eps);
  else
    return fail(SPECDEC_ERR_INVALID, "rmsnorm supports float32 and bfloat16");
  return after_launch("rmsnorm_kernel");
}

extern "C" int specdec_apply_rope(const void* x, int64_t stride_b, int64_t stride_h, int64_t stride_s,
                                  const void* cos, const void* sin, void* out, int32_t dtype, int32_t B, int32_t H,
                                  int32_t S, int32_t D, specdec_stream_t stream) {
  if (!x || !cos || !sin || !out) return fail(SPECDEC_ERR_INVALID, "tensors must be CUDA");
  if (D % 2 != 0) return fail(SPECDEC_ERR_INVALID, "head_dim must be even");
  const int64_t n = static_cast<int64_t>(B) * H * S * D;
  if (n == 0) return SPECDEC_OK;
  if (B < 0 || H < 0 || S < 0 || D < 0) return fail(SPECDEC_ERR_INVALID, "negative shape");
  const int64_t blocks = (n + 255) / 256;
  if (blocks > 0x7fffffff) return fail(SPECDEC_ERR_INVALID, "tensor too large");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPECDEC_F32)
    rope_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const float*>(x), stride_b, stride_h, stride_s, static_cast<const float*>(cos),
        static_cast<const float*>(sin), static_cast<float*>(out), H, S, D, n);
  else if (dtype == SPECDEC_BF16)
    rope_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), stride_b, stride_h, stride_s, static_cast<const __nv_bfloat16*>(cos),
        static_cast<const __nv_bfloat16*>(sin), static_cast<__nv_bfloat16*>(out), H, S, D, n);
  else
    return fail(SPECDEC_ERR_INVALID, "rope supports float32 and bfloat16");
  return after_launch("rope_kernel");
}

extern "C" int specdec_swiglu(const void* gate, const void* up, void* out, int32_t dtype, int64_t n,
                              specdec_stream_t stream) {
  if (!gate || !up || !out) return fail(SPECDEC_ERR_INVALID, "tensors must be CUDA");
  if (n == 0) return SPECDEC_OK;
  if (n < 0) return fail(SPECDEC_ERR_INVALID, "negative size");
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPECDEC_F32)
    swiglu_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const float*>(gate), static_cast<const float*>(up), static_cast<float*>(out), n);
  else if (dtype == SPECDEC_BF16)
    swiglu_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
        static_cast<__nv_bfloat16*>(out), n);
  else
    return fail(SPECDEC_ERR_INVALID, "swiglu supports float32 and bfloat16");
  return after_launch("swiglu_kernel");
}
