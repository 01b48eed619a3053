// accept_trim.cu -- device-side greedy accept and cache rollback, no host sync.
//
// Greedy accept follows the vectorised form of the reference executor
// (experiments/execution_optimization/fast_spec_dec.py:246-256):
//     g = argmax(rows, -1);  m = cumprod(g[:kp] == cands[:kp]).sum()
// and the rollback trims the cache to the accepted prefix
// (spec_dec.py:235-250, spec_cache.trim_cache semantics).
//
// argmax over a 151936-wide bf16 row is split into chunks; each CTA reduces one
// (row, chunk) to (value, index), the last CTA of a row (atomic ticket)
// reduces the row, and the last row of a sequence runs the prefix scan and
// writes m, the next token and the rolled-back length.  Tickets are reset by
// their last user, so the zero-initialised workspace stays reusable and the
// whole step can sit in a CUDA graph.
#include <math.h>
#include <string.h>

#include "sd_common.cuh"
#include "sd_internal.h"

namespace sd {

constexpr int kArgmaxThreads = 256;
constexpr int kChunkElems = 8192;
constexpr int kMaxChunks = 64;

struct AcceptParams {
  const void* logits;
  int32_t f32;
  int64_t row_stride;
  int32_t vocab, chunks, chunk_elems;
  const int32_t* row0;
  const int32_t* n_rows;
  const int32_t* cands;
  const int32_t* kp;
  int32_t B, max_rows, max_cands;
  int32_t* g;
  int32_t* m;
  int32_t* next_token;
  const int32_t* len_before;
  int32_t* len_after;
  int32_t keep_offset;
  float* part_val;    // [B*max_rows][chunks]
  int32_t* part_idx;  // [B*max_rows][chunks]
  int32_t* row_ticket;  // [B*max_rows]
  int32_t* seq_ticket;  // [B]
  int32_t* status;
};

// torch.argmax order: NaN is the maximum, ties go to the lower index.
SD_DEV bool beats(float v, int i, float bv, int bi) {
  const bool vn = isnan(v), bn = isnan(bv);
  if (vn || bn) return (vn && bn) ? (i < bi) : vn;
  if (v != bv) return v > bv;
  return i < bi;
}

SD_DEV void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (beats(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

// Block-wide argmax; the result is valid in thread 0.
SD_DEV void block_argmax(float& v, int& i) {
  __shared__ float s_v[kArgmaxThreads / 32];
  __shared__ int s_i[kArgmaxThreads / 32];
  warp_argmax(v, i);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = v;
    s_i[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    v = lane < kArgmaxThreads / 32 ? s_v[lane] : -INFINITY;
    i = lane < kArgmaxThreads / 32 ? s_i[lane] : 0x7fffffff;
    warp_argmax(v, i);
  }
}

__global__ void __launch_bounds__(kArgmaxThreads) accept_kernel(const AcceptParams p) {
  const int chunk = blockIdx.x;
  const int rowid = blockIdx.y;  // b * max_rows + j
  const int b = rowid / p.max_rows, j = rowid - b * p.max_rows;
  const int nrows = p.n_rows[b];
  if (nrows < 0 || nrows > p.max_rows) {
    if (chunk == 0 && j == 0 && threadIdx.x == 0) raise_status(p.status, SPECDEC_STATUS_ACCEPT_RANGE);
    return;
  }
  if (nrows == 0) {  // inactive sequence
    if (chunk == 0 && j == 0 && threadIdx.x == 0) {
      p.m[b] = 0;
      p.next_token[b] = -1;
      if (p.len_after) p.len_after[b] = p.len_before ? p.len_before[b] : 0;
    }
    return;
  }
  if (j >= nrows) return;

  // ---- chunk argmax
  const int64_t rbase = static_cast<int64_t>(p.row0[b] + j) * p.row_stride;
  const int c0 = chunk * p.chunk_elems;
  const int c1 = min(p.vocab, c0 + p.chunk_elems);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if (p.f32) {
    const float* row = static_cast<const float*>(p.logits) + rbase;
    for (int x = c0 + threadIdx.x; x < c1; x += kArgmaxThreads) {
      const float v = row[x];
      if (beats(v, x, bv, bi)) {
        bv = v;
        bi = x;
      }
    }
  } else {
    const __nv_bfloat16* row = static_cast<const __nv_bfloat16*>(p.logits) + rbase;
    const bool vec = ((reinterpret_cast<uintptr_t>(row + c0) & 15u) == 0) && ((c1 - c0) % 8 == 0);
    if (vec) {
      for (int x = c0 + threadIdx.x * 8; x < c1; x += kArgmaxThreads * 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + x);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float v = __bfloat162float(e[t]);
          if (beats(v, x + t, bv, bi)) {
            bv = v;
            bi = x + t;
          }
        }
      }
    } else {
      for (int x = c0 + threadIdx.x; x < c1; x += kArgmaxThreads) {
        const float v = __bfloat162float(row[x]);
        if (beats(v, x, bv, bi)) {
          bv = v;
          bi = x;
        }
      }
    }
  }
  block_argmax(bv, bi);
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    p.part_val[static_cast<int64_t>(rowid) * p.chunks + chunk] = bv;
    p.part_idx[static_cast<int64_t>(rowid) * p.chunks + chunk] = bi;
    __threadfence();
    const int t = atomicAdd(p.row_ticket + rowid, 1);
    s_last = (t == p.chunks - 1);
  }
  __syncthreads();
  if (!s_last) return;

  // ---- last chunk of this row: reduce the row
  __threadfence();
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int c = threadIdx.x; c < p.chunks; c += kArgmaxThreads) {
    const float cv = *reinterpret_cast<volatile float*>(p.part_val + static_cast<int64_t>(rowid) * p.chunks + c);
    const int ci = *reinterpret_cast<volatile int*>(p.part_idx + static_cast<int64_t>(rowid) * p.chunks + c);
    if (beats(cv, ci, v, idx)) {
      v = cv;
      idx = ci;
    }
  }
  __syncthreads();
  block_argmax(v, idx);
  if (threadIdx.x == 0) {
    p.g[static_cast<int64_t>(b) * p.max_rows + j] = idx;
    p.row_ticket[rowid] = 0;  // reset for the next launch
    __threadfence();
    const int t = atomicAdd(p.seq_ticket + b, 1);
    s_last = (t == nrows - 1);
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;

  // ---- last row of this sequence: accept scan + rollback length
  __threadfence();
  p.seq_ticket[b] = 0;
  const volatile int32_t* gb = p.g + static_cast<int64_t>(b) * p.max_rows;
  const int kp = p.kp[b];
  int mm = 0;
  if (kp < 0 || kp > p.max_cands || kp > nrows) {
    raise_status(p.status, SPECDEC_STATUS_ACCEPT_RANGE);
  } else {
    const int32_t* cb = p.cands + static_cast<int64_t>(b) * p.max_cands;
    while (mm < kp && gb[mm] == cb[mm]) ++mm;
  }
  p.m[b] = mm;
  p.next_token[b] = (mm < nrows) ? gb[mm] : -1;
  if (p.len_after) p.len_after[b] = (p.len_before ? p.len_before[b] : 0) + p.keep_offset + mm;
}

// Accept from argmaxes computed beforehand (g[b][j], e.g. by the fused LM-head argmax):
// one thread per sequence runs the first-mismatch scan of accept_kernel's last step.
__global__ void accept_scan_kernel(const AcceptParams p) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.B) return;
  const int nrows = p.n_rows[b];
  if (nrows < 0 || nrows > p.max_rows) {
    raise_status(p.status, SPECDEC_STATUS_ACCEPT_RANGE);
    return;
  }
  if (nrows == 0) {  // inactive sequence
    p.m[b] = 0;
    p.next_token[b] = -1;
    if (p.len_after) p.len_after[b] = p.len_before ? p.len_before[b] : 0;
    return;
  }
  const int32_t* gb = p.g + static_cast<int64_t>(b) * p.max_rows;
  const int kp = p.kp[b];
  int mm = 0;
  if (kp < 0 || kp > p.max_cands || kp > nrows) {
    raise_status(p.status, SPECDEC_STATUS_ACCEPT_RANGE);
  } else {
    const int32_t* cb = p.cands + static_cast<int64_t>(b) * p.max_cands;
    while (mm < kp && gb[mm] == cb[mm]) ++mm;
  }
  p.m[b] = mm;
  p.next_token[b] = (mm < nrows) ? gb[mm] : -1;
  if (p.len_after) p.len_after[b] = (p.len_before ? p.len_before[b] : 0) + p.keep_offset + mm;
}

__global__ void trim_kernel(const int32_t* __restrict__ cur, const int32_t* __restrict__ req,
                            int32_t* __restrict__ out, int B, int32_t* status) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int c = cur[b], n = req[b];
  if (n <= 0 || n > c) {
    raise_status(status, SPECDEC_STATUS_TRIM_RANGE);
    out[b] = c;
  } else {
    out[b] = n;
  }
}

static int chunks_for(int vocab) {
  int c = (vocab + kChunkElems - 1) / kChunkElems;
  return c < 1 ? 1 : (c > kMaxChunks ? kMaxChunks : c);
}

struct AcceptWs {
  size_t val, idx, rt, st, total;
};
static AcceptWs accept_ws(int B, int max_rows, int chunks) {
  AcceptWs w;
  const size_t rows = static_cast<size_t>(B) * max_rows;
  w.val = 0;
  w.idx = align_up(w.val + rows * chunks * sizeof(float), 256);
  w.rt = align_up(w.idx + rows * chunks * sizeof(int32_t), 256);
  w.st = align_up(w.rt + rows * sizeof(int32_t), 256);
  w.total = align_up(w.st + static_cast<size_t>(B) * sizeof(int32_t), 256);
  return w;
}

}  // namespace sd

using namespace sd;

extern "C" size_t specdec_accept_workspace_bytes(int32_t num_seqs, int32_t max_rows, int32_t vocab) {
  if (num_seqs <= 0 || max_rows <= 0 || vocab <= 0) return 0;
  return accept_ws(num_seqs, max_rows, chunks_for(vocab)).total;
}

extern "C" int specdec_greedy_accept(const SpecdecAcceptArgs* a, specdec_stream_t stream) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  if (!a->logits) {
    // the argmaxes are given in g: only the scan
    if (!a->n_rows || !a->cands || !a->kp || !a->g || !a->m || !a->next_token)
      return fail(SPECDEC_ERR_INVALID, "n_rows, cands, kp, g, m and next_token must be set");
    if (a->num_seqs <= 0 || a->max_rows <= 0 || a->max_cands <= 0)
      return fail(SPECDEC_ERR_INVALID, "num_seqs, max_rows and max_cands must be positive");
    AcceptParams p;
    memset(&p, 0, sizeof(p));
    p.n_rows = a->n_rows;
    p.cands = a->cands;
    p.kp = a->kp;
    p.B = a->num_seqs;
    p.max_rows = a->max_rows;
    p.max_cands = a->max_cands;
    p.g = a->g;
    p.m = a->m;
    p.next_token = a->next_token;
    p.len_before = a->len_before;
    p.len_after = a->len_after;
    p.keep_offset = a->keep_offset;
    p.status = a->status;
    accept_scan_kernel<<<(a->num_seqs + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return after_launch("accept_scan_kernel");
  }
  if (!a->row0 || !a->n_rows || !a->cands || !a->kp || !a->g || !a->m || !a->next_token)
    return fail(SPECDEC_ERR_INVALID, "logits, row0, n_rows, cands, kp, g, m and next_token must be set");
  if (a->num_seqs <= 0 || a->max_rows <= 0 || a->max_cands <= 0 || a->vocab <= 0)
    return fail(SPECDEC_ERR_INVALID, "num_seqs, max_rows, max_cands and vocab must be positive");
  if (a->logits_dtype != SPECDEC_BF16 && a->logits_dtype != SPECDEC_F32)
    return fail(SPECDEC_ERR_UNSUPPORTED, "logits must be bf16 or f32");
  if (a->row_stride < a->vocab) return fail(SPECDEC_ERR_INVALID, "row_stride is smaller than vocab");
  if (static_cast<int64_t>(a->num_seqs) * a->max_rows > 65535)
    return fail(SPECDEC_ERR_UNSUPPORTED, "num_seqs * max_rows must be <= 65535");
  const int chunks = chunks_for(a->vocab);
  const AcceptWs w = accept_ws(a->num_seqs, a->max_rows, chunks);
  if (!a->workspace || a->workspace_bytes < w.total)
    return fail(SPECDEC_ERR_WORKSPACE, "accept workspace of %zu bytes is smaller than %zu", a->workspace_bytes,
                w.total);
  AcceptParams p;
  p.logits = a->logits;
  p.f32 = a->logits_dtype == SPECDEC_F32;
  p.row_stride = a->row_stride;
  p.vocab = a->vocab;
  p.chunks = chunks;
  p.chunk_elems = (a->vocab + chunks - 1) / chunks;
  p.chunk_elems = (p.chunk_elems + 7) / 8 * 8;
  p.row0 = a->row0;
  p.n_rows = a->n_rows;
  p.cands = a->cands;
  p.kp = a->kp;
  p.B = a->num_seqs;
  p.max_rows = a->max_rows;
  p.max_cands = a->max_cands;
  p.g = a->g;
  p.m = a->m;
  p.next_token = a->next_token;
  p.len_before = a->len_before;
  p.len_after = a->len_after;
  p.keep_offset = a->keep_offset;
  uint8_t* base = static_cast<uint8_t*>(a->workspace);
  p.part_val = reinterpret_cast<float*>(base + w.val);
  p.part_idx = reinterpret_cast<int32_t*>(base + w.idx);
  p.row_ticket = reinterpret_cast<int32_t*>(base + w.rt);
  p.seq_ticket = reinterpret_cast<int32_t*>(base + w.st);
  p.status = a->status;
  dim3 grid(chunks, a->num_seqs * a->max_rows);
  accept_kernel<<<grid, kArgmaxThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return after_launch("accept_kernel");
}

extern "C" int specdec_trim(const int32_t* cur_len, const int32_t* new_len, int32_t* len_out, int32_t num_seqs,
                            int32_t* status, specdec_stream_t stream) {
  if (!cur_len || !new_len || !len_out) return fail(SPECDEC_ERR_INVALID, "length arrays must be set");
  if (num_seqs <= 0) return fail(SPECDEC_ERR_INVALID, "num_seqs must be positive");
  trim_kernel<<<(num_seqs + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(cur_len, new_len, len_out,
                                                                                          num_seqs, status);
  return after_launch("trim_kernel");
}
