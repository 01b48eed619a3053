/*
 * specdec_b200.h -- C ABI of the B200 (sm_100a) decode-attention path.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t,
 * launches on that stream, never allocates device memory, and returns an
 * SpecdecResult code (0 = launched).  Host-side argument errors return
 * SPECDEC_ERR_INVALID and leave a message readable with
 * specdec_last_error().  Conditions that only the device can see (a length
 * past the page table, a bad page id, a trim out of range, a timed-out wait)
 * are OR-ed into an int32 device status word that the caller reads when it
 * next synchronises; the kernels never trap.
 *
 * Reference interfaces replaced (paths inside RichardF123/SpecDec-Context-Scaling):
 *   specdec_attention            <- attention_cuda, specdec/kernels/cuda/attention.cu:244-288,
 *                                   bound as "attention" in specdec/kernels/cuda/bind.cpp:16
 *   specdec_rmsnorm              <- rmsnorm_cuda, bind.cpp:13 (specdec/kernels/cuda/rmsnorm.cu)
 *   specdec_apply_rope           <- rope_cuda, bind.cpp:14 (specdec/kernels/cuda/rope.cu)
 *   specdec_swiglu               <- swiglu_cuda, bind.cpp:15 (specdec/kernels/cuda/swiglu.cu)
 *   specdec_paged_attention      <- the eager decode/verify branch of SelfAttention.forward,
 *                                   specdec/engine/model_self.py:715-775 (K/V history cat,
 *                                   whole-history V dequantisation, kv_repeat, masked softmax)
 *   specdec_append_kv            <- quantize_kv_fp8(v, GROUP_V) + cache append,
 *                                   specdec/engine/model_self.py:304-314 and :778-800
 *   specdec_rope_append          <- apply_rope of q and k (specdec/engine/model_self.py:286-296)
 *                                   followed by the cache append above, in one launch
 *   specdec_swiglu_packed        <- swiglu_cuda over a fused gate|up projection
 *   specdec_greedy_accept        <- vectorised accept, experiments/execution_optimization/
 *                                   fast_spec_dec.py:246-256 (strict form spec_dec.py:230-250)
 *   specdec_trim                 <- spec_cache.trim_cache, specdec/engine/spec_cache.py:10-28
 *   specdec_ragged_plan          <- no counterpart (the reference runs batch 1); builds the
 *                                   split-KV work list for a ragged batch on the device
 *   specdec_lmhead_argmax        <- logits = x @ embed_tokens.weight.T (model_self.py:857)
 *                                   followed by the executors' argmax (spec_dec.py:230-236,
 *                                   fast_spec_dec.py:246-249), fused: no logits are written
 */
#ifndef SPECDEC_B200_H_
#define SPECDEC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* specdec_stream_t; /* == cudaStream_t */

#define SPECDEC_ABI_VERSION 3
#define SPECDEC_PAGE_TOKENS 16 /* tokens per KV page */

typedef enum SpecdecResult {
  SPECDEC_OK = 0,
  SPECDEC_ERR_INVALID = 1,     /* bad argument; see specdec_last_error() */
  SPECDEC_ERR_UNSUPPORTED = 2, /* shape / dtype this build does not implement */
  SPECDEC_ERR_CUDA = 3,        /* launch failed; cuda error string in specdec_last_error() */
  SPECDEC_ERR_WORKSPACE = 4    /* workspace smaller than the *_workspace_bytes() answer */
} SpecdecResult;

/* Bits OR-ed into the device status word. */
#define SPECDEC_STATUS_BAD_LENGTH 0x1    /* ctx_len < q_len, or q_len > max_q_len     */
#define SPECDEC_STATUS_PAGE_OVERFLOW 0x2 /* position beyond max_pages_per_seq pages   */
#define SPECDEC_STATUS_BAD_PAGE 0x4      /* page id outside [0, num_pages)            */
#define SPECDEC_STATUS_TRIM_RANGE 0x8    /* trim length <= 0 or > current length      */
#define SPECDEC_STATUS_TIMEOUT 0x10      /* a bounded device wait gave up             */
#define SPECDEC_STATUS_ACCEPT_RANGE 0x20 /* accept: kp outside [1, max_cands]         */
#define SPECDEC_STATUS_PLAN_MISMATCH 0x40 /* reused plan built for another launch shape */

typedef enum SpecdecDtype { SPECDEC_F32 = 0, SPECDEC_BF16 = 1, SPECDEC_E4M3 = 2 } SpecdecDtype;

/*
 * Paged KV pool of one layer.  Pages hold SPECDEC_PAGE_TOKENS tokens; one
 * page id addresses the same token slots in every KV head.
 *   k_pool : bf16, [num_pages][num_kv_heads][16 * head_dim], each (page, head)
 *            block in the 128-byte-swizzled order that a TMA SWIZZLE_128B
 *            load of a {64 dims x 16 tokens} box writes to shared memory.
 *   v_pool : bf16 in the k_pool order            (v_dtype == SPECDEC_BF16), or
 *            e4m3 [num_pages][num_kv_heads][16][head_dim] code rows
 *            (v_dtype == SPECDEC_E4M3).
 *   v_scale: f32 [num_pages][num_kv_heads][16]: one max-abs/448 scale per
 *            token and KV head (E4M3 only; NULL for bf16 V).
 *   page_table: int32 [num_seqs][max_pages_per_seq]; token t of sequence b
 *            lives in page page_table[b][t / 16], slot t % 16.
 * The layout helpers in specdec_b200/engine/paged_cache.py (and the CPU
 * oracle) gather a pool back into the reference (B, KV, T, D) layout.
 */
typedef struct SpecdecPagedKV {
  const void* k_pool;
  const void* v_pool;
  const float* v_scale;
  const int32_t* page_table;
  int32_t num_pages;
  int32_t num_kv_heads;
  int32_t head_dim;          /* 64 or 128; E4M3 V requires 128 (GROUP_V == head_dim) */
  int32_t v_dtype;           /* SPECDEC_BF16 or SPECDEC_E4M3 */
  int32_t max_pages_per_seq;
} SpecdecPagedKV;

/*
 * Ragged batch description shared by the plan and the attention call.
 * Query row i (0-based) of sequence b sees keys j <= i + (ctx_len[b] - q_len[b]),
 * the engine's offset-causal mask (reference.py:40-44); q_len == 1 sees all keys.
 * Query/output element (b, i, h, d) lives at
 *     (q_row0[b] + i) * stride_tok + h * stride_head + d.
 * All arrays are device int32 [num_seqs].  q_len[b] == 0 skips sequence b.
 */
typedef struct SpecdecBatch {
  const int32_t* q_row0;
  const int32_t* q_len;
  const int32_t* ctx_len; /* KV tokens, the new q_len tokens included */
  int32_t num_seqs;
  int32_t num_q_heads;
  int32_t max_q_len; /* upper bound of q_len[], host-known; sizes the plan */
  int32_t max_ctx_len; /* upper bound of ctx_len[] when the host knows one, else 0; a small batch
                          of short contexts then runs on thread-block clusters (cluster_size) */
} SpecdecBatch;

typedef struct SpecdecAttnArgs {
  const void* q; /* bf16 */
  void* out;     /* bf16 */
  int64_t q_stride_tok, q_stride_head;
  int64_t o_stride_tok, o_stride_head;
  SpecdecBatch batch;
  SpecdecPagedKV kv;
  float sm_scale;       /* usually 1/sqrt(head_dim) */
  void* workspace;      /* >= specdec_attn_workspace_bytes(...) bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t* status;      /* device int32, may be NULL */
  int32_t reuse_plan;   /* 1: the workspace already holds the plan for this batch
                           (built by specdec_ragged_plan or an earlier call) */
  int32_t num_sms;      /* SMs the call may use; 0 or more than the device has: all of them
                           (the attention kernel runs one CTA per SM and its CTAs synchronise,
                           so all of them must fit on the device at once) */
  /* Optional profiling hook: cudaEvent_t handles recorded on `stream` right before
     and right after the split-KV kernel (as external event nodes under stream
     capture).  NULL = no events. */
  void* split_event_begin;
  void* split_event_end;
  /* 1: the caller promises that the KV history of every sequence (positions below
     ctx_len - q_len), the page table and, with reuse_plan, the plan are final when
     this call is enqueued -- the work immediately before it on the stream writes none
     of them.  The kernel then starts loading them while that work finishes (Q is
     still read, and outputs written, only after it).  0: nothing is read early. */
  int32_t history_ready;
  /* Thread-block clusters for small batches: the CTAs of a cluster reduce their split
     partials through distributed shared memory instead of a grid barrier and a merge
     through global memory.  0 = the library's choice: clusters when batch.max_ctx_len is
     known and every (sequence, query tile, KV head) group fits one cluster at one 128-key
     tile per CTA; 1 = never; 8 or 16 = clusters of that many CTAs whenever every group gets
     clusters of its own.  The plan (specdec_ragged_plan) and the attention calls that reuse
     it must pass the same value (a mismatch is refused: SPECDEC_STATUS_PLAN_MISMATCH). */
  int32_t cluster_size;
} SpecdecAttnArgs;

/* Bytes of workspace (plan + split-KV partials) for a batch of this shape. */
size_t specdec_attn_workspace_bytes(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t max_q_len, int32_t num_sms);

/* Build the split-KV work list of a ragged batch on the device (no host sync).
   The attention call with reuse_plan=1 consumes it; one plan serves every layer
   that shares the batch's lengths. */
int specdec_ragged_plan(const SpecdecAttnArgs* args, specdec_stream_t stream);

/* The launch shape specdec_paged_attention would use for these arguments (host-only, no
   launch): the verify kernel's grid and its cluster size (0: the persistent grid, no
   clusters).  No counterpart in the reference. */
int specdec_attn_launch_shape(const SpecdecAttnArgs* args, int32_t* grid, int32_t* cluster_size);

/* Paged decode (q_len 1) / block-verify (q_len k+1) / ragged attention. */
int specdec_paged_attention(const SpecdecAttnArgs* args, specdec_stream_t stream);

/*
 * specdec_paged_attention without a caller workspace.  This entry point has no
 * counterpart in the reference.  It serves callers that cannot allocate device
 * memory: a plugin host that owns all device memory and gives a plugin only its
 * inputs, outputs and a stream, or an FFI binding with no CUDA allocator of its
 * own.  It allocates nothing (no cudaMalloc, no allocating library call); its
 * scratch (plan + split partials) is a 32 MiB array compiled into the library,
 * held by every GPU that loads the library until the process exits.
 *   - args->workspace, args->workspace_bytes and args->reuse_plan are ignored; the
 *     plan is rebuilt on every call.
 *   - A batch needing more than 32 MiB of scratch (see specdec_attn_workspace_bytes)
 *     is rejected with SPECDEC_ERR_WORKSPACE before anything is launched.
 *   - The first call on a device looks up the scratch's device address with that
 *     device current; make that first call before any stream capture.  The address
 *     is cached per device and CUDA context: the first call in a new context (after
 *     cudaDeviceReset, say) looks it up again, so make that call outside capture too.
 *   - All calls share the one scratch area, which keeps the previous call's
 *     contents (nothing in it needs to start at zero).  Calls whose kernels
 *     overlap on the GPU (different streams, or different host threads) race on
 *     it: serialise them on one stream.
 */
int specdec_paged_attention_noalloc(const SpecdecAttnArgs* args, specdec_stream_t stream);

/*
 * Append n_new[b] tokens per sequence at positions pos0[b] .. pos0[b]+n_new[b]-1.
 * K is copied (bf16); V is copied (bf16 pool) or quantised to E4M3 with one
 * scale per token and KV head: s = max|v| / 448 (s = 1 when the max is 0),
 * code = rn_satfinite_e4m3(v / s) with IEEE division, which is bit-identical
 * to quantize_kv_fp8(v, 128) (model_self.py:304-314).
 * Element (b, i, h, d) of k_new / v_new is at
 *     (row0[b] + i) * stride_tok + h * stride_head + d.
 * len_out (optional) receives pos0[b] + n_new[b].
 */
typedef struct SpecdecAppendArgs {
  const void* k_new; /* bf16 */
  const void* v_new; /* bf16 */
  int64_t stride_tok, stride_head;
  const int32_t* row0;  /* [num_seqs] */
  const int32_t* n_new; /* [num_seqs] */
  const int32_t* pos0;  /* [num_seqs] */
  int32_t* len_out;     /* [num_seqs] or NULL */
  int32_t num_seqs;
  int32_t max_new; /* upper bound of n_new[], host-known */
  /* destination pool (written through these pointers) */
  void* k_pool;
  void* v_pool;
  float* v_scale;
  const int32_t* page_table;
  int32_t num_pages, num_kv_heads, head_dim, v_dtype, max_pages_per_seq;
  int32_t* status;
} SpecdecAppendArgs;

int specdec_append_kv(const SpecdecAppendArgs* args, specdec_stream_t stream);

/*
 * Fused rotary embedding + KV append of one decode / verify step (engine seam
 * after the fused QKV projection; the reference applies apply_rope to q and k
 * (specdec/engine/model_self.py:286-296) and then writes the cache).  qkv holds
 * `rows` packed rows of (num_q_heads + 2 num_kv_heads) heads x head_dim bf16 values
 * (q heads, k heads, v heads); cos / sin are (rows, head_dim) bf16 at each row's
 * position.  q_out (rows, num_q_heads, head_dim) receives the rotated queries; the
 * rotated k rows and the v rows of every sequence's first n_new[b] rows go to the
 * pool exactly as specdec_append_kv writes them (kv.k_new, kv.v_new and the strides
 * are unused).  Rounding: bf16(bf16(x cos) + bf16(rotate_half(x) sin)).
 */
typedef struct SpecdecRopeAppendArgs {
  const void* qkv;
  int64_t qkv_row_stride; /* elements */
  const void* cos;
  const void* sin;
  void* q_out;
  int32_t rows, num_q_heads;
  SpecdecAppendArgs kv;
} SpecdecRopeAppendArgs;

int specdec_rope_append(const SpecdecRopeAppendArgs* args, specdec_stream_t stream);

/*
 * Greedy accept on the device.  For sequence b, rows j = 0 .. n_rows[b]-1 of
 * logits (row (row0[b] + j), row stride `row_stride` elements, `vocab` columns)
 * give g[b][j] = argmax (first index on ties, NaN counts as the maximum, as
 * torch.argmax).  The accepted count m[b] is the length of the common prefix
 * of g[b][0 .. kp[b]-1] and cands[b][0 .. kp[b]-1]; next_token[b] = g[b][m[b]]
 * (the correction, or the bonus when every candidate matched and row kp exists).
 * When len_before/len_after are given: len_after[b] = len_before[b] + keep_offset + m[b]
 * (the cache rollback of the rejected tail; keep_offset = 1 when the verify block
 * started with the pending token).
 */
typedef struct SpecdecAcceptArgs {
  const void* logits; /* bf16 or f32 */
  int32_t logits_dtype;
  int64_t row_stride;
  int32_t vocab;
  const int32_t* row0;   /* [num_seqs] */
  const int32_t* n_rows; /* [num_seqs], <= max_rows */
  const int32_t* cands;  /* [num_seqs][max_cands] */
  const int32_t* kp;     /* [num_seqs] */
  int32_t num_seqs, max_rows, max_cands;
  int32_t* g;          /* [num_seqs][max_rows] */
  int32_t* m;          /* [num_seqs] */
  int32_t* next_token; /* [num_seqs] */
  const int32_t* len_before; /* optional */
  int32_t* len_after;        /* optional */
  int32_t keep_offset;
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;
} SpecdecAcceptArgs;

size_t specdec_accept_workspace_bytes(int32_t num_seqs, int32_t max_rows, int32_t vocab);
/* With logits == NULL the accept call takes g[b][j] as given (computed beforehand, e.g. by
   specdec_lmhead_argmax into that layout) and only runs the first-mismatch scan, the next
   token and the rollback length; it then needs no workspace. */
int specdec_greedy_accept(const SpecdecAcceptArgs* args, specdec_stream_t stream);

/*
 * Greedy tokens of `rows` hidden-state rows through the tied LM head, without the logits:
 *     argmax[r] = argmax_j bf16( sum_d x[r][d] w[j][d] )   (j < vocab)
 * with fp32 accumulation on the tensor cores and torch.argmax's order on the bf16 values
 * (NaN largest, first index on ties).  max_value[r] (optional) receives the winning bf16
 * logit.  x: bf16 [rows][x_stride] (hidden used), w: bf16 [vocab][hidden] contiguous;
 * hidden a multiple of 64; x, w 16-byte aligned.  The workspace
 * (specdec_lmhead_workspace_bytes(rows), 256-byte aligned) must be zero before the first
 * call; every call leaves it zero again.  Calls sharing a workspace must not overlap.
 */
typedef struct SpecdecLmHeadArgs {
  const void* x;
  int64_t x_stride; /* elements between rows of x */
  const void* w;
  int32_t rows, hidden, vocab;
  int32_t* argmax;  /* [rows] */
  float* max_value; /* [rows] or NULL */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;
  int32_t num_sms; /* 0: every SM */
} SpecdecLmHeadArgs;

size_t specdec_lmhead_workspace_bytes(int32_t rows);
int specdec_lmhead_argmax(const SpecdecLmHeadArgs* args, specdec_stream_t stream);

/* len_out[b] = new_len[b] when 0 < new_len[b] <= cur_len[b]; otherwise
   len_out[b] = cur_len[b] and SPECDEC_STATUS_TRIM_RANGE is raised
   (the ValueError of spec_cache.trim_cache, spec_cache.py:18-19). */
int specdec_trim(const int32_t* cur_len, const int32_t* new_len, int32_t* len_out, int32_t num_seqs,
                 int32_t* status, specdec_stream_t stream);

/* Contiguous-cache attention with the reference op's contract:
   q (B,H,S,D), k/v (B,KV,T,D), contiguous, f32 or bf16, D in {64,128},
   row i sees keys j <= i + (T - S).  bf16 runs the tensor-core split-KV kernel
   (TMA tensor maps over k/v); f32 runs a CUDA-core fp32 kernel. */
size_t specdec_attention_workspace_bytes(int32_t B, int32_t H, int32_t KV, int32_t S, int32_t D,
                                         int32_t num_sms);
int specdec_attention(const void* q, const void* k, const void* v, void* out, int32_t dtype,
                      int32_t B, int32_t H, int32_t KV, int32_t S, int32_t T, int32_t D,
                      void* workspace, size_t workspace_bytes, specdec_stream_t stream);

/* The contiguous op over a V-only FP8 dict cache (the engine's "v_fp8" format): bf16 q
   (B,H,S,128) and k (B,KV,T,128), E4M3 V codes (B,KV,T,128) with their per-token scales
   (B,KV,T) f32 -- the cache's "v" and "v_scale" tensors as they are.  The codes are widened
   inside the PV product with the scale folded into the probabilities, so no dequantised
   history is ever formed.  Replaces dequantize_kv_fp8 of the whole history followed by the
   attention of the patched forward (specdec/kernels/patch.py:94-103, model_self.py:723-725).
   Workspace as specdec_attention_workspace_bytes. */
int specdec_attention_fp8v(const void* q, const void* k, const void* v_codes, const float* v_scale, void* out,
                           int32_t B, int32_t H, int32_t KV, int32_t S, int32_t T, int32_t D, void* workspace,
                           size_t workspace_bytes, specdec_stream_t stream);

/* RMSNorm over the last dim (fp32 mean of squares; the normalised value is
   rounded to the input dtype before the weight multiply, as model_self.RMSNORM). */
int specdec_rmsnorm(const void* x, const void* weight, void* out, int32_t dtype, int64_t rows,
                    int32_t hidden, float eps, specdec_stream_t stream);
/* out = x * cos + rotate_half(x) * sin for x (B, H, S, D) with element strides
   (stride_b, stride_h, stride_s, 1); cos/sin contiguous (S, D); out contiguous (B, H, S, D). */
int specdec_apply_rope(const void* x, int64_t stride_b, int64_t stride_h, int64_t stride_s, const void* cos,
                       const void* sin, void* out, int32_t dtype, int32_t B, int32_t H, int32_t S, int32_t D,
                       specdec_stream_t stream);
/* out = silu(gate) * up, elementwise. */
int specdec_swiglu(const void* gate, const void* up, void* out, int32_t dtype, int64_t n,
                   specdec_stream_t stream);
/* SwiGLU of a fused gate|up projection (rows, 2 inter) bf16 -> (rows, inter):
 * bf16(bf16(silu(g)) * u) with silu from the hardware exponential and reciprocal (at most
 * one bf16 ulp from specdec_swiglu); inter % 8 == 0, 16-byte aligned rows. */
int specdec_swiglu_packed(const void* gate_up, void* out, int64_t rows, int64_t inter, specdec_stream_t stream);

/* Diagnostics. */
/* Tensor-core self-check (no counterpart in the reference): one CTA computes, with
   tcgen05 MMAs from 128-byte-swizzled shared memory into TMEM,
   out1[128][32] = k[128][128] . q[32][128]^T and out2[128][32] = v[128][128]^T . p[32][128]^T
   (bf16 row-major inputs, fp32 outputs) -- the operand layouts of the verify kernel. */
/* TMA gather self-check (no counterpart in the reference): one CTA fetches rows
   rows[0..3] of a [n_rows][2048 B] tensor `big` and of a [n_rows][64 B] tensor `small`
   with one four-row tensor gather each -- the page-row loads of the attention kernel --
   and writes the 4 x 2048 + 4 x 64 bytes received to `out`. */
int specdec_gather4_selftest(const void* big, const void* small, int64_t n_rows, const int32_t* rows, void* out,
                             int32_t* status, specdec_stream_t stream);
int specdec_umma_selftest(const void* k, const void* q, const void* v, const void* p, float* out1, float* out2,
                          int32_t* status, specdec_stream_t stream);
/* Bounded-wait self-check (no counterpart in the reference): every device wait of this
   library gives up after a time limit, raises SPECDEC_STATUS_TIMEOUT and returns.  This
   entry point runs those waits with a short limit `limit_ns` (1 us .. 100 ms) where nothing
   can complete them, so the timeout path itself can be tested:
     mode 0: one CTA waits on an mbarrier that nothing arrives on (grid must be 1);
     mode 1: `grid` CTAs (1 .. 8) meet at the grid barrier of the verify kernel expecting
             `n_ctas` arrivals on the zeroed device u64 `counter` (n_ctas > grid times out,
             n_ctas == grid passes).
   waited_ns (device u64, may be NULL) receives the time CTA 0 spent in its wait. */
int specdec_wait_selftest(int32_t mode, void* counter, int32_t n_ctas, int32_t grid, int64_t limit_ns,
                          int32_t* status, void* waited_ns, specdec_stream_t stream);
const char* specdec_last_error(void);
int specdec_abi_version(void);
/* Number of kernels this library launched since load (all entry points). */
int64_t specdec_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* SPECDEC_B200_H_ */
