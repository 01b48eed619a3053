// verify_kernel.cuh -- split-KV decode / verify attention on the fifth-generation
// tensor cores (tcgen05, TMEM accumulators) for head_dim 128 and 64 (head_dim-64 KV-head
// pairs run as 128-dim groups).  Included inside namespace sd by paged_attention.cu.
//
// Persistent CTAs (one per SM) over a balanced page range, 320 threads (448 for E4M3 V):
//   warps 0-7  softmax + epilogue; warp w owns keys 32 (w % 4) .. +31 of each
//              128-key tile (TMEM lane quarter w % 4) for the query rows of half
//              w / 4, and in the epilogue output dims 32 (w % 4) .. +31 of those rows
//   warp 8     producer: bulk-TMA copies of the pages into an NS-deep ring of
//              128-key tiles (K [2 halves][128 rows][128 B] in the 128-byte-swizzled
//              image of the pool; V likewise, or raw E4M3 rows + per-token scales),
//              and the Q rows of each item
//   warp 9     MMA issuer (one lane) and owner of the TMEM allocation
//   warps 10-13 (E4M3 V only) converters: hand each tile's per-token scales to the
//              softmax, then widen its E4M3 rows to f16 over the tile's K (once QK^T
//              has read it) while the softmax warps work on the same tile
// Per tile t (buffer b = t & 1):
//   S^T[b] (128 keys x NR rows, fp32, TMEM)  = K_tile . Q^T            (8 x K=16 MMAs)
//   softmax warps: row maxima over the tile, lazy online rescale of O (only when a
//   row max grows by more than 2^8), P = exp2(S - M) written to shared memory as
//   the MN-major B operand; E4M3 tiles are widened to f16 in shared memory and the
//   per-token scale is folded into P
//   O^T (128 dims x NR rows, fp32, TMEM)    += V_tile^T . P^T           (8 MMAs)
// QK^T of tile t+1 is issued before PV of tile t, so softmax and MMAs overlap.
// Rows: the n_rep query heads x q query positions of one KV head (NR = 16 or 32).
#pragma once

constexpr int kSmWarps = 8;                    // softmax warps: (key quarter, row half)
constexpr int kProducerWarp = kSmWarps;        // bulk-TMA producer
constexpr int kMmaWarp = kSmWarps + 1;         // MMA issuer, TMEM owner
constexpr int kCvtWarp0 = kSmWarps + 2;        // E4M3 V: first of kCvtWarps converter warps
constexpr int kCvtWarps = 4;
// threads of one CTA: softmax, producer, MMA (+ converters for E4M3 V)
template <bool VF8>
constexpr int v3_threads() { return 32 * (kSmWarps + 2 + (VF8 ? kCvtWarps : 0)); }
// register budget per thread: each SM sub-partition holds 16384 registers and ceil(warps / 4)
// of the CTA's warps (allocation in steps of 8 per thread)
template <bool VF8>
constexpr int v3_max_regs() { return (16384 / (32 * ((v3_threads<VF8>() / 32 + 3) / 4))) & ~7; }
constexpr int kTileKeys = 128;
constexpr int kTilePages = 8;
constexpr float kRescaleLog2 = 8.f;   // lazy rescale threshold (log2 units)
constexpr float kScaleSlack = 16.f;   // lazy growth of the E4M3 reference scale

// Shared-memory / TMEM plan of one CTA.  D = 128: K and V tiles are [2 dim halves]
// [128 keys][128 B].  D = 64: one dim half.  The PV MMA still runs with M = 128: its
// second 64-row half of V^T is the 16 KB that follow the stage (the next V stage, or
// K stage 0 after the last one -- the V stages come first), which only feeds rows
// 64-127 of O^T; those rows are never read.
template <int NR, bool VF8, int D>
struct V3Geom {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(!VF8 || D == 128, "E4M3 V needs head_dim 128");
  static constexpr int KH = D / 64;                      // 128-byte dim halves of a K row
  // ring depth (tiles).  E4M3: the converter warps widen a tile's V codes into the K half of
  // its own stage once QK^T of the tile has read K (no separate widened-V buffers), so four
  // 48.5 KB stages fit; the stage is free after PV
  static constexpr int NS = VF8 ? 4 : (D == 128 ? 3 : 6);
  static constexpr int KT = 16384 * KH;                  // K tile bytes
  static constexpr int VT = VF8 ? 16384 : 16384 * KH;    // V tile bytes as staged
  static constexpr int ST = VF8 ? 512 : 0;               // 128 scales
  static constexpr int V_OFF = D == 64 ? 0 : NS * KT;
  static constexpr int K_OFF = D == 64 ? NS * VT : 0;
  static constexpr int S_OFF = (D == 64 ? K_OFF + NS * KT : V_OFF + NS * VT);
  static constexpr int Q_OFF = ((S_OFF + NS * ST + 1023) / 1024) * 1024;
  static constexpr int QH = NR * 128;                    // one dim half of Q: [NR rows][128 B]
  static constexpr int QB = NR * 256;                    // one P buffer: [128 keys][NR rows x 2 B], MN-major
  static constexpr int P_OFF = Q_OFF + KH * QH;
  static constexpr int SMEM = P_OFF + 2 * QB + 1024;     // + alignment slack
  static constexpr int TMEM_COLS = NR <= 16 ? 64 : 128;  // S[2] + O = 3 NR columns
  static constexpr int PAGE_BYTES = 2048 * KH + (VF8 ? 2048 + 64 : 2048 * KH);  // bytes copied per page
  static_assert(D == 128 || (V_OFF == 0 && K_OFF == NS * VT), "D 64: PV's upper half reads the next 16 KB");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Row-wise maximum / sum over the 32 keys of a warp when each lane holds one key's
// NR row values: a transposing butterfly -- at each step a lane keeps one half of
// its values and swaps the other half with its partner.  Afterwards lane l holds
// the result for row (l % NR).
template <int NR>
SD_DEV float warp_rows_max(const float (&v)[NR], int lane) {
  float a[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) a[i] = v[i];
#pragma unroll
  for (int off = NR / 2; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? a[i] : a[i + off];
      const float keep = upper ? a[i + off] : a[i];
      a[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, off));
    }
  }
  if (NR < 32) {
#pragma unroll
    for (int off = NR; off < 32; off <<= 1) a[0] = fmaxf(a[0], __shfl_xor_sync(0xffffffffu, a[0], off));
  }
  return a[0];
}
template <int NR>
SD_DEV float warp_rows_sum(const float (&v)[NR], int lane) {
  float a[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) a[i] = v[i];
#pragma unroll
  for (int off = NR / 2; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? a[i] : a[i + off];
      const float keep = upper ? a[i + off] : a[i];
      a[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  if (NR < 32) {
#pragma unroll
    for (int off = NR; off < 32; off <<= 1) a[0] += __shfl_xor_sync(0xffffffffu, a[0], off);
  }
  return a[0];
}


#include "verify_kernel_body.inc"
