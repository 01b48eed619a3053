// paged_attention.cu -- split-KV decode / block-verify attention over the paged
// BF16-K / (BF16 | E4M3)-V pool, and over contiguous (B, KV, T, D) tensors.
//
// What it computes (the eager branch of SelfAttention.forward,
// specdec/engine/model_self.py:740-775, and reference.attention,
// specdec/kernels/reference.py:47-56):
//     out[b, h, i] = softmax_j( q[b,h,i] . k[b,h/n_rep,j] * sm_scale ) . v[b,h/n_rep,j]
// over keys j <= i + (T - S) (reference.py:40-44; S == 1 sees every key), with
// GQA handled by sharing one K/V stream among the n_rep query heads of a KV
// head instead of materialising kv_repeat (model_self.py:294-298).  For an E4M3
// V cache the dequantisation of model_self.py:316-320 happens inside the PV
// product: the per-token scale is folded into the probabilities and the codes
// feed the tensor cores as exact f16 values.
//
// Launch structure (one attention call):
//   1. plan_kernel     (1 CTA)   device lengths -> work items (seq, kv head,
//                                query tile, key-block range) + merge groups.
//                                One plan serves all layers of a step.
//   2. verify_kernel   (head_dim 64 / 128; persistent, one CTA per SM over a
//                                balanced page range) tcgen05 QK^T / PV with TMEM
//                                accumulators, see verify_kernel.cuh.
//      The same kernel merges the split partials of groups with more than one
//      split after a grid barrier (merge_splits: by the CTAs with pages, or by spare
//      blocks without pages where the grid has room), or -- small batches of short
//      contexts -- inside thread-block clusters through distributed shared memory
//      (cluster_merge).  head_dim-64 KV-head pairs run as 128-dim groups.
#include <cudaTypedefs.h>

#include <math.h>

#include <mutex>
#include <utility>

#include "sd_common.cuh"
#include "sd_internal.h"
#include "umma.cuh"

namespace sd {

// ---------------------------------------------------------------- plan records
struct WorkItem {             // 48 bytes
  int32_t b, h, q0, nq;       // sequence, kv head, first query row, query rows in the tile
  int32_t page_begin, page_end;  // key blocks [page_begin, page_end) of 16 tokens
  int32_t group, nsplit;      // merge group; splits in the group (1 = write the output directly)
  int32_t ctx, qlen, row0;    // the sequence's context length, query rows and first output row
  int32_t cta;                // the persistent CTA that processes the item
};
static_assert(sizeof(WorkItem) == 48, "work item is 48 bytes");
// What a persistent CTA needs before its first copies: its item range, its first
// kDescItems work items (every role reads them from shared memory, so switching items
// waits for no global load; later ones come from the item list), the first item's first 32
// page ids (0 past the item), and for after its items the merge counts -- one 384-byte line.
constexpr int kDescItems = 4;
struct CtaDesc {
  WorkItem items[kDescItems];  // cluster mode: items[0] is the CTA's group (its item, or the
                               // group's fields when it has no pages)
  int32_t item_begin, item_end;  // the CTA's items: [item_begin, item_end) (every CTA of the grid)
  int32_t cl_first, cl_count;    // cluster mode: the group's first cluster and cluster count (0: idle)
  int32_t pages[32];
  // the plan header's merge counts and CTA count, so the merge needs no header load
  int32_t num_merge_wide, num_merge_narrow, num_ctas;
  // the launch shape the plan was built for: the verify kernel runs nothing when the
  // descriptor does not match its own grid (a plan reused with another cluster choice)
  int32_t plan_magic, plan_cluster, plan_grid;
  // split merge: this block's place among the merging CTAs (-1: it merges nothing), their
  // count, and the grid-barrier arrivals per launch (0: this block does not arrive)
  int32_t merge_cta, merge_ctas, bar_ctas;
  int32_t pad1[3];
};
constexpr int32_t kPlanMagic = 0x53504c4e;
static_assert(sizeof(CtaDesc) == 384, "CTA descriptor is 384 bytes");
struct GroupInfo {
  int32_t first_item, nsplit, b, h, q0, nq, pad0, pad1;
};
struct PlanHeader {
  int32_t num_items, pages_per_split, num_groups, total_pages;
  int32_t num_merge_wide;    // split groups with >= kMergeWide splits: merge_list[0 ..)
  int32_t num_merge_narrow;  // other split groups: merge_list[max_groups - 1], [max_groups - 2], ...
  int32_t num_ctas;          // CTAs that get pages (the verify grid's blocks: see CtaDesc)
  int32_t pad0[25];
  unsigned long long bar_arrive;  // grid-barrier arrivals of the verify kernel (own 128-byte line)
  int32_t pad1[30];
};
static_assert(sizeof(PlanHeader) == 256, "plan header is 256 bytes");

constexpr int kMaxRows = 64;  // query rows (n_rep x query positions) per work item
constexpr int kPlanTilePages = 8;  // pages per 128-key tile of the verify kernel
constexpr int kWholeTileMax = 4;   // the plan gives CTAs whole tiles up to this many per CTA
// what starting one more item costs a CTA of a bandwidth-bound call, in pages (measured: about
// 3 us per extra item against 0.18 us per page of a ragged batch, bf16 or E4M3 V)
constexpr int kItemCostPages = 16;
// per split item and row, one 32-byte sector: the row max (log2 units), the four
// key-quarter partial sums and three unused words
constexpr int kStatStride = 8;
constexpr int kMergeWide = 16;  // groups with at least this many splits are merged by whole CTAs

struct WsLayout {
  size_t items, groups, ctas, cdesc, mlist, tickets, lse, po, total;
  int32_t max_items, max_groups;
};

static WsLayout ws_layout(int B, int KV, int max_qtiles, int D, int target_items) {
  WsLayout w;
  w.max_groups = B * max_qtiles * KV;
  w.max_items = target_items + w.max_groups;
  w.items = sizeof(PlanHeader);
  w.groups = align_up(w.items + sizeof(WorkItem) * (size_t)w.max_items, 256);
  w.ctas = align_up(w.groups + sizeof(GroupInfo) * (size_t)w.max_groups, 256);
  w.cdesc = align_up(w.ctas + sizeof(int32_t) * (size_t)(target_items / 4 + 1), 256);
  w.mlist = align_up(w.cdesc + sizeof(CtaDesc) * (size_t)(target_items / 4 + 1), 256);
  w.tickets = align_up(w.mlist + sizeof(GroupInfo) * (size_t)w.max_groups, 256);
  w.lse = align_up(w.tickets + sizeof(int32_t) * kMaxRows * (size_t)(target_items / 4 + 1), 256);
  w.po = align_up(w.lse + sizeof(float) * kStatStride * kMaxRows * (size_t)w.max_items, 256);
  w.total = align_up(w.po + sizeof(float) * kMaxRows * (size_t)D * w.max_items, 256);
  return w;
}

struct AttnParams {
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  int64_t q_st, q_sh, o_st, o_sh;
  const int32_t* q_row0;
  const int32_t* q_len;
  const int32_t* ctx_len;
  int32_t uni_q_len, uni_ctx_len, uni_row_stride;  // used where the arrays are NULL
  int32_t B, H, KV, n_rep, max_q_len, q_tile, max_qtiles;
  const uint8_t* k_pool;
  const uint8_t* v_pool;
  const float* v_scale;
  const int32_t* page_table;
  int32_t num_pages, max_pages;
  float scale_log2;
  PlanHeader* hdr;
  WorkItem* items;
  GroupInfo* groups;
  int32_t* cta_first;  // [C + 1]: items of persistent CTA c are cta_first[c] .. cta_first[c+1]-1
  CtaDesc* cdesc;      // [C]: first item and page ids of every CTA
  GroupInfo* merge_list;  // [max_groups]: the groups with more than one split (see PlanHeader)
  float* p_stat;  // [item][kMaxRows][kStatStride]: row max, then key-quarter sums
  float* p_o;
  int32_t max_items, max_groups, target_items;
  int32_t tile_pages;  // the verify kernel consumes keys in tiles of this many pages
  int32_t early_loads;  // 1: plan, page table and KV history may be read before the dependency wait
  int32_t* status;
  // cluster mode (cluster_size > 0): the grid is num_clusters clusters of cluster_size CTAs;
  // every cluster works on one group and reduces its CTAs' partials in distributed shared
  // memory; groups spread over several clusters meet through per-row tickets
  int32_t cluster_size, num_clusters;
  int32_t* tickets;  // [num_clusters][kMaxRows]: arrivals of a group's clusters per row
  int32_t max_ctx_hint;  // host-known upper bound of the context lengths, 0 when unknown
  // Paired heads (head_dim 64): KV heads 2j and 2j + 1 run as one 128-dim group j -- a page's
  // two 2 KB head blocks are the two dim halves of one 128-dim key row, each query row
  // carries its 64 dims in its own head's half and zeros in the other, so the 128-dim scores
  // are the per-head ones and a query row's output is its own half of the 128-dim O row.
  // half_heads = query heads per original KV head (n_rep / 2 here); 0 = not paired.
  int32_t half_heads;
};

SD_DEV int seq_q_len(const AttnParams& p, int b) { return p.q_len ? p.q_len[b] : p.uni_q_len; }
SD_DEV int seq_ctx_len(const AttnParams& p, int b) { return p.ctx_len ? p.ctx_len[b] : p.uni_ctx_len; }
SD_DEV int seq_row0(const AttnParams& p, int b) { return p.q_row0 ? p.q_row0[b] : b * p.uni_row_stride; }
// Output dim of O-row dim d for the query row of group head hh: d itself, or with paired
// heads d's place in the row's own head (-1 for the other head's half).  PAIR: the kernel
// form can run paired heads (bf16 V, 128-dim tiles, paged pools); the others compile none
// of this.
template <bool PAIR>
SD_DEV int paired_dim(const AttnParams& p, int hh, int d) {
  if (!PAIR || p.half_heads == 0) return d;
  return (d >> 6) == hh / p.half_heads ? (d & 63) : -1;
}

// ---------------------------------------------------------------- plan
// Key blocks a (sequence, query tile) group must read, or 0 for an empty /
// invalid group.  Invalid lengths are reported once per sequence.
SD_DEV int group_pages(const AttnParams& p, int gi, int& b, int& h, int& q0, int& nq) {
  const int per_b = p.max_qtiles * p.KV;
  b = gi / per_b;
  const int rem = gi - b * per_b;
  const int qt = rem / p.KV;
  h = rem - qt * p.KV;
  const int qlen = seq_q_len(p, b);
  const int ctx = seq_ctx_len(p, b);
  q0 = qt * p.q_tile;
  nq = min(p.q_tile, qlen - q0);
  if (qlen <= 0 || nq <= 0) return 0;
  if (qlen > p.max_q_len || ctx < qlen) {
    if (qt == 0 && h == 0) raise_status(p.status, SPECDEC_STATUS_BAD_LENGTH);
    return 0;
  }
  if (ctx > p.max_pages * kPage) {
    if (qt == 0 && h == 0) raise_status(p.status, SPECDEC_STATUS_PAGE_OVERFLOW);
    return 0;
  }
  const int visible = q0 + nq + (ctx - qlen);  // keys seen by the last row of the tile
  return (visible + kPage - 1) / kPage;
}

// Exclusive block scan of one int per thread (blockDim.x <= 1024); returns the
// block total through `total`.
SD_DEV int block_exclusive_scan(int v, int& total, int* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive prefix of warp totals
  }
  __syncthreads();
  const int before = warp > 0 ? s_warp[warp - 1] : 0;
  total = s_warp[((blockDim.x + 31) >> 5) - 1];
  __syncthreads();
  return before + x - v;
}

// ---------------------------------------------------------------- cluster-mode plan
// Small batches (every group fits a cluster of its own) run the verify kernel as
// num_clusters clusters of cluster_size CTAs.  Group g gets c_g clusters: the fewest tiles
// per CTA k such that sum_g ceil(tiles_g / (cluster_size k)) clusters fit the grid, with
// c_g = ceil(tiles_g / (cluster_size k)); its c_g * cluster_size CTAs split the group's
// 128-key tiles evenly (some CTAs of a short group get none).  Clusters without a group
// come first in the grid (dispatched first, they leave at once).  One item per CTA, item
// index = block index.  The per-row tickets of the clusters start at zero.
constexpr int kClusterMaxGroups = 32;
constexpr int kClusterMaxSlots = 8;  // clusters a group may span (the last one merges that many partials)
SD_DEV void cluster_plan(const AttnParams& p) {
  __shared__ int s_pages[kClusterMaxGroups], s_c[kClusterMaxGroups], s_cl0[kClusterMaxGroups];
  const int G = p.max_groups, CS = p.cluster_size, NC = p.num_clusters, grid = NC * CS;
  const int t = threadIdx.x;
  if (t < kClusterMaxGroups) {
    int b, h, q0, nq;
    s_pages[t] = t < G ? group_pages(p, t, b, h, q0, nq) : 0;
  }
  __syncthreads();
  if (t == 0) {
    // (a group spans at most kClusterMaxSlots clusters: the last one merges that many partials)
    int k = 1;
    for (;; ++k) {
      int need = 0, widest = 0;
      for (int g = 0; g < G; ++g) {
        const int tiles = (s_pages[g] + kPlanTilePages - 1) / kPlanTilePages;
        const int c = (tiles + CS * k - 1) / (CS * k);
        need += c;
        widest = max(widest, c);
      }
      if (need <= NC && widest <= kClusterMaxSlots) break;
    }
    int used = 0;
    for (int g = 0; g < G; ++g) {
      const int tiles = (s_pages[g] + kPlanTilePages - 1) / kPlanTilePages;
      s_c[g] = (tiles + CS * k - 1) / (CS * k);
      used += s_c[g];
    }
    int cl = NC - used;  // idle clusters first
    for (int g = 0; g < G; ++g) {
      s_cl0[g] = cl;
      cl += s_c[g];
    }
  }
  __syncthreads();
  for (int x = t; x < grid; x += blockDim.x) {
    const int cl = x / CS, cr = x - cl * CS;
    int g = -1;
    for (int j = 0; j < G; ++j)
      if (s_c[j] > 0 && cl >= s_cl0[j] && cl < s_cl0[j] + s_c[j]) g = j;
    CtaDesc& d = p.cdesc[x];
    WorkItem it;
    memset(&it, 0, sizeof(it));
    d.cl_first = 0;
    d.cl_count = 0;
    if (g >= 0) {
      int b, h, q0, nq;
      const int P = group_pages(p, g, b, h, q0, nq);
      const int n = s_c[g] * CS, j = (cl - s_cl0[g]) * CS + cr;
      const int tiles = (P + kPlanTilePages - 1) / kPlanTilePages;
      const int t0 = static_cast<int>(static_cast<long long>(j) * tiles / n);
      const int t1 = static_cast<int>(static_cast<long long>(j + 1) * tiles / n);
      it.b = b;
      it.h = h;
      it.q0 = q0;
      it.nq = nq;
      it.page_begin = min(t0 * kPlanTilePages, P);
      it.page_end = min(t1 * kPlanTilePages, P);
      it.group = g;
      it.nsplit = n;  // > 1: the epilogue writes a partial
      it.ctx = seq_ctx_len(p, b);
      it.qlen = seq_q_len(p, b);
      it.row0 = seq_row0(p, b);
      it.cta = x;
      d.cl_first = s_cl0[g];
      d.cl_count = s_c[g];
    }
    p.items[x] = it;
    d.items[0] = it;
    d.item_begin = x;
    d.item_end = x + (it.page_end > it.page_begin ? 1 : 0);
    d.num_merge_wide = 0;
    d.num_merge_narrow = 0;
    d.num_ctas = grid;
    d.plan_magic = kPlanMagic;
    d.plan_cluster = CS;
    d.plan_grid = grid;
    d.merge_cta = -1;
    d.merge_ctas = 0;
    d.bar_ctas = 0;
  }
  __syncthreads();
  for (int u = t; u < grid * 32; u += blockDim.x) {
    const int x = u >> 5, kk = u & 31;
    const WorkItem& it = p.cdesc[x].items[0];
    p.cdesc[x].pages[kk] = (p.page_table != nullptr && kk < it.page_end - it.page_begin)
                               ? p.page_table[static_cast<int64_t>(it.b) * p.max_pages + it.page_begin + kk]
                               : 0;
  }
  for (int i = t; i < NC * kMaxRows; i += blockDim.x) p.tickets[i] = 0;
  if (t == 0) {
    p.hdr->num_items = grid;
    p.hdr->pages_per_split = 0;
    p.hdr->num_groups = G;
    p.hdr->bar_arrive = 0ull;
    p.hdr->num_merge_wide = 0;
    p.hdr->num_merge_narrow = 0;
    p.hdr->total_pages = 0;
    p.hdr->num_ctas = grid;
  }
}

__global__ void __launch_bounds__(1024) plan_kernel(const AttnParams p) {
  if (p.cluster_size > 0) {
    cluster_plan(p);
    return;
  }
  __shared__ int s_warp[32];
  __shared__ long long s_total;
  __shared__ int s_rows, s_live;
  __shared__ int s_first[1024], s_pages[1024], s_nq[1024], s_c0[1024];
  __shared__ long long s_start[1024];
  // each persistent CTA's first item (index and copy), recorded as the items are written
  constexpr int kPlanCtas = 192;
  __shared__ int s_cfirst[kPlanCtas + 1];
  __shared__ WorkItem s_fitem[kPlanCtas];
  const int ngroups = p.max_groups;
  if (threadIdx.x == 0) {
    s_total = 0;
    s_rows = 0;
    s_live = 0;
  }
  for (int c = threadIdx.x; c <= kPlanCtas; c += blockDim.x) s_cfirst[c] = -1;  // -1: no item
  __syncthreads();
  long long local = 0;
  int lrows = 0;  // query rows of the groups with pages
  int llive = 0;  // groups with pages
  for (int gi = threadIdx.x; gi < ngroups; gi += blockDim.x) {
    int b, h, q0, nq;
    const int pg = group_pages(p, gi, b, h, q0, nq);
    local += pg;
    if (pg > 0) {
      lrows += p.n_rep * nq;
      ++llive;
    }
  }
  // warp reduce then one atomic per warp
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    local += __shfl_xor_sync(0xffffffffu, local, o);
    lrows += __shfl_xor_sync(0xffffffffu, lrows, o);
    llive += __shfl_xor_sync(0xffffffffu, llive, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&s_total), static_cast<unsigned long long>(local));
    atomicAdd(&s_rows, lrows);
    atomicAdd(&s_live, llive);
  }
  __syncthreads();
  const long long P = s_total;
  // Balanced split: the concatenation of every group's pages (groups in order) is
  // cut into C equal ranges, range c = [c*P/C, (c+1)*P/C) for CTA c of the
  // persistent kernel.  An item is the intersection of a range with a group, so
  // a group yields one item per range it meets: num_items <= C + groups.
  // C <= P keeps every range non-empty (so no item is empty); the CTAs past C get no items.
  // Small calls (at most kWholeTileMax tiles per CTA, e.g. one sequence of a few thousand
  // tokens) are latency-bound: there C is the fewest CTAs that each take k whole 128-key
  // tiles (an 8192-token sequence: 2 x 64 CTAs of one tile, not 148 of 7 pages), so no CTA
  // pays a tile's latency for a fraction of one and the merge has fewer splits -- but no
  // fewer CTAs than split rows when the grid has that many, so the merge of rows split
  // across many CTAs (a CTA each) still runs in one round.  Spare merge: when the grid
  // also has a block for every query row beside the CTAs of k whole tiles, those spare
  // blocks merge the split rows and the CTAs with pages leave at their barrier arrival --
  // the SMs they free take the next launch's CTAs, which load their KV history while this
  // launch merges.  (Measured: 8192-token q 1 9.3 -> 8.85 us per layer, 2048-token q 5 on
  // the persistent grid 9.1 -> 8.65 us; taking k + 1 tiles per CTA to make room for spare
  // blocks was slower, and so was staging several rows per spare block with bulk copies --
  // 128 small copies per row cost ~3 us.)
  const int grid = p.target_items / 4;
  bool spare = false;
  int C = static_cast<int>(min(static_cast<long long>(grid), max(P, 1LL)));
  // Bandwidth-bound calls: every item a CTA starts costs about as much as kItemCostPages
  // pages (its last PV and epilogue are not overlapped with the next item's tiles), so the
  // split runs over a cost axis on which each group is preceded by that many units without
  // pages; CTAs then finish together whatever their item counts.
  long long ov = kItemCostPages;
  {
    const long long tile_slots = static_cast<long long>(kPlanTilePages) * grid;
    const long long k = (P + tile_slots - 1) / tile_slots;  // tiles per CTA with the whole grid
    if (k >= 1 && k <= kWholeTileMax) {
      const long long per = k * kPlanTilePages;
      long long want = (P + per - 1) / per;
      if (want > 1 && want + s_rows <= grid) {
        spare = true;
      } else if (s_rows <= grid) {
        want = max(want, static_cast<long long>(s_rows));
      }
      C = static_cast<int>(min(static_cast<long long>(C), want));
      ov = 0;  // whole tiles: no cost axis
    }
  }
  // the cost axis: pages plus ov per group with pages (every range of a bandwidth-bound call
  // spans more than kWholeTileMax tiles > ov units, so each one holds real pages)
  const long long Pc = P + ov * s_live;
  auto cta_of = [&](long long pos) { return static_cast<int>(((pos + 1) * C + Pc - 1) / Pc) - 1; };
  auto range_lo = [&](int c) { return static_cast<long long>(c) * Pc / C; };

  int carry = 0, wcarry = 0, ncarry = 0;
  long long pcarry = 0;
  for (int base = 0; base < ngroups; base += blockDim.x) {
    const int gi = base + threadIdx.x;
    int b = 0, h = 0, q0 = 0, nq = 0, pages = 0;
    if (gi < ngroups) pages = group_pages(p, gi, b, h, q0, nq);
    const int cost = pages > 0 ? pages + static_cast<int>(ov) : 0;
    int chunk_pages;
    // the group's pages start after its ov units on the cost axis
    const long long start = pcarry + block_exclusive_scan(cost, chunk_pages, s_warp) + ov;
    int n = 0, c0 = 0;
    if (pages > 0) {
      c0 = cta_of(start);
      n = cta_of(start + pages - 1) - c0 + 1;
    }
    int chunk_total;
    const int first = carry + block_exclusive_scan(n, chunk_total, s_warp);
    const bool wide = n >= kMergeWide, narrow = n > 1 && !wide;
    int chunk_wide, chunk_narrow;
    const int wpos = wcarry + block_exclusive_scan(wide ? 1 : 0, chunk_wide, s_warp);
    const int npos = ncarry + block_exclusive_scan(narrow ? 1 : 0, chunk_narrow, s_warp);
    if (gi < ngroups) {
      GroupInfo g;
      g.first_item = first;
      g.nsplit = n;
      g.b = b;
      g.h = h;
      g.q0 = q0;
      g.nq = nq;
      g.pad0 = g.pad1 = 0;
      p.groups[gi] = g;
      if (wide) p.merge_list[wpos] = g;
      if (narrow) p.merge_list[p.max_groups - 1 - npos] = g;
    }
    // items of this chunk of groups, written in parallel: item i belongs to the
    // last group whose first item is <= i (empty groups never match)
    s_first[threadIdx.x] = (gi < ngroups) ? first - carry : 0x7fffffff;
    s_pages[threadIdx.x] = pages;
    s_nq[threadIdx.x] = nq;
    s_c0[threadIdx.x] = c0;
    s_start[threadIdx.x] = start;
    __syncthreads();
    for (int i = threadIdx.x; i < chunk_total; i += blockDim.x) {
      int lo = 0, hi = blockDim.x - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_first[mid] <= i) lo = mid; else hi = mid - 1;
      }
      const int g2 = base + lo;
      const int c = s_c0[lo] + (i - s_first[lo]);
      const long long gs = s_start[lo];
      const int pg = s_pages[lo];
      const int per_b = p.max_qtiles * p.KV;
      const int b2 = g2 / per_b;
      const int rem = g2 - b2 * per_b;
      WorkItem it;
      it.b = b2;
      it.h = rem % p.KV;
      it.q0 = (rem / p.KV) * p.q_tile;
      it.nq = s_nq[lo];
      it.page_begin = static_cast<int>(max(range_lo(c) - gs, 0LL));
      it.page_end = static_cast<int>(min(range_lo(c + 1) - gs, static_cast<long long>(pg)));
      it.group = g2;
      it.nsplit = cta_of(gs + pg - 1) - s_c0[lo] + 1;
      it.ctx = seq_ctx_len(p, b2);
      it.qlen = seq_q_len(p, b2);
      it.row0 = seq_row0(p, b2);
      it.cta = c;
      p.items[carry + i] = it;
      // range c starts inside this group (its cost units included): CTA c's first item
      if (range_lo(c) >= gs - ov && c < kPlanCtas) {
        s_cfirst[c] = carry + i;
        s_fitem[c] = it;
      }
    }
    __syncthreads();
    carry += chunk_total;
    wcarry += chunk_wide;
    ncarry += chunk_narrow;
    pcarry += chunk_pages;
  }
  // first item of every CTA of the grid (items are ordered by CTA): cta_first[c] .. cta_first[c+1];
  // the CTAs past C have none
  const bool recorded = grid <= kPlanCtas;
  for (int c = threadIdx.x; c <= grid; c += blockDim.x) {
    int first;
    if (recorded) {
      first = (c < C && s_cfirst[c] >= 0) ? s_cfirst[c] : carry;
    } else {
      int lo = 0, hi = carry;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (p.items[mid].cta < c) lo = mid + 1; else hi = mid;
      }
      first = lo;
    }
    p.cta_first[c] = first;
  }
  __syncthreads();
  // Descriptors by block.  Merged by the CTAs with pages: blocks 0 .. idle - 1 of the verify
  // grid get no pages -- they are dispatched first and leave at once, so they never wait for
  // an SM that a previous launch still holds -- and block idle + c runs CTA c's range.
  // Spare merge: block c runs CTA c's range, blocks C .. C + M - 1 merge (dispatched after
  // the CTAs with pages, onto the SMs the previous launch's merge frees last), and the
  // remaining blocks leave at once.  M: a block for every wide row and for the narrow rows
  // at one warp each (a CTA has at least eight warps).
  const int idle = grid - C;
  const int ru = p.n_rep * min(p.q_tile, p.max_q_len);
  const int M = spare ? min(grid - C, max(wcarry * ru, (ncarry * ru + 7) / 8)) : C;
  auto blk = [&](int c) { return spare ? c : idle + c; };
  for (int bx = threadIdx.x; bx < grid; bx += blockDim.x) {
    const int c = spare ? (bx < C ? bx : -1) : bx - idle;
    const int mc = spare ? (bx >= C && bx < C + M ? bx - C : -1) : c;
    p.cdesc[bx].item_begin = c < 0 ? 0 : p.cta_first[c];
    p.cdesc[bx].item_end = c < 0 ? 0 : p.cta_first[c + 1];
    p.cdesc[bx].num_merge_wide = wcarry;
    p.cdesc[bx].num_merge_narrow = ncarry;
    p.cdesc[bx].num_ctas = C;
    p.cdesc[bx].cl_first = 0;
    p.cdesc[bx].cl_count = 0;
    p.cdesc[bx].plan_magic = kPlanMagic;
    p.cdesc[bx].plan_cluster = 0;
    p.cdesc[bx].plan_grid = grid;
    p.cdesc[bx].merge_cta = mc;
    p.cdesc[bx].merge_ctas = M;
    p.cdesc[bx].bar_ctas = (c >= 0 || mc >= 0) ? (spare ? C + M : C) : 0;
  }
  // first item and page ids: thread t fills page slot t % 32 of CTA t / 32
  for (int u = threadIdx.x; u < C * 32; u += blockDim.x) {
    const int c = u >> 5, k = u & 31;
    // no work (no pages at all, P == 0): the CTA reads no descriptor
    if (recorded ? s_cfirst[c] < 0 : p.cta_first[c] >= p.cta_first[c + 1]) continue;
    const WorkItem it = recorded ? s_fitem[c] : p.items[p.cta_first[c]];
    CtaDesc& d = p.cdesc[blk(c)];
    if (k == 0) d.items[0] = it;
    if (k > 0 && k < kDescItems && p.cta_first[c] + k < p.cta_first[c + 1]) d.items[k] = p.items[p.cta_first[c] + k];
    d.pages[k] = (p.page_table != nullptr && k < it.page_end - it.page_begin)
                     ? p.page_table[static_cast<int64_t>(it.b) * p.max_pages + it.page_begin + k]
                     : 0;
  }
  if (threadIdx.x == 0) {
    p.hdr->num_items = carry;
    p.hdr->pages_per_split = static_cast<int32_t>(C > 0 ? (P + C - 1) / C : 0);
    p.hdr->num_groups = ngroups;
    p.hdr->bar_arrive = 0ull;
    p.hdr->num_merge_wide = wcarry;
    p.hdr->num_merge_narrow = ncarry;
    p.hdr->total_pages = static_cast<int32_t>(P);
    p.hdr->num_ctas = C;
  }
}

// ---------------------------------------------------------------- split merge
// Log-sum-exp merge of split partials, run by the verify kernel's CTAs once every
// CTA has written its partials (after its grid barrier).  A split item leaves, per
// query row, its unnormalised O row (sum over its keys of p v, p = 2^(s - m)), its
// row max m and four key-quarter partial sums of p; the merge rescales them to the
// common max and normalises once.  A unit is one query row of a group in the plan's
// merge_list (the groups with more than one split).  Rows of groups with >=
// kMergeWide splits are merged by a whole CTA (its warps take every NWARP-th split
// and combine in shared memory); the other rows by one warp each.  Lane l owns dims
// 4(l % NQ) .. +3 of the splits s = l / NQ (mod SPW), so every lane streams float4
// partial rows; the state is an online (max, sum, acc).  Partials come from other
// CTAs of the same launch, so they are read with L1-bypassing loads.
struct MergeState {
  float m, l;
  float4 a;
};
SD_DEV void merge_combine(MergeState& st, const MergeState& o) {
  if (o.m == -INFINITY) return;
  const float m = fmaxf(st.m, o.m);
  const float f = (st.m == -INFINITY) ? 0.f : fast_exp2(st.m - m);
  const float g = fast_exp2(o.m - m);
  st.a.x = st.a.x * f + o.a.x * g;
  st.a.y = st.a.y * f + o.a.y * g;
  st.a.z = st.a.z * f + o.a.z * g;
  st.a.w = st.a.w * f + o.a.w * g;
  st.l = st.l * f + o.l * g;
  st.m = m;
}

// s_st: NWARP x 32 states of shared memory (the caller's free staging area).
// cta: the caller's place among the n_ctas merging CTAs (the CTAs with pages, or the
// plan's spare blocks).
// n_wide / n_narrow: the plan's merge-list counts; pre_w / pre_n: the merge-list
// entries of this CTA's first wide unit and this warp's first narrow unit, loaded
// before the grid barrier.
template <int D, int NWARP, bool PAIR>
SD_DEV void merge_splits(const AttnParams& p, MergeState* s_st, int cta, int warp, int lane, int n_wide, int n_narrow,
                         int n_ctas, const GroupInfo& pre_w, const GroupInfo& pre_n) {
  constexpr int NQ = D / 4;     // dim quads
  constexpr int SPW = 32 / NQ;  // split slots per warp
  const int quad = lane % NQ, slot = lane / NQ;
  const int RU = p.n_rep * min(p.q_tile, p.max_q_len);  // row slots per group
  const int wide_units = n_wide * RU;
  const int narrow_units = n_narrow * RU;

  // the splits s = s0, s0 + step, ... of row r of group grp
  auto stream = [&](const GroupInfo& grp, int r, int s0, int step, MergeState& st) {
    st.m = -INFINITY;
    st.l = 0.f;
    st.a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = s0; s < grp.nsplit; s += 8 * step) {
      float ms[8], ls[8];
      float4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int sk = s + k * step;
        const bool in = sk < grp.nsplit;
        const int64_t item = static_cast<int64_t>(grp.first_item) + sk;
        const float* st_row = p.p_stat + (item * kMaxRows + r) * kStatStride;  // one sector
        const float4 st4 = in ? __ldcg(reinterpret_cast<const float4*>(st_row)) : make_float4(-INFINITY, 0.f, 0.f, 0.f);
        const float l3 = in ? __ldcg(st_row + 4) : 0.f;
        ms[k] = st4.x;
        ls[k] = (st4.y + st4.z) + (st4.w + l3);
        v[k] = in ? __ldcg(reinterpret_cast<const float4*>(p.p_o + (item * kMaxRows + r) * D) + quad)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      // the batch's max first, so the eight weights are independent
      float mb = ms[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) mb = fmaxf(mb, ms[k]);
      if (mb == -INFINITY) continue;
      MergeState bt;
      bt.m = mb;
      bt.l = 0.f;
      bt.a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float w = fast_exp2(ms[k] - mb);  // 0 for an empty split (-inf)
        bt.a.x += v[k].x * w;
        bt.a.y += v[k].y * w;
        bt.a.z += v[k].z * w;
        bt.a.w += v[k].w * w;
        bt.l += ls[k] * w;
      }
      merge_combine(st, bt);
    }
  };
  auto finish = [&](const GroupInfo& grp, int r, MergeState st) {
    if (SPW == 2) {
      MergeState o;
      o.m = __shfl_xor_sync(0xffffffffu, st.m, 16);
      o.l = __shfl_xor_sync(0xffffffffu, st.l, 16);
      o.a.x = __shfl_xor_sync(0xffffffffu, st.a.x, 16);
      o.a.y = __shfl_xor_sync(0xffffffffu, st.a.y, 16);
      o.a.z = __shfl_xor_sync(0xffffffffu, st.a.z, 16);
      o.a.w = __shfl_xor_sync(0xffffffffu, st.a.w, 16);
      merge_combine(st, o);
    }
    const int hh = r / grp.nq, qi = grp.q0 + r % grp.nq;
    const int dd = paired_dim<PAIR>(p, hh, quad * 4);
    if (slot == 0 && dd >= 0) {
      const float inv = st.l > 0.f ? 1.f / st.l : 0.f;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(seq_row0(p, grp.b) + qi) * p.o_st +
                           static_cast<int64_t>(grp.h * p.n_rep + hh) * p.o_sh + dd;
      uint2 pk;
      pk.x = pack_bf16(st.a.x * inv, st.a.y * inv);
      pk.y = pack_bf16(st.a.z * inv, st.a.w * inv);
      *reinterpret_cast<uint2*>(dst) = pk;
    }
  };

  // wide rows: one CTA each
  for (int u = cta; u < wide_units; u += n_ctas) {
    const GroupInfo grp = u == cta ? pre_w : p.merge_list[u / RU];
    const int r = u % RU;
    if (r >= p.n_rep * grp.nq) continue;  // uniform per CTA
    MergeState st;
    stream(grp, r, warp * SPW + slot, NWARP * SPW, st);
    s_st[warp * 32 + lane] = st;
    __syncthreads();
    if (warp == 0) {
      // the warps' states: common max first, then independent weights
      float m = st.m;
#pragma unroll
      for (int w = 1; w < NWARP; ++w) m = fmaxf(m, s_st[w * 32 + lane].m);
      if (m != -INFINITY) {
        MergeState tot;
        tot.m = m;
        tot.l = 0.f;
        tot.a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
          const MergeState o = s_st[w * 32 + lane];
          const float g = fast_exp2(o.m - m);  // 0 for an empty state (-inf)
          tot.a.x += o.a.x * g;
          tot.a.y += o.a.y * g;
          tot.a.z += o.a.z * g;
          tot.a.w += o.a.w * g;
          tot.l += o.l * g;
        }
        st = tot;
      }
      finish(grp, r, st);
    }
    __syncthreads();
  }
  // narrow rows: one warp each
  const int u0 = cta * NWARP + warp;
  for (int u = u0; u < narrow_units; u += n_ctas * NWARP) {
    const GroupInfo grp = u == u0 ? pre_n : p.merge_list[p.max_groups - 1 - u / RU];
    const int r = u % RU;
    if (r >= p.n_rep * grp.nq) continue;  // uniform per warp
    MergeState st;
    stream(grp, r, slot, SPW, st);
    finish(grp, r, st);
  }
}

// Grid-wide barrier of the persistent verify kernel: its grid is at most one CTA per
// SM at one CTA per SM, so every CTA is resident once the kernel's CTAs run (and no CTA
// with pages ever waits for a spare block).  The arrival counter grows by n_ctas (the
// plan's arrivals: the CTAs with pages, plus the merging spare blocks) per launch (the
// plan zeroes it); every arrival of a launch follows the previous launch's completion, so
// a CTA that arrives as number `old` waits for the counter to reach the next multiple of
// n_ctas.  Only CTAs with merge work wait.  Called by one thread per CTA; bounded: false
// after `limit_ns` (~1 s by default).
SD_DEV bool grid_barrier(unsigned long long* counter, unsigned n_ctas, bool wait, uint64_t limit_ns = kWaitLimitNs) {
  __threadfence();  // this CTA's partials before its arrival
  const unsigned long long old = atomicAdd(counter, 1ull);
  if (!wait) return true;
  const unsigned long long target = (old / n_ctas + 1) * n_ctas;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned long long now;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(now) : "l"(counter) : "memory");
    if (now >= target) break;
    if (globaltimer_ns() - t0 > limit_ns) return false;
    __nanosleep(64);
  }
  return true;
}

// ---------------------------------------------------------------- cluster-mode merge
// After its item every CTA of a cluster holds, in its own shared memory, the split partial
// of its key range: per query row the unnormalised O row (D floats at cl_o + row * D) and
// the statistics (row max, four key-quarter sums at cl_st + row * kStatStride); a CTA
// without pages holds zero rows with max -inf.  After a cluster barrier, CTA rank cr owns
// rows cr, cr + CS, ... and combines the CS partials of each through distributed shared
// memory: every warp issues the loads of all its (row, peer) units at once, then combines
// them max-first; the warps' states meet in this CTA's scratch `s_st` (no peer reads it).
// Once its loads are in, the CTA arrives on the cluster's exit barrier, so peers never wait
// for its global work.  A group on one cluster writes the output row; a group on c > 1
// clusters writes the cluster's partial of the row to the workspace (slot = cluster
// index), and the row's last-arriving cluster (per-row ticket, counted after a release
// fence) combines the c partials, writes the output and resets the ticket.
constexpr int kClusterMaxOwn = 4;   // rows per CTA: at most 32 rows over clusters of >= 8 CTAs
constexpr int kClusterMaxUnits = 4;  // (row, peer) units per warp step: 32 units over >= 8 warps

template <int D, int NWARP, bool PAIR>
SD_DEV void cluster_merge(const AttnParams& p, const CtaDesc& cd, const float* cl_o, const float* cl_st,
                          MergeState* s_st, int warp, int lane) {
  constexpr int NQ = D / 4;     // dim quads: lanes per row
  constexpr int SPW = 32 / NQ;  // units per warp step
  // a CTA has at most 32 units: 32 rows over clusters of 8 or 16 CTAs
  static_assert(NWARP * SPW * kClusterMaxUnits >= 32, "units of a CTA in one step");
  const int quad = lane % NQ, slot = lane / NQ;
  const int CS = static_cast<int>(cluster_nctarank()), cr = static_cast<int>(cluster_ctarank());
  const WorkItem& g = cd.items[0];
  const int R = p.n_rep * g.nq;
  const int own = R > cr ? (R - cr + CS - 1) / CS : 0;  // rows cr, cr + CS, ...
  const int units = own * CS;
  const uint32_t o_base = smem_u32(cl_o), st_base = smem_u32(cl_st);

  // all loads of this lane's units first (unit u = warp * SPW + slot + k * NWARP * SPW)
  float4 s4[kClusterMaxUnits], o4[kClusterMaxUnits];
  float l3[kClusterMaxUnits];
  int ju[kClusterMaxUnits];
#pragma unroll
  for (int k = 0; k < kClusterMaxUnits; ++k) {
    const int u = warp * SPW + slot + k * NWARP * SPW;
    ju[k] = -1;
    if (u < units) {
      const int j = u / CS, peer = u - j * CS;
      const int row = cr + j * CS;
      ju[k] = j;
      s4[k] = dsmem_ld4(dsmem_addr(st_base + row * kStatStride * 4, peer));
      l3[k] = dsmem_ld(dsmem_addr(st_base + (row * kStatStride + 4) * 4, peer));
      o4[k] = dsmem_ld4(dsmem_addr(o_base + (row * D + 4 * quad) * 4, peer));
    }
  }
  // per row: the max of this lane's units first, then independent weights
  MergeState st[kClusterMaxOwn];
#pragma unroll
  for (int j = 0; j < kClusterMaxOwn; ++j) {
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kClusterMaxUnits; ++k)
      if (ju[k] == j) m = fmaxf(m, s4[k].x);
    st[j].m = m;
    st[j].l = 0.f;
    st[j].a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m != -INFINITY) {
#pragma unroll
      for (int k = 0; k < kClusterMaxUnits; ++k) {
        if (ju[k] != j) continue;
        const float w = fast_exp2(s4[k].x - m);  // 0 for an empty partial (-inf)
        st[j].l += ((s4[k].y + s4[k].z) + (s4[k].w + l3[k])) * w;
        st[j].a.x += o4[k].x * w;
        st[j].a.y += o4[k].y * w;
        st[j].a.z += o4[k].z * w;
        st[j].a.w += o4[k].w * w;
      }
    }
    if (SPW == 2) {
      // head_dim 64: the warp's two unit slots, folded into slot 0
      MergeState o;
      o.m = __shfl_xor_sync(0xffffffffu, st[j].m, 16);
      o.l = __shfl_xor_sync(0xffffffffu, st[j].l, 16);
      o.a.x = __shfl_xor_sync(0xffffffffu, st[j].a.x, 16);
      o.a.y = __shfl_xor_sync(0xffffffffu, st[j].a.y, 16);
      o.a.z = __shfl_xor_sync(0xffffffffu, st[j].a.z, 16);
      o.a.w = __shfl_xor_sync(0xffffffffu, st[j].a.w, 16);
      merge_combine(st[j], o);
    }
    if (j < own) s_st[(j * NWARP + warp) * 32 + lane] = st[j];
  }
  __syncthreads();  // every DSMEM load of this CTA has returned
  cluster_arrive();  // the peers may leave once they are done too
  if (warp >= own || slot != 0) return;
  // warp j finishes row cr + j * CS: the warps' states, common max first
  const int j = warp, row = cr + j * CS;
  MergeState tot;
  {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) m = fmaxf(m, s_st[(j * NWARP + w) * 32 + lane].m);
    tot.m = m;
    tot.l = 0.f;
    tot.a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        const MergeState o = s_st[(j * NWARP + w) * 32 + lane];
        const float wt = fast_exp2(o.m - m);
        tot.a.x += o.a.x * wt;
        tot.a.y += o.a.y * wt;
        tot.a.z += o.a.z * wt;
        tot.a.w += o.a.w * wt;
        tot.l += o.l * wt;
      }
    }
  }
  const unsigned lanes = NQ == 32 ? 0xffffffffu : 0x0000ffffu;
  if (cd.cl_count > 1) {
    // this cluster's partial of the row, then the row's ticket
    const int cl = static_cast<int>(cluster_id_x());
    const int64_t slot_row = static_cast<int64_t>(cl) * kMaxRows + row;
    reinterpret_cast<float4*>(p.p_o + slot_row * D)[quad] = tot.a;
    if (quad == 0) {
      p.p_stat[slot_row * kStatStride] = tot.m;
      p.p_stat[slot_row * kStatStride + 1] = tot.l;
    }
    __threadfence();
    __syncwarp(lanes);
    int last = 0;
    if (quad == 0) {
      const int old = atomicAdd(&p.tickets[static_cast<int64_t>(cd.cl_first) * kMaxRows + row], 1);
      last = old == cd.cl_count - 1;
    }
    last = __shfl_sync(lanes, last, 0);
    if (!last) return;
    __threadfence();
    float ms[kClusterMaxSlots], ls[kClusterMaxSlots];
    float4 os[kClusterMaxSlots];
#pragma unroll
    for (int c = 0; c < kClusterMaxSlots; ++c) {
      ms[c] = -INFINITY;
      ls[c] = 0.f;
      os[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < cd.cl_count) {
        const int64_t sr = static_cast<int64_t>(cd.cl_first + c) * kMaxRows + row;
        ms[c] = __ldcg(p.p_stat + sr * kStatStride);
        ls[c] = __ldcg(p.p_stat + sr * kStatStride + 1);
        os[c] = __ldcg(reinterpret_cast<const float4*>(p.p_o + sr * D) + quad);
      }
    }
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < kClusterMaxSlots; ++c) m = fmaxf(m, ms[c]);
    tot.m = m;
    tot.l = 0.f;
    tot.a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int c = 0; c < kClusterMaxSlots; ++c) {
      const float wt = ms[c] == -INFINITY ? 0.f : fast_exp2(ms[c] - m);
      tot.l += ls[c] * wt;
      tot.a.x += os[c].x * wt;
      tot.a.y += os[c].y * wt;
      tot.a.z += os[c].z * wt;
      tot.a.w += os[c].w * wt;
    }
    if (quad == 0) p.tickets[static_cast<int64_t>(cd.cl_first) * kMaxRows + row] = 0;
  }
  const float inv = tot.l > 0.f ? 1.f / tot.l : 0.f;
  const int hh = row / g.nq, qi = g.q0 + row % g.nq;
  const int dd = paired_dim<PAIR>(p, hh, quad * 4);
  if (dd < 0) return;
  __nv_bfloat16* dst = p.out + static_cast<int64_t>(g.row0 + qi) * p.o_st +
                       static_cast<int64_t>(g.h * p.n_rep + hh) * p.o_sh + dd;
  uint2 pk;
  pk.x = pack_bf16(tot.a.x * inv, tot.a.y * inv);
  pk.y = pack_bf16(tot.a.z * inv, tot.a.w * inv);
  *reinterpret_cast<uint2*>(dst) = pk;
}

#include "verify_kernel.cuh"
static_assert(kTilePages == kPlanTilePages, "the plan and the verify kernel agree on the tile");

// ---------------------------------------------------------------- fp32 contiguous path
// CUDA-core kernel for the f32 dtype of the reference op (attention.cu:262-272).
// One CTA per (b, h, query row); keys in chunks of 128: warps compute the
// chunk's scores into shared memory, then threads over `d` accumulate P.V.
__global__ void __launch_bounds__(128) attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, float* __restrict__ out,
                                                       int H, int KV, int S, int T, int D, float sm_scale) {
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (H / KV);
  __shared__ float s_q[128];
  __shared__ float s_p[128];
  __shared__ float s_red[4];
  __shared__ float s_stat[2];
  const float* qrow = q + ((static_cast<int64_t>(b) * H + h) * S + i) * D;
  const float* kb = k + (static_cast<int64_t>(b) * KV + kvh) * T * D;
  const float* vb = v + (static_cast<int64_t>(b) * KV + kvh) * T * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) s_q[d] = qrow[d];
  __syncthreads();
  const int nvis = min(T, i + (T - S) + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
  for (int j0 = 0; j0 < nvis; j0 += 128) {
    const int nc = min(128, nvis - j0);
    for (int jj = warp; jj < nc; jj += 4) {
      const float* kr = kb + static_cast<int64_t>(j0 + jj) * D;
      float part = 0.f;
      for (int d = lane; d < D; d += 32) part += s_q[d] * kr[d];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) s_p[jj] = part * sm_scale;
    }
    __syncthreads();
    float mx = (threadIdx.x < nc) ? s_p[threadIdx.x] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      const float cm = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
      s_stat[0] = fmaxf(m_run, cm);
    }
    __syncthreads();
    const float m_new = s_stat[0];
    float e = 0.f;
    if (threadIdx.x < nc) {
      e = expf(s_p[threadIdx.x] - m_new);
      s_p[threadIdx.x] = e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    __syncthreads();
    if (lane == 0) s_red[warp] = e;
    __syncthreads();
    const float csum = s_red[0] + s_red[1] + s_red[2] + s_red[3];
    const float alpha = expf(m_run - m_new);
    l_run = l_run * alpha + csum;
    if (threadIdx.x < D) {
      float a = acc * alpha;
      for (int jj = 0; jj < nc; ++jj) a += s_p[jj] * vb[static_cast<int64_t>(j0 + jj) * D + threadIdx.x];
      acc = a;
    }
    m_run = m_new;
    __syncthreads();
  }
  if (threadIdx.x < D) {
    out[((static_cast<int64_t>(b) * H + h) * S + i) * D + threadIdx.x] = (l_run > 0.f) ? acc / l_run : 0.f;
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 3-D map over a contiguous (B*KV, T, D) bf16 tensor with a {64, 16, 1} box and
// 128-byte swizzle; out-of-range rows read as zero.
static int encode_kv_map(CUtensorMap* map, const void* base, int planes, int T, int D) {
  auto fn = get_encode_fn();
  if (!fn) return fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(T) * D * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kPage), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPECDEC_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SPECDEC_OK;
}

// 2-D map over `n_rows` contiguous rows of `row_bytes` bytes (64-bit elements, no
// swizzle) whose box is one row: the shape tile::gather4 loads fetch four rows of.
static int encode_rows_map(CUtensorMap* map, const void* base, uint64_t n_rows, uint32_t row_bytes) {
  auto fn = get_encode_fn();
  if (!fn) return fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (row_bytes % 16 || row_bytes / 8 > 256 || n_rows == 0)
    return fail(SPECDEC_ERR_INVALID, "row map: bad row size %u", row_bytes);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 8), static_cast<cuuint64_t>(n_rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {row_bytes / 8, 1};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPECDEC_ERR_INVALID, "cuTensorMapEncodeTiled (rows) failed (%d)", static_cast<int>(r));
  return SPECDEC_OK;
}

// Query positions per work item: rows (n_rep x positions) must fit the verify
// kernel's row tile of 32 (TMEM columns of S and O).
static int q_tile_for(int n_rep, int D) {
  (void)D;
  constexpr int rows = 32;
  return n_rep >= rows ? 1 : rows / n_rep;
}
static int tile_pages_for(int D) {
  (void)D;
  return kTilePages;
}

// dynamic shared memory opt-in, once per (kernel, device)
template <typename K>
static void set_smem_attr(K kern, int bytes, bool* done_per_device) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!done_per_device[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done_per_device[dev] = true;
  }
}

// Launches with programmatic stream serialization when `pdl` is set: the kernel may
// start (and run the part before its grid_dep_wait) while the previous kernel on the
// stream finishes.  Kernels launched this way read and write device data only after
// grid_dep_wait().
template <typename... KArgs, typename... Args>
static int launch_k(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                    bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return after_launch(what);
}

template <int NR, bool VF8, bool TMAP, int D, bool PP, bool PAIR = false>
static int launch_verify(const AttnParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                         const CUtensorMap& smap, cudaStream_t st,
                         bool pdl) {
  using Geo = V3Geom<NR < 16 ? 16 : NR, VF8, D>;
  if (p.cluster_size > 0) {
    // cluster mode: num_clusters clusters of cluster_size CTAs, one item per CTA
    auto kern = verify_kernel<NR, VF8, TMAP, D, PP, true, PAIR>;
    static bool attr[64] = {};
    set_smem_attr(kern, Geo::SMEM, attr);
    // clusters of 16 are a non-portable size: each kernel form opts in before its first such
    // launch (resident_clusters does so for the form it measures)
    static bool wide[64] = {};
    int dev = 0;
    if (p.cluster_size > 8 && cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64 && !wide[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return fail(SPECDEC_ERR_CUDA, "verify_kernel: clusters of %d CTAs are not available", p.cluster_size);
      wide[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.num_clusters * p.cluster_size);
    cfg.blockDim = dim3(v3_threads<VF8>());
    cfg.dynamicSmemBytes = Geo::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = static_cast<unsigned>(p.cluster_size);
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, kmap, vmap, smap);
    if (e != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "verify_kernel (clusters) launch: %s", cudaGetErrorString(e));
    return after_launch("verify_kernel");
  }
  static bool attr[64] = {};
  set_smem_attr(verify_kernel<NR, VF8, TMAP, D, PP, false, PAIR>, Geo::SMEM, attr);
  // persistent: one CTA per SM, the plan's C = target_items / 4 ranges
  const int grid = p.target_items / 4;
  return launch_k("verify_kernel", verify_kernel<NR, VF8, TMAP, D, PP, false, PAIR>, dim3(grid), dim3(v3_threads<VF8>()),
                  Geo::SMEM, st, pdl, p, kmap, vmap, smap);
}

// Clusters of `cs` CTAs of this verify kernel that can be resident at once (cached per
// device); 0 when the device cannot run such clusters.
template <int NR, bool VF8, bool TMAP, int D, bool PP>
static int resident_clusters(int cs) {
  using Geo = V3Geom<NR < 16 ? 16 : NR, VF8, D>;
  static int cache[64][2] = {};
  static bool known[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int ci = cs == 16 ? 1 : 0;
  if (known[dev][ci]) return cache[dev][ci];
  auto kern = verify_kernel<NR, VF8, TMAP, D, PP, true>;
  static bool attr[64] = {};
  set_smem_attr(kern, Geo::SMEM, attr);
  if (cs > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    known[dev][ci] = true;
    return cache[dev][ci] = 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs);
  cfg.blockDim = dim3(v3_threads<VF8>());
  cfg.dynamicSmemBytes = Geo::SMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(cs);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  known[dev][ci] = true;
  return cache[dev][ci] = n;
}

// CTAs of the persistent verify kernel: the caller's SM budget, at most the device's
// SM count (its CTAs meet at a grid barrier, so all of them must be resident at once)
static int sm_budget(int requested) {
  const int dev = device_sm_count();
  return (requested > 0 && requested < dev) ? requested : dev;
}

static int target_items_for(int num_sms, int occ) {
  // the plan makes at most ~4 waves of one-CTA-per-SM items (see plan_kernel);
  // this bound sizes the workspace and never depends on a device query
  (void)occ;
  return num_sms * 4;
}

// Records a profiling event; under stream capture it becomes an external
// event node so the graph's replays can be timed.
static int record_event(void* ev, cudaStream_t stream) {
  if (ev == nullptr) return SPECDEC_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "cudaStreamIsCapturing failed");
  const cudaError_t e = (cs == cudaStreamCaptureStatusActive)
                            ? cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev), stream, cudaEventRecordExternal)
                            : cudaEventRecord(static_cast<cudaEvent_t>(ev), stream);
  if (e != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "event record: %s", cudaGetErrorString(e));
  return SPECDEC_OK;
}

// softmax form per row class: two warp groups on alternate tiles (true) or one
// group on every tile with the rows split in halves (false)
constexpr bool kTwoGroup16 = true;
constexpr bool kTwoGroup32 = false;
// in cluster mode a CTA takes at most a few tiles: two groups on alternate tiles run them
// side by side
constexpr bool kTwoGroup32Clusters = false;

template <int D, bool VF8, bool TMAP, bool PAIR = false>
static int run_attention(AttnParams p, const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& smap,
                         bool build_plan,
                         cudaStream_t stream, void* ev_begin = nullptr, void* ev_end = nullptr) {
  if (build_plan) {
    plan_kernel<<<1, 1024, 0, stream>>>(p);
    if (int rc = after_launch("plan_kernel")) return rc;
  }
  if (int rc = record_event(ev_begin, stream)) return rc;
  // programmatic launches overlap each kernel's start with its predecessor's tail;
  // profiling events between the kernels need ordinary launches
  const bool pdl = ev_begin == nullptr && ev_end == nullptr;
  const int rows_max = p.n_rep * (p.q_tile < p.max_q_len ? p.q_tile : p.max_q_len);
  const int rc = rows_max <= 8    ? launch_verify<8, VF8, TMAP, D, true, PAIR>(p, kmap, vmap, smap, stream, pdl)
                 : rows_max <= 16 ? launch_verify<16, VF8, TMAP, D, kTwoGroup16, PAIR>(p, kmap, vmap, smap, stream, pdl)
                 : p.cluster_size > 0
                     ? launch_verify<32, VF8, TMAP, D, kTwoGroup32Clusters, PAIR>(p, kmap, vmap, smap, stream, pdl)
                     : launch_verify<32, VF8, TMAP, D, kTwoGroup32, PAIR>(p, kmap, vmap, smap, stream, pdl);
  if (rc) return rc;
  return record_event(ev_end, stream);
}

// Cluster mode for small batches: every group of the batch (sequence x query tile x KV head)
// gets clusters of its own, so the split reduction stays inside clusters (distributed shared
// memory) instead of a grid barrier and a global merge.  `hint`: 0 the library's choice
// (clusters of 16, else 8), 1 no clusters, 8 or 16 that size.  Sets p.cluster_size and
// p.num_clusters (0 = the persistent grid).
// The library's own choice (hint 0) takes clusters only where they are measured to win:
// every group on one cluster with at most one 128-key tile per CTA (no cross-cluster step,
// no second tile), which needs the host's bound on the context length.  On this B200 at
// most 7 clusters of 16 and 15 of 8 CTAs are resident, so an 8192-token sequence (64 tiles
// per KV head) would need two tiles per CTA or several clusters per group; the persistent
// grid (128 CTAs of one tile) is faster there.
template <int NR, bool VF8, bool TMAP, int D, bool PP>
static void choose_clusters_nr(AttnParams& p, int hint, int sms) {
  p.cluster_size = 0;
  p.num_clusters = 0;
  if (hint == 1 || p.max_groups > kClusterMaxGroups) return;
  if (hint == 0 && p.max_ctx_hint <= 0) return;
  const int tiles_max = (p.max_ctx_hint + kPlanTilePages * kPage - 1) / (kPlanTilePages * kPage);
  const int sizes[2] = {16, 8};
  for (int cs : sizes) {
    if (hint != 0 && hint != cs) continue;
    if (hint == 0 && tiles_max > cs) continue;
    const int nc = std::min(resident_clusters<NR, VF8, TMAP, D, PP>(cs), sms / cs);
    if (nc >= p.max_groups && nc > 0) {
      p.cluster_size = cs;
      p.num_clusters = nc;
      return;
    }
  }
}

template <int D, bool VF8, bool TMAP>
static void choose_clusters(AttnParams& p, int hint, int sms) {
  const int rows_max = p.n_rep * (p.q_tile < p.max_q_len ? p.q_tile : p.max_q_len);
  if (rows_max <= 8)
    choose_clusters_nr<8, VF8, TMAP, D, true>(p, hint, sms);
  else if (rows_max <= 16)
    choose_clusters_nr<16, VF8, TMAP, D, kTwoGroup16>(p, hint, sms);
  else
    choose_clusters_nr<32, VF8, TMAP, D, kTwoGroup32Clusters>(p, hint, sms);
}

static int fill_workspace(AttnParams& p, void* ws, size_t ws_bytes, int B, int KV, int D, int num_sms, int occ) {
  const int target = target_items_for(num_sms, occ);
  const WsLayout w = ws_layout(B, KV, p.max_qtiles, D, target);
  if (ws == nullptr || ws_bytes < w.total)
    return fail(SPECDEC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required", ws_bytes,
                w.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(SPECDEC_ERR_INVALID, "workspace must be 256-byte aligned");
  uint8_t* base = static_cast<uint8_t*>(ws);
  p.hdr = reinterpret_cast<PlanHeader*>(base);
  p.items = reinterpret_cast<WorkItem*>(base + w.items);
  p.groups = reinterpret_cast<GroupInfo*>(base + w.groups);
  p.cta_first = reinterpret_cast<int32_t*>(base + w.ctas);
  p.cdesc = reinterpret_cast<CtaDesc*>(base + w.cdesc);
  p.merge_list = reinterpret_cast<GroupInfo*>(base + w.mlist);
  p.tickets = reinterpret_cast<int32_t*>(base + w.tickets);
  p.p_stat = reinterpret_cast<float*>(base + w.lse);
  p.p_o = reinterpret_cast<float*>(base + w.po);
  p.max_items = w.max_items;
  p.max_groups = w.max_groups;
  p.target_items = target;
  return SPECDEC_OK;
}

static int occupancy_for(int D, bool vf8, bool tmap) {
  (void)D;
  (void)vf8;
  (void)tmap;
  return 1;  // both split kernels run one CTA per SM
}

static int validate_paged(const SpecdecAttnArgs* a) {
  if (!a) return fail(SPECDEC_ERR_INVALID, "args is NULL");
  const SpecdecPagedKV& kv = a->kv;
  const SpecdecBatch& bt = a->batch;
  if (!a->q || !a->out) return fail(SPECDEC_ERR_INVALID, "q and out must be device pointers");
  if (!bt.q_row0 || !bt.q_len || !bt.ctx_len) return fail(SPECDEC_ERR_INVALID, "batch arrays must be set");
  if (!kv.k_pool || !kv.v_pool || !kv.page_table) return fail(SPECDEC_ERR_INVALID, "kv pool pointers must be set");
  if (bt.num_seqs <= 0 || bt.num_q_heads <= 0 || kv.num_kv_heads <= 0)
    return fail(SPECDEC_ERR_INVALID, "num_seqs, num_q_heads and num_kv_heads must be positive");
  if (bt.num_q_heads % kv.num_kv_heads != 0) return fail(SPECDEC_ERR_INVALID, "query heads must divide KV heads");
  if (bt.num_q_heads / kv.num_kv_heads > 32)
    return fail(SPECDEC_ERR_UNSUPPORTED, "at most 32 query heads per KV head");
  if (kv.head_dim != 64 && kv.head_dim != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (kv.v_dtype != SPECDEC_BF16 && kv.v_dtype != SPECDEC_E4M3)
    return fail(SPECDEC_ERR_UNSUPPORTED, "v_dtype must be SPECDEC_BF16 or SPECDEC_E4M3");
  if (kv.v_dtype == SPECDEC_E4M3 && kv.head_dim != 128)
    return fail(SPECDEC_ERR_UNSUPPORTED, "E4M3 V needs head_dim 128 (one scale group per head)");
  if (kv.v_dtype == SPECDEC_E4M3 && !kv.v_scale) return fail(SPECDEC_ERR_INVALID, "E4M3 V needs v_scale");
  if (bt.max_q_len <= 0) return fail(SPECDEC_ERR_INVALID, "max_q_len must be positive");
  if (kv.num_pages <= 0 || kv.max_pages_per_seq <= 0) return fail(SPECDEC_ERR_INVALID, "empty page pool");
  const uintptr_t al = reinterpret_cast<uintptr_t>(kv.k_pool) | reinterpret_cast<uintptr_t>(kv.v_pool) |
                       reinterpret_cast<uintptr_t>(kv.v_scale);
  if (al & 15u) return fail(SPECDEC_ERR_INVALID, "pool pointers must be 16-byte aligned");
  if ((a->q_stride_head | a->o_stride_head | a->q_stride_tok | a->o_stride_tok) & 3)
    return fail(SPECDEC_ERR_INVALID, "q/out strides must be multiples of 4 elements (8-byte vectors)");
  if ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->out)) & 7u)
    return fail(SPECDEC_ERR_INVALID, "q/out must be 8-byte aligned");
  return SPECDEC_OK;
}

// Paired heads (AttnParams::half_heads): head_dim 64 with bf16 V and an even number of KV
// heads whose query rows, for both heads of a pair, fit the 32-row tile: a 128-key tile then
// streams both heads' 2 KB page blocks (64 KB of K and V per tile instead of 32 KB).
static bool paired_geometry(int H, int KV, int D, bool vf8) {
  return D == 64 && !vf8 && KV % 2 == 0 && 2 * (H / KV) <= 32;
}

static AttnParams params_from(const SpecdecAttnArgs* a) {
  AttnParams p;
  memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.q_st = a->q_stride_tok;
  p.q_sh = a->q_stride_head;
  p.o_st = a->o_stride_tok;
  p.o_sh = a->o_stride_head;
  p.q_row0 = a->batch.q_row0;
  p.q_len = a->batch.q_len;
  p.ctx_len = a->batch.ctx_len;
  p.B = a->batch.num_seqs;
  p.H = a->batch.num_q_heads;
  p.KV = a->kv.num_kv_heads;
  p.n_rep = p.H / p.KV;
  int D = a->kv.head_dim;
  if (paired_geometry(p.H, p.KV, D, a->kv.v_dtype == SPECDEC_E4M3)) {
    p.half_heads = p.n_rep;
    p.KV /= 2;
    p.n_rep *= 2;
    D = 128;
  }
  p.max_q_len = a->batch.max_q_len;
  p.q_tile = q_tile_for(p.n_rep, D);
  p.tile_pages = tile_pages_for(D);
  p.max_qtiles = (p.max_q_len + p.q_tile - 1) / p.q_tile;
  p.k_pool = static_cast<const uint8_t*>(a->kv.k_pool);
  p.v_pool = static_cast<const uint8_t*>(a->kv.v_pool);
  p.v_scale = a->kv.v_scale;
  p.page_table = a->kv.page_table;
  p.num_pages = a->kv.num_pages;
  p.max_pages = a->kv.max_pages_per_seq;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.status = a->status;
  p.max_ctx_hint = a->batch.max_ctx_len;
  return p;
}

static int paged_entry(const SpecdecAttnArgs* a, cudaStream_t stream, bool plan_only) {
  if (int rc = validate_paged(a)) return rc;
  AttnParams p = params_from(a);
  const int D = p.half_heads > 0 ? 128 : a->kv.head_dim;  // paired heads run the 128-dim kernel
  const bool vf8 = a->kv.v_dtype == SPECDEC_E4M3;
  const int sms = sm_budget(a->num_sms);
  if (int rc = fill_workspace(p, a->workspace, a->workspace_bytes, p.B, p.KV, D, sms, occupancy_for(D, vf8, false)))
    return rc;
  const int hint = a->cluster_size;
  if (hint != 0 && hint != 1 && hint != 8 && hint != 16)
    return fail(SPECDEC_ERR_INVALID, "cluster_size must be 0 (automatic), 1 (none), 8 or 16");
  if (D == 128) {
    if (vf8)
      choose_clusters<128, true, false>(p, hint, sms);
    else
      choose_clusters<128, false, false>(p, hint, sms);
  } else {
    choose_clusters<64, false, false>(p, hint, sms);
  }
  if (plan_only) {
    plan_kernel<<<1, 1024, 0, stream>>>(p);
    return after_launch("plan_kernel");
  }
  // page-row maps over the pools for the kernel's four-row gathers: K (and bf16 V) as
  // rows of 128 bytes x 16 tokens = one dim half of a page-head block (paired heads: one
  // head's block of a page-pair block), E4M3 V as one 2048-byte row per page-head block,
  // scales as one 64-byte row
  const int KH = D / 64;
  const uint64_t blocks = static_cast<uint64_t>(a->kv.num_pages) * p.KV;
  CUtensorMap kmap, vmap, smap;
  memset(&smap, 0, sizeof(smap));
  if (int rc = encode_rows_map(&kmap, a->kv.k_pool, blocks * KH, 2048)) return rc;
  if (int rc = encode_rows_map(&vmap, a->kv.v_pool, vf8 ? blocks : blocks * KH, 2048)) return rc;
  if (vf8) {
    if (int rc = encode_rows_map(&smap, a->kv.v_scale, blocks, 64)) return rc;
  }
  const bool build = a->reuse_plan == 0;
  // early loads need a plan from an earlier call (one built now is written by the
  // kernel right before) and the caller's promise about the history
  p.early_loads = (!build && a->history_ready != 0) ? 1 : 0;
  void* eb = a->split_event_begin;
  void* ee = a->split_event_end;
  if (p.half_heads > 0) return run_attention<128, false, false, true>(p, kmap, vmap, smap, build, stream, eb, ee);
  if (D == 128) {
    return vf8 ? run_attention<128, true, false>(p, kmap, vmap, smap, build, stream, eb, ee)
               : run_attention<128, false, false>(p, kmap, vmap, smap, build, stream, eb, ee);
  }
  return run_attention<64, false, false>(p, kmap, vmap, smap, build, stream, eb, ee);
}

}  // namespace sd

using namespace sd;

extern "C" size_t specdec_attn_workspace_bytes(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                               int32_t head_dim, int32_t max_q_len, int32_t num_sms) {
  if (num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_q_len <= 0 || num_q_heads % num_kv_heads)
    return 0;
  int n_rep = num_q_heads / num_kv_heads, kv = num_kv_heads, d = head_dim;
  if (paired_geometry(num_q_heads, num_kv_heads, head_dim, false)) {  // head_dim 64 is bf16 V
    n_rep *= 2;
    kv /= 2;
    d = 128;
  }
  const int qt = q_tile_for(n_rep, d);
  const int max_qtiles = (max_q_len + qt - 1) / qt;
  const int sms = num_sms > 0 ? num_sms : device_sm_count();
  // occupancy is not known without a device query; size for 4 CTAs per SM (an upper bound)
  const int target = target_items_for(sms, 4);
  return ws_layout(num_seqs, kv, max_qtiles, d, target).total;
}

extern "C" int specdec_attn_launch_shape(const SpecdecAttnArgs* a, int32_t* grid, int32_t* cluster_size) {
  if (int rc = validate_paged(a)) return rc;
  if (!grid || !cluster_size) return fail(SPECDEC_ERR_INVALID, "grid and cluster_size must be set");
  AttnParams p = params_from(a);
  const int D = p.half_heads > 0 ? 128 : a->kv.head_dim;
  const bool vf8 = a->kv.v_dtype == SPECDEC_E4M3;
  const int sms = sm_budget(a->num_sms);
  const int target = target_items_for(sms, 0);
  p.max_groups = ws_layout(p.B, p.KV, p.max_qtiles, D, target).max_groups;
  const int hint = a->cluster_size;
  if (hint != 0 && hint != 1 && hint != 8 && hint != 16)
    return fail(SPECDEC_ERR_INVALID, "cluster_size must be 0 (automatic), 1 (none), 8 or 16");
  if (D == 128) {
    if (vf8)
      choose_clusters<128, true, false>(p, hint, sms);
    else
      choose_clusters<128, false, false>(p, hint, sms);
  } else {
    choose_clusters<64, false, false>(p, hint, sms);
  }
  *grid = p.cluster_size > 0 ? p.num_clusters * p.cluster_size : target / 4;
  *cluster_size = p.cluster_size;
  return SPECDEC_OK;
}

extern "C" int specdec_ragged_plan(const SpecdecAttnArgs* args, specdec_stream_t stream) {
  return paged_entry(args, reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int specdec_paged_attention(const SpecdecAttnArgs* args, specdec_stream_t stream) {
  return paged_entry(args, reinterpret_cast<cudaStream_t>(stream), false);
}

// ---------------------------------------------------------------- no-allocation variant
// Some callers cannot hand this library any scratch memory: a plugin host that
// owns every byte of device memory and passes a plugin only its inputs, outputs
// and a stream, or an FFI binding (cgo, JNI, a C caller) that has no CUDA
// allocator and must not call cudaMalloc itself.  For them the paged attention
// call can use a fixed scratch area compiled into this library instead of the
// caller's workspace.  The area is a file-scope device array of
// kStaticScratchBytes (32 MiB), so every GPU that loads the library keeps those
// 32 MiB until the process exits.  Batches whose plan and split partials need
// more than that are rejected with SPECDEC_ERR_WORKSPACE.
constexpr size_t kStaticScratchBytes = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Host code cannot use g_static_scratch's name as a device address (on the host it
// is only a stand-in symbol).  The device address is looked up once per device, with
// that device current, and cached together with the CUDA context it belongs to: a call
// made in another context on the same device (after cudaDeviceReset, or from a caller
// that manages its own contexts) looks the address up again instead of using a stale one.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
static CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  }
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

static int static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  static CUcontext owner[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SPECDEC_ERR_CUDA, "no current CUDA device for the static scratch");
  const CUcontext ctx = current_context();  // NULL before the runtime's first use of the device
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr || ctx == nullptr || owner[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);  // makes the context current if needed
    if (e != cudaSuccess || p == nullptr)
      return fail(SPECDEC_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    addr[dev] = p;
    owner[dev] = current_context();
  }
  *out = addr[dev];
  return SPECDEC_OK;
}

extern "C" int specdec_paged_attention_noalloc(const SpecdecAttnArgs* args, specdec_stream_t stream) {
  if (int rc = validate_paged(args)) return rc;
  // the same size a caller workspace would need (head_dim-64 KV-head pairs included)
  const size_t need =
      specdec_attn_workspace_bytes(args->batch.num_seqs, args->batch.num_q_heads, args->kv.num_kv_heads,
                                   args->kv.head_dim, args->batch.max_q_len, sm_budget(args->num_sms));
  if (need > kStaticScratchBytes)
    return fail(SPECDEC_ERR_WORKSPACE,
                "this batch needs %zu bytes of scratch; the static scratch of the no-allocation entry point "
                "holds %zu bytes (use specdec_paged_attention with a caller workspace)",
                need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  SpecdecAttnArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kStaticScratchBytes;
  a.reuse_plan = 0;  // the shared scratch may hold another call's plan: always rebuild it
  return paged_entry(&a, reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" size_t specdec_attention_workspace_bytes(int32_t B, int32_t H, int32_t KV, int32_t S, int32_t D,
                                                    int32_t num_sms) {
  return specdec_attn_workspace_bytes(B, H, KV, D, S, num_sms);
}

// The contiguous op: bf16 / f32 K and V (v_scale NULL), or bf16 K with E4M3 V codes and
// their per-token scales (v_scale set; the codes are widened inside the PV product).
static int contiguous_attention(const void* q, const void* k, const void* v, const float* v_scale, void* out,
                                int32_t dtype, int32_t B, int32_t H, int32_t KV, int32_t S, int32_t T, int32_t D,
                                void* workspace, size_t workspace_bytes, specdec_stream_t stream) {
  // argument checks of attention_cuda (attention.cu:245-260)
  if (!q || !k || !v || !out) return fail(SPECDEC_ERR_INVALID, "tensors must be CUDA");
  if (B <= 0 || H <= 0 || KV <= 0) return fail(SPECDEC_ERR_INVALID, "batch mismatch");
  if (H % KV != 0) return fail(SPECDEC_ERR_INVALID, "query heads must divide KV heads");
  if (D != 64 && D != 128) return fail(SPECDEC_ERR_INVALID, "head_dim must be 64 or 128");
  if (S <= 0 || T <= 0) return fail(SPECDEC_ERR_INVALID, "empty sequence");
  if (S > T) return fail(SPECDEC_ERR_INVALID, "query rows (%d) exceed keys (%d): early rows would see no key", S, T);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPECDEC_F32) {
    dim3 grid(S, H, B);
    attn_f32_kernel<<<grid, 128, 0, st>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                           static_cast<const float*>(v), static_cast<float*>(out), H, KV, S, T, D,
                                           1.0f / sqrtf(static_cast<float>(D)));
    return after_launch("attn_f32_kernel");
  }
  if (dtype != SPECDEC_BF16) return fail(SPECDEC_ERR_INVALID, "attention supports float32 and bfloat16");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u)
    return fail(SPECDEC_ERR_INVALID, "k and v must be 16-byte aligned for TMA");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 7u)
    return fail(SPECDEC_ERR_INVALID, "q and out must be 8-byte aligned");
  AttnParams p;
  memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.q_st = D;
  p.q_sh = static_cast<int64_t>(S) * D;
  p.o_st = D;
  p.o_sh = static_cast<int64_t>(S) * D;
  p.uni_q_len = S;
  p.uni_ctx_len = T;
  p.uni_row_stride = H * S;
  p.B = B;
  p.H = H;
  p.KV = KV;
  p.n_rep = H / KV;
  if (p.n_rep > kMaxRows) return fail(SPECDEC_ERR_UNSUPPORTED, "more than %d query heads per KV head", kMaxRows);
  if (p.n_rep > 32) return fail(SPECDEC_ERR_UNSUPPORTED, "at most 32 query heads per KV head");
  p.max_q_len = S;
  p.q_tile = q_tile_for(p.n_rep, D);
  p.tile_pages = tile_pages_for(D);
  p.max_qtiles = (S + p.q_tile - 1) / p.q_tile;
  p.num_pages = 1;
  p.max_pages = (T + kPage - 1) / kPage;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.v_scale = v_scale;
  if (v_scale && (reinterpret_cast<uintptr_t>(v_scale) & 3u)) return fail(SPECDEC_ERR_INVALID, "v_scale must be 4-byte aligned");
  const int sms = device_sm_count();
  if (int rc = fill_workspace(p, workspace, workspace_bytes, B, KV, D, sms, occupancy_for(D, false, true))) return rc;
  p.max_ctx_hint = T;
  if (v_scale)
    choose_clusters<128, true, true>(p, 0, sms);
  else if (D == 128)
    choose_clusters<128, false, true>(p, 0, sms);
  else
    choose_clusters<64, false, true>(p, 0, sms);
  CUtensorMap kmap, vmap;
  if (int rc = encode_kv_map(&kmap, k, B * KV, T, D)) return rc;
  if (v_scale != nullptr) {
    // E4M3 codes (B*KV, T, 128) bytes: one 16-token page of codes = one {128, 16, 1} box
    auto fn = get_encode_fn();
    if (!fn) return fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B * KV)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T) * D};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(D), static_cast<cuuint32_t>(kPage), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(&vmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(v), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPECDEC_ERR_INVALID, "cuTensorMapEncodeTiled (codes) failed (%d)", static_cast<int>(r));
  } else if (int rc = encode_kv_map(&vmap, v, B * KV, T, D)) {
    return rc;
  }
  CUtensorMap smap;
  memset(&smap, 0, sizeof(smap));
  if (v_scale != nullptr) return run_attention<128, true, true>(p, kmap, vmap, smap, true, st);
  if (D == 128) return run_attention<128, false, true>(p, kmap, vmap, smap, true, st);
  return run_attention<64, false, true>(p, kmap, vmap, smap, true, st);
}

extern "C" int specdec_attention(const void* q, const void* k, const void* v, void* out, int32_t dtype, int32_t B,
                                 int32_t H, int32_t KV, int32_t S, int32_t T, int32_t D, void* workspace,
                                 size_t workspace_bytes, specdec_stream_t stream) {
  return contiguous_attention(q, k, v, nullptr, out, dtype, B, H, KV, S, T, D, workspace, workspace_bytes, stream);
}

extern "C" int specdec_attention_fp8v(const void* q, const void* k, const void* v_codes, const float* v_scale,
                                      void* out, int32_t B, int32_t H, int32_t KV, int32_t S, int32_t T, int32_t D,
                                      void* workspace, size_t workspace_bytes, specdec_stream_t stream) {
  if (!v_scale) return fail(SPECDEC_ERR_INVALID, "v_scale must be set");
  if (D != 128) return fail(SPECDEC_ERR_UNSUPPORTED, "E4M3 V needs head_dim 128 (one scale group per head)");
  return contiguous_attention(q, k, v_codes, v_scale, out, SPECDEC_BF16, B, H, KV, S, T, D, workspace,
                              workspace_bytes, stream);
}

// ---------------------------------------------------------------- gather4 self-check
// One CTA loads rows r[0..3] of a [n_rows][2048 B] tensor and of a [n_rows][64 B]
// tensor with one tile::gather4 request each (the page-row loads of the attention
// kernel) and writes the 8192 + 256 bytes it received to `out`.
namespace sd {
__global__ void __launch_bounds__(128) gather4_selftest_kernel(const __grid_constant__ CUtensorMap big,
                                                               const __grid_constant__ CUtensorMap small, int4 rows,
                                                               uint8_t* out, int32_t* status) {
  __shared__ __align__(1024) uint8_t buf[8192 + 256];
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t pol = l2_evict_first();
    mbar_arrive_expect_tx(&bar, 8192 + 256);
    tma_gather4(buf, &big, 0, rows.x, rows.y, rows.z, rows.w, &bar, pol);
    tma_gather4(buf + 8192, &small, 0, rows.x, rows.y, rows.z, rows.w, &bar, pol);
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar, 0));
  if (!ok) {
    if (threadIdx.x == 0) raise_status(status, SPECDEC_STATUS_TIMEOUT);
    return;
  }
  for (int i = threadIdx.x; i < (8192 + 256) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(buf)[i];
}
}  // namespace sd

extern "C" int specdec_gather4_selftest(const void* big, const void* small, int64_t n_rows, const int32_t* rows,
                                        void* out, int32_t* status, specdec_stream_t stream) {
  if (!big || !small || !rows || !out || n_rows <= 0) return fail(SPECDEC_ERR_INVALID, "bad gather4 self-test arguments");
  for (int i = 0; i < 4; ++i)
    if (rows[i] < 0 || rows[i] >= n_rows) return fail(SPECDEC_ERR_INVALID, "gather4 self-test row out of range");
  if ((reinterpret_cast<uintptr_t>(big) | reinterpret_cast<uintptr_t>(small)) & 15u)
    return fail(SPECDEC_ERR_INVALID, "gather4 self-test tensors must be 16-byte aligned");
  CUtensorMap mb, ms;
  if (int rc = encode_rows_map(&mb, big, static_cast<uint64_t>(n_rows), 2048)) return rc;
  if (int rc = encode_rows_map(&ms, small, static_cast<uint64_t>(n_rows), 64)) return rc;
  sd::gather4_selftest_kernel<<<1, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      mb, ms, make_int4(rows[0], rows[1], rows[2], rows[3]), static_cast<uint8_t*>(out), status);
  return after_launch("gather4_selftest_kernel");
}

// ---------------------------------------------------------------- bounded-wait self-check
// Exercises the two waits every kernel of this library relies on with a short limit:
// mode 0 waits on an mbarrier that nothing arrives on (mbar_wait), mode 1 meets at the
// grid barrier with `n_ctas` arrivals expected from a grid of `grid` CTAs (grid_barrier).
// A wait that gives up raises SPECDEC_STATUS_TIMEOUT and the kernel returns; the time the
// first CTA spent waiting goes to *waited_ns.
namespace sd {
__global__ void __launch_bounds__(32) wait_selftest_kernel(int mode, unsigned long long* counter, unsigned n_ctas,
                                                           uint64_t limit_ns, int32_t* status,
                                                           unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  if (mode == 0) {
    ok = __all_sync(0xffffffffu, mbar_wait(&bar, 0, limit_ns));
  } else if (threadIdx.x == 0) {
    ok = grid_barrier(counter, n_ctas, true, limit_ns);
  }
  if (threadIdx.x == 0) {
    if (!ok) raise_status(status, SPECDEC_STATUS_TIMEOUT);
    if (blockIdx.x == 0 && waited_ns != nullptr) *waited_ns = globaltimer_ns() - t0;
  }
}
}  // namespace sd

extern "C" int specdec_wait_selftest(int32_t mode, void* counter, int32_t n_ctas, int32_t grid, int64_t limit_ns,
                                     int32_t* status, void* waited_ns, specdec_stream_t stream) {
  if (mode != 0 && mode != 1) return fail(SPECDEC_ERR_INVALID, "wait self-test mode must be 0 or 1");
  if (limit_ns < 1000 || limit_ns > 100000000) return fail(SPECDEC_ERR_INVALID, "wait limit must be 1 us .. 100 ms");
  if (grid < 1 || grid > 8) return fail(SPECDEC_ERR_INVALID, "wait self-test grid must be 1 .. 8 CTAs");
  if (mode == 1 && (counter == nullptr || n_ctas < 1))
    return fail(SPECDEC_ERR_INVALID, "grid-barrier self-test needs a zeroed device counter and n_ctas >= 1");
  if (mode == 0 && grid != 1) return fail(SPECDEC_ERR_INVALID, "mbarrier self-test runs one CTA");
  sd::wait_selftest_kernel<<<grid, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      mode, static_cast<unsigned long long*>(counter), static_cast<unsigned>(n_ctas),
      static_cast<uint64_t>(limit_ns), status, static_cast<unsigned long long*>(waited_ns));
  return after_launch("wait_selftest_kernel");
}
