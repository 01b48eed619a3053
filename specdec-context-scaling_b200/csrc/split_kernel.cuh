// split_kernel.cuh -- the split-KV attention kernel and the split merge (included by
// paged_attention.cu, which defines WorkItem / GroupInfo / PlanHeader / AttnParams).
//
// One CTA per work item, 1 CTA per SM:
//   warp 8      producer: page ids of the item in one coalesced round trip, then one
//               bulk-TMA copy per (page, part) into a ring of NST page slots
//               (full/empty mbarrier pair per slot).
//   warps 0-7   consumers: warp w serves row group g = w % G (16 query rows) and key
//               slice ks = w / G.  Key slice ks owns 4-page chunks c = ks, ks+KS, ...;
//               per chunk it runs QK^T for 64 keys (8 independent m16n8k16 chains),
//               one online-softmax update, and PV (64 MMAs), then frees the pages.
//   epilogue    the KS key slices of each row group merge through shared memory; the
//               item writes the normalised output (1 split) or a (partial O, lse) pair.
#pragma once

// (included inside namespace sd)
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kChunkPages = 4;

template <int D, bool VF8>
struct StageGeom {
  static constexpr int KB = D * 32;                 // 16 tokens x D x bf16 (multiple of 1024)
  static constexpr int VB = VF8 ? D * 16 : D * 32;  // E4M3 codes or bf16 (bf16 needs 1024 alignment)
  static constexpr int SB = VF8 ? 64 : 0;           // 16 fp32 scales
  static constexpr int SLOT = KB + VB + SB;
  static constexpr int NST = ((227 * 1024 - 2048) / SLOT) > 32 ? 32 : ((227 * 1024 - 2048) / SLOT);
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = NST * KB;
  static constexpr int S_OFF = V_OFF + NST * VB;
  static constexpr int SMEM = S_OFF + NST * SB + 1024;  // + alignment slack
  static constexpr int MERGE_ROW = D + 8;               // padded fp32 row in the merge area
  static constexpr int MERGE_WARP = 16 * MERGE_ROW * 4 + 256;
  static_assert(kConsumerWarps * MERGE_WARP <= NST * SLOT, "merge area fits in the ring");
  static_assert(NST >= 2 * kChunkPages, "ring holds two chunks");
};

template <int D, bool VF8, bool TMAP>
__global__ void __launch_bounds__(kThreads, 1) split_kernel(const AttnParams p,
                                                            const __grid_constant__ CUtensorMap kmap,
                                                            const __grid_constant__ CUtensorMap vmap) {
  using Geo = StageGeom<D, VF8>;
  constexpr int NST = Geo::NST;
  constexpr int NKK = D / 16;  // k-steps of QK^T
  constexpr int NNT = D / 8;   // n-tiles of PV
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[NST];
  __shared__ uint64_t empty_bar[NST];
  __shared__ int s_abort;
  __shared__ int s_issued;

  grid_dep_wait();
  grid_dep_launch();
  // the header and the item are independent loads: issue both, then test
  const int num_items = p.hdr->num_items;
  const WorkItem it = p.items[blockIdx.x];
  if (static_cast<int>(blockIdx.x) >= num_items) return;  // uniform per CTA
  const int R = p.n_rep * it.nq;
  int G = (R + 15) >> 4;
  if (G == 3) G = 4;
  const int KS = kConsumerWarps / G;
  const int npages = it.page_end - it.page_begin;
  const int nchunks = (npages + kChunkPages - 1) / kChunkPages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], G);
    }
    s_abort = 0;
    s_issued = 0;
    fence_barrier_init();
  }
  __syncthreads();

  float o[NNT][4];
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f, sref = 0.f;
  const int gq = lane >> 2, cq = lane & 3;
  const int g = warp % G;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------ producer warp
    if (TMAP && lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
    }
    const int32_t* pt = p.page_table + static_cast<int64_t>(it.b) * p.max_pages + it.page_begin;
    int li = 0;
    bool stop = false;
    for (int base = 0; base < npages && !stop; base += 32) {
      int my_page = 0;
      if (!TMAP && base + lane < npages) my_page = __ldg(pt + base + lane);
      const int n = min(32, npages - base);
      for (int j = 0; j < n; ++j, ++li) {
        const int page = __shfl_sync(0xffffffffu, my_page, j);
        const int slot = li % NST;
        bool ok = true;
        if (li >= NST) ok = mbar_wait(&empty_bar[slot], ((li / NST) - 1) & 1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0) {
            raise_status(p.status, SPECDEC_STATUS_TIMEOUT);
            atomicExch(&s_abort, 1);
          }
          stop = true;
          break;
        }
        if (__shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort), 0)) {
          stop = true;
          break;
        }
        if (lane == 0) {
          uint8_t* kd = smem + Geo::K_OFF + slot * Geo::KB;
          uint8_t* vd = smem + Geo::V_OFF + slot * Geo::VB;
          const int blk = it.page_begin + li;
          if (TMAP) {
            mbar_arrive_expect_tx(&full_bar[slot], Geo::KB + Geo::VB);
            const int plane = it.b * p.KV + it.h;
#pragma unroll
            for (int hf = 0; hf < D / 64; ++hf) {
              tma_load_3d(kd + hf * 2048, &kmap, hf * 64, blk * kPage, plane, &full_bar[slot]);
              tma_load_3d(vd + hf * 2048, &vmap, hf * 64, blk * kPage, plane, &full_bar[slot]);
            }
          } else if (page < 0 || page >= p.num_pages) {
            raise_status(p.status, SPECDEC_STATUS_BAD_PAGE);
            mbar_arrive(&full_bar[slot]);  // complete the phase without data
          } else {
            const int64_t ph = static_cast<int64_t>(page) * p.KV + it.h;
            mbar_arrive_expect_tx(&full_bar[slot], Geo::KB + Geo::VB + Geo::SB);
            bulk_g2s(kd, p.k_pool + ph * Geo::KB, Geo::KB, &full_bar[slot]);
            bulk_g2s(vd, p.v_pool + ph * Geo::VB, Geo::VB, &full_bar[slot]);
            if (VF8)
              bulk_g2s(smem + Geo::S_OFF + slot * Geo::SB, p.v_scale + ph * kPage, Geo::SB, &full_bar[slot]);
          }
        }
      }
    }
    if (lane == 0) s_issued = li;
  } else {
    // ------------------------------------------------ consumers
    const int ks = warp / G;
    const int qlen = seq_q_len(p, it.b);
    const int ctx = seq_ctx_len(p, it.b);
    const int row0 = seq_row0(p, it.b);
    const int ra = g * 16 + gq, rb = ra + 8;
    int lim_a = -1, lim_b = -1;
    uint32_t qf[NKK][4];
    {
      const __nv_bfloat16* qa = nullptr;
      const __nv_bfloat16* qb = nullptr;
      if (ra < R) {
        const int hh = ra / it.nq, qi = it.q0 + ra % it.nq;
        qa = p.q + static_cast<int64_t>(row0 + qi) * p.q_st + static_cast<int64_t>(it.h * p.n_rep + hh) * p.q_sh;
        lim_a = qi + ctx - qlen;
      }
      if (rb < R) {
        const int hh = rb / it.nq, qi = it.q0 + rb % it.nq;
        qb = p.q + static_cast<int64_t>(row0 + qi) * p.q_st + static_cast<int64_t>(it.h * p.n_rep + hh) * p.q_sh;
        lim_b = qi + ctx - qlen;
      }
#pragma unroll
      for (int kk = 0; kk < NKK; ++kk) {
        const int d0 = kk * 16 + 2 * cq;
        qf[kk][0] = qa ? *reinterpret_cast<const uint32_t*>(qa + d0) : 0u;
        qf[kk][1] = qb ? *reinterpret_cast<const uint32_t*>(qb + d0) : 0u;
        qf[kk][2] = qa ? *reinterpret_cast<const uint32_t*>(qa + d0 + 8) : 0u;
        qf[kk][3] = qb ? *reinterpret_cast<const uint32_t*>(qb + d0 + 8) : 0u;
      }
    }
#pragma unroll
    for (int nt = 0; nt < NNT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;

    for (int c = ks; c < nchunks; c += KS) {
      const int li0 = c * kChunkPages;
      const int np = min(kChunkPages, npages - li0);
      bool ok = true;
#pragma unroll
      for (int pg = 0; pg < kChunkPages; ++pg)
        if (pg < np) ok = ok && mbar_wait(&full_bar[(li0 + pg) % NST], ((li0 + pg) / NST) & 1);
      // every lane polls; the give-up decision is warp-wide so the warp leaves together
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) {
          raise_status(p.status, SPECDEC_STATUS_TIMEOUT);
          atomicExch(&s_abort, 1);
        }
        break;
      }
#include "split_consumer_chunk.inc"
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int pg = 0; pg < kChunkPages; ++pg)
          if (pg < np) mbar_arrive(&empty_bar[(li0 + pg) % NST]);
      }
    }
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  }
  __syncthreads();  // (A) every page consumed, every copy landed; the ring is free

#include "split_epilogue.inc"
}
