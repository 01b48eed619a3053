"""Paged-pool oracle (test infrastructure): numpy restatement of the specdec_b200 pool layout.

The reference keeps each layer's cache as contiguous (1, KV, T, D) tensors grown by
torch.cat (specdec/engine/model_self.py:778-800; the v_fp8 dict is
{"k": bf16, "v": e4m3, "v_scale": fp32 (1,KV,T,1), "fmt": "v_fp8"},
docs/design_g4_cache_api.md:8-10).  The B200 pool stores the same values in
16-token pages addressed through a page table; this module builds pools from
reference-layout tensors and gathers them back, independently of the CUDA code,
so appends, trims and attention can be checked bit-exactly.

Block layouts (per page, per KV head):
  bf16 K / V : element (r, d) at  (d // 64) * 1024 + r * 64 + (((d % 64) // 8) ^ (r % 8)) * 8 + d % 8
  E4M3 V     : byte    (r, d) at  r * D + d  (plain token rows)
  scales     : (r) at r
"""

from __future__ import annotations

import numpy as np

PAGE = 16


def kblock_perm(head_dim: int) -> np.ndarray:
    """perm[r * D + d] = element offset of (r, d) inside a bf16 block."""
    out = np.empty(PAGE * head_dim, dtype=np.int64)
    for r in range(PAGE):
        for d in range(head_dim):
            out[r * head_dim + d] = (d // 64) * 1024 + r * 64 + ((((d % 64) // 8) ^ (r % 8)) * 8) + d % 8
    return out


def vblock_perm(head_dim: int) -> np.ndarray:
    return np.arange(PAGE * head_dim, dtype=np.int64)


def random_page_table(num_seqs: int, max_pages: int, num_pages: int, seed: int) -> np.ndarray:
    """Seeded random assignment of distinct physical pages (a permutation when num_pages == B*max_pages)."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(num_pages)[: num_seqs * max_pages]
    return perm.reshape(num_seqs, max_pages).astype(np.int32)


def pack_bf16_rows(rows_u16: np.ndarray, head_dim: int) -> np.ndarray:
    """rows (16, D) uint16 -> one block (16*D,) uint16 in the swizzled order."""
    blk = np.zeros(PAGE * head_dim, dtype=np.uint16)
    blk[kblock_perm(head_dim)] = rows_u16.reshape(-1)
    return blk


def build_pools(k_u16, v, page_table, num_pages: int, v_scale=None):
    """Pools from reference-layout per-sequence tensors.

    k_u16: list over sequences of (KV, T_b, D) uint16 (bf16 bits).
    v: same shape, uint16 (bf16 V) or uint8 (E4M3 codes, then v_scale is a list of (KV, T_b) f32).
    Returns (k_pool (P, KV, 16*D) u16, v_pool, scale_pool or None)."""
    KV, _, D = k_u16[0].shape
    fp8 = v[0].dtype == np.uint8
    kpool = np.zeros((num_pages, KV, PAGE * D), dtype=np.uint16)
    vpool = np.zeros((num_pages, KV, PAGE * D), dtype=np.uint8 if fp8 else np.uint16)
    spool = np.zeros((num_pages, KV, PAGE), dtype=np.float32) if fp8 else None
    kp, vp = kblock_perm(D), vblock_perm(D)
    for b, kb in enumerate(k_u16):
        T = kb.shape[1]
        for t in range(T):
            page = page_table[b, t // PAGE]
            r = t % PAGE
            for h in range(KV):
                kpool[page, h, kp[r * D:(r + 1) * D]] = kb[h, t]
                if fp8:
                    vpool[page, h, vp[r * D:(r + 1) * D]] = v[b][h, t]
                    spool[page, h, r] = v_scale[b][h, t]
                else:
                    vpool[page, h, kp[r * D:(r + 1) * D]] = v[b][h, t]
    return kpool, vpool, spool


def gather(kpool, vpool, spool, page_table, seq: int, length: int):
    """Reference layout of one sequence: (k (KV,T,D) u16, v (KV,T,D) u16|u8, scale (KV,T) f32 | None)."""
    num_pages, KV, blk = kpool.shape
    D = blk // PAGE
    fp8 = vpool.dtype == np.uint8
    kp, vp = kblock_perm(D), vblock_perm(D)
    k = np.zeros((KV, length, D), dtype=np.uint16)
    v = np.zeros((KV, length, D), dtype=np.uint8 if fp8 else np.uint16)
    s = np.zeros((KV, length), dtype=np.float32) if fp8 else None
    for t in range(length):
        page = page_table[seq, t // PAGE]
        r = t % PAGE
        k[:, t] = kpool[page][:, kp[r * D:(r + 1) * D]]
        if fp8:
            v[:, t] = vpool[page][:, vp[r * D:(r + 1) * D]]
            s[:, t] = spool[page, :, r]
        else:
            v[:, t] = vpool[page][:, kp[r * D:(r + 1) * D]]
    return k, v, s
