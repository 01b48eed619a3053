"""Paged KV cache: one static-capacity page pool per layer, one page table per batch.

Layout of a (page, kv head) block (the same bytes the attention kernel stages
into shared memory with one bulk-TMA copy):

* K (and V when it stays bf16): 16 tokens x head_dim bf16, as head_dim/64
  half-tiles of [16 rows][128 bytes]; 16-byte chunk ``j`` of row ``r`` is stored
  at chunk position ``j ^ (r & 7)`` -- the image a TMA SWIZZLE_128B load of a
  {64, 16} box writes to shared memory.
* V as E4M3: plain [16 tokens][head_dim] code rows (token ``r``, dim ``d`` at
  byte ``r * head_dim + d``); the verify kernel widens a tile to f16 in shared
  memory before its PV MMA.
* V scales: [16] fp32 per (page, kv head).

The reference cache (specdec/engine/model_self.py:778-800, contract in
docs/design_g4_cache_api.md:8-10) is a per-layer dict of contiguous
(1, KV, T, D) tensors grown with ``torch.cat``.  This cache keeps the same
information in fixed pools; ``gather_layer`` returns the reference layout.
Every page of a sequence is assigned when the cache is created (static
capacity), so appends, rollback and attention never need the host.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

PAGE = 16


def kblock_index(head_dim: int, device=None) -> torch.Tensor:
    """Element permutation of a bf16 page-head block: ``block.flatten()[idx] = rows.flatten()``.

    ``idx[r * head_dim + d]`` is the bf16 element offset of (row r, dim d)."""
    r = torch.arange(PAGE, device=device).view(PAGE, 1)
    d = torch.arange(head_dim, device=device).view(1, head_dim)
    half = d // 64
    chunk = (d % 64) // 8
    elem = half * 1024 + r * 64 + ((chunk ^ (r & 7)) * 8) + (d % 8)
    return elem.reshape(-1)


def vblock_index(head_dim: int, device=None) -> torch.Tensor:
    """Byte offsets of an E4M3 page-head block: ``idx[r * head_dim + d] = r * head_dim + d`` (plain rows)."""
    return torch.arange(PAGE * head_dim, device=device)


@dataclass
class LayerPool:
    """Device pools of one layer."""

    k: torch.Tensor  # bf16 [num_pages, KV, 16 * D]
    v: torch.Tensor  # bf16 [num_pages, KV, 16 * D] or uint8 [num_pages, KV, D * 16]
    v_scale: torch.Tensor | None  # f32 [num_pages, KV, 16]


@dataclass
class PagedKVCache:
    """Paged cache of ``num_layers`` layers for ``num_seqs`` sequences.

    ``lengths`` (device int32 [num_seqs]) is the committed token count of every
    sequence; ``host_lengths`` mirrors it while only host-driven operations have
    touched it (``None`` once a device-side rollback made it unknown).
    """

    num_layers: int
    num_seqs: int
    num_kv_heads: int
    head_dim: int
    capacity: int  # tokens per sequence
    v_dtype: str  # "bf16" | "e4m3"
    device: torch.device
    pools: list[LayerPool]
    page_table: torch.Tensor  # int32 [num_seqs, max_pages]
    lengths: torch.Tensor  # int32 [num_seqs]
    host_lengths: list[int] | None = field(default_factory=list)
    fmt: str = "fp16"

    @classmethod
    def allocate(
        cls,
        num_layers: int,
        num_seqs: int,
        num_kv_heads: int,
        head_dim: int,
        capacity: int,
        *,
        v_dtype: str = "bf16",
        device: torch.device | str = "cuda",
        page_order_seed: int | None = None,
        num_pages: int | None = None,
    ) -> "PagedKVCache":
        if v_dtype not in ("bf16", "e4m3"):
            raise ValueError(f"v_dtype must be 'bf16' or 'e4m3', got {v_dtype!r}")
        if head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        if v_dtype == "e4m3" and head_dim != 128:
            raise ValueError("E4M3 V needs head_dim 128 (one scale group per head, GROUP_V = 128)")
        device = torch.device(device)
        max_pages = max(1, math.ceil(capacity / PAGE))
        need = num_seqs * max_pages
        total = need if num_pages is None else int(num_pages)
        if total < need:
            raise ValueError(f"pool of {total} pages cannot hold {num_seqs} x {max_pages} pages")
        if page_order_seed is None:
            order = torch.arange(need, dtype=torch.int32)
        else:
            g = torch.Generator().manual_seed(int(page_order_seed))
            order = torch.randperm(total, generator=g)[:need].to(torch.int32)
        page_table = order.view(num_seqs, max_pages).to(device)
        pools = []
        for _ in range(num_layers):
            # zero-filled: pages past a sequence's length hold finite data, so a
            # masked key multiplies a finite value by a zero probability
            k = torch.zeros(total, num_kv_heads, PAGE * head_dim, dtype=torch.bfloat16, device=device)
            if v_dtype == "e4m3":
                v = torch.zeros(total, num_kv_heads, head_dim * PAGE, dtype=torch.uint8, device=device)
                sc = torch.zeros(total, num_kv_heads, PAGE, dtype=torch.float32, device=device)
            else:
                v = torch.zeros(total, num_kv_heads, PAGE * head_dim, dtype=torch.bfloat16, device=device)
                sc = None
            pools.append(LayerPool(k, v, sc))
        return cls(
            num_layers=num_layers,
            num_seqs=num_seqs,
            num_kv_heads=num_kv_heads,
            head_dim=head_dim,
            capacity=max_pages * PAGE,
            v_dtype=v_dtype,
            device=device,
            pools=pools,
            page_table=page_table,
            lengths=torch.zeros(num_seqs, dtype=torch.int32, device=device),
            host_lengths=[0] * num_seqs,
            fmt="v_fp8" if v_dtype == "e4m3" else "fp16",
        )

    # ------------------------------------------------------------------ views
    @property
    def num_pages(self) -> int:
        return int(self.pools[0].k.shape[0])

    @property
    def max_pages(self) -> int:
        return int(self.page_table.shape[1])

    def with_lengths(self, lengths: torch.Tensor, host_lengths: list[int] | None) -> "PagedKVCache":
        """A view sharing the pools and page table with other lengths (the trim result)."""
        return PagedKVCache(
            num_layers=self.num_layers,
            num_seqs=self.num_seqs,
            num_kv_heads=self.num_kv_heads,
            head_dim=self.head_dim,
            capacity=self.capacity,
            v_dtype=self.v_dtype,
            device=self.device,
            pools=self.pools,
            page_table=self.page_table,
            lengths=lengths,
            host_lengths=None if host_lengths is None else list(host_lengths),
            fmt=self.fmt,
        )

    def set_host_lengths(self, lens: list[int]) -> None:
        if len(lens) != self.num_seqs:
            raise ValueError("one length per sequence")
        for n in lens:
            if n < 0 or n > self.capacity:
                raise ValueError(f"length {n} outside [0, {self.capacity}]")
        self.host_lengths = [int(n) for n in lens]
        self.lengths.copy_(torch.tensor(self.host_lengths, dtype=torch.int32))

    def sync_host_lengths(self) -> list[int]:
        """Read the device lengths back (one device->host copy)."""
        self.host_lengths = [int(x) for x in self.lengths.cpu().tolist()]
        return self.host_lengths

    # ------------------------------------------------------------------ layout helpers
    def gather_layer(self, layer: int, seq: int, length: int | None = None) -> dict:
        """Reference-layout copy of one sequence of one layer:
        {"k": bf16 (1,KV,T,D), "v": bf16 or e4m3 (1,KV,T,D), "v_scale": f32 (1,KV,T,1)}."""
        if length is None:
            if self.host_lengths is None:
                self.sync_host_lengths()
            length = self.host_lengths[seq]
        D, KV = self.head_dim, self.num_kv_heads
        npg = math.ceil(length / PAGE)
        pages = self.page_table[seq, :npg].long()
        pool = self.pools[layer]
        kidx = kblock_index(D, self.device)
        kb = pool.k[pages]  # [npg, KV, 16*D]
        k = kb[:, :, kidx].view(npg, KV, PAGE, D).permute(1, 0, 2, 3).reshape(KV, npg * PAGE, D)[:, :length]
        out = {"k": k.unsqueeze(0)}
        if self.v_dtype == "e4m3":
            vidx = vblock_index(D, self.device)
            vb = pool.v[pages][:, :, vidx].view(npg, KV, PAGE, D)
            v = vb.permute(1, 0, 2, 3).reshape(KV, npg * PAGE, D)[:, :length]
            out["v"] = v.contiguous().view(torch.float8_e4m3fn).unsqueeze(0)
            sc = pool.v_scale[pages].permute(1, 0, 2).reshape(KV, npg * PAGE)[:, :length]
            out["v_scale"] = sc.unsqueeze(0).unsqueeze(-1)
            out["fmt"] = "v_fp8"
        else:
            vb = pool.v[pages][:, :, kidx].view(npg, KV, PAGE, D)
            out["v"] = vb.permute(1, 0, 2, 3).reshape(KV, npg * PAGE, D)[:, :length].unsqueeze(0)
        return out
