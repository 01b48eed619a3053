"""Cache length / trim / consistency contract (specdec/engine/spec_cache.py:4-46) for
the reference's per-layer dict caches and for the paged cache of this build.

Dict caches (a list of per-layer dicts of (1, KV, T, D) tensors) behave exactly as
in the reference: ``trim_cache`` returns a new list of new dicts holding
``t[:, :, :n]`` views and leaves the input untouched.

A ``PagedKVCache`` keeps one length per sequence for all layers.  With one
sequence, ``cache_length``/``trim_cache`` take and return plain ints with the
reference's ``ValueError`` rules; the result is a view sharing the pools and
page table (the original's length metadata is unchanged; slots past the new
length are overwritten by the next append).  ``trim_cache_device`` is the
batched, sync-free rollback: lengths stay on the device and out-of-range
requests raise a status bit that the caller checks at the round boundary.
"""

from __future__ import annotations

import torch

from .paged_cache import PagedKVCache


def cache_length(cache) -> int:
    if cache is None:
        return 0
    if isinstance(cache, PagedKVCache):
        if cache.num_seqs != 1:
            raise TypeError("cache_length of a batched PagedKVCache is per sequence; use cache.lengths")
        if cache.host_lengths is None:
            cache.sync_host_lengths()
        return int(cache.host_lengths[0])
    return int(cache[0]["k"].shape[2])


def trim_cache(cache, new_len):
    if cache is None:
        if new_len == 0:
            return None
        raise ValueError("trim_cache(None, n > 0): a missing cache can only be trimmed to 0")
    cur = cache_length(cache)
    if not isinstance(new_len, int) or isinstance(new_len, bool):
        raise ValueError("new_len must be an int")
    if new_len <= 0 or new_len > cur:
        raise ValueError(f"new_len {new_len} out of range (current {cur})")
    if isinstance(cache, PagedKVCache):
        lengths = torch.full_like(cache.lengths, new_len)
        return cache.with_lengths(lengths, [new_len])
    out = []
    for layer in cache:
        out.append({key: (val[:, :, :new_len] if isinstance(val, torch.Tensor) else val)
                    for key, val in layer.items()})
    return out


def trim_cache_device(cache: PagedKVCache, new_lengths: torch.Tensor, status: torch.Tensor | None = None):
    """Batched rollback on the device (no host sync): a view whose lengths are
    ``new_lengths[b]`` where ``0 < new_lengths[b] <= lengths[b]``; other sequences keep
    their length and raise SPECDEC_STATUS_TRIM_RANGE in ``status``."""
    from ..kernels import ops

    out = ops.trim_lengths(cache.lengths, new_lengths.to(torch.int32), status=status)
    return cache.with_lengths(out, None)


def check_consistent(cache) -> None:
    if cache is None:
        return
    if isinstance(cache, PagedKVCache):
        lens = cache.sync_host_lengths()
        bad = [n for n in lens if n < 0 or n > cache.capacity]
        if bad:
            raise RuntimeError(f"paged cache length outside [0, {cache.capacity}]: {bad[:4]}")
        return
    per_layer = []
    for i, layer in enumerate(cache):
        cur = [(key, int(val.shape[2])) for key, val in layer.items()
               if isinstance(val, torch.Tensor) and val.dim() >= 3]
        if len({n for _, n in cur}) != 1:
            raise RuntimeError(f"cache token dim mismatch at layer {i}: {cur}")
        per_layer.append(cur[0][1])
    if len(set(per_layer)) != 1:
        raise RuntimeError(f"cross-layer token length mismatch: {per_layer}")
