"""spec_cache oracle (test infrastructure): restatement of specdec/engine/spec_cache.py:4-46.

  cache_length(c)     : 0 for None, else c[0]["k"].shape[2]
  trim_cache(c, n)    : None & n == 0 -> None; None & n != 0 -> ValueError;
                        n not an int (bool excluded) -> ValueError; n <= 0 or n > len -> ValueError;
                        otherwise a NEW list of NEW dicts whose tensors are t[:, :, :n] views
                        (non-tensor values such as "fmt" copied by reference); the input is unchanged
  check_consistent(c) : every tensor of dim >= 3 in a layer has one dim-2 length, and all layers
                        share it; otherwise RuntimeError
plus the batched rollback rule of the device path: per sequence, a request
outside (0, cur] leaves the length unchanged and flags an error.
"""

from __future__ import annotations

import torch


def cache_length(cache) -> int:
    if cache is None:
        return 0
    return int(cache[0]["k"].shape[2])


def trim_cache(cache, new_len):
    if cache is None:
        if new_len == 0:
            return None
        raise ValueError("trim_cache(None, n > 0)")
    cur = cache_length(cache)
    if not isinstance(new_len, int) or isinstance(new_len, bool):
        raise ValueError("new_len must be an int")
    if new_len <= 0 or new_len > cur:
        raise ValueError(f"new_len {new_len} out of range (current {cur})")
    return [{key: (val[:, :, :new_len] if isinstance(val, torch.Tensor) else val) for key, val in layer.items()}
            for layer in cache]


def check_consistent(cache) -> None:
    if cache is None:
        return
    per_layer = []
    for i, layer in enumerate(cache):
        lens = {int(v.shape[2]) for v in layer.values() if isinstance(v, torch.Tensor) and v.dim() >= 3}
        if len(lens) != 1:
            raise RuntimeError(f"cache token dim mismatch at layer {i}")
        per_layer.append(lens.pop())
    if len(set(per_layer)) != 1:
        raise RuntimeError("cross-layer token length mismatch")


def batched_trim(cur, req):
    """Device-rollback rule: (new lengths, error flag)."""
    out, err = [], False
    for c, n in zip(cur, req):
        if n <= 0 or n > c:
            out.append(int(c))
            err = True
        else:
            out.append(int(n))
    return out, err
