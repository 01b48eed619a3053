"""Greedy-accept oracle (test infrastructure).

strict_accept   : spec_dec.py:230-250 -- g = [argmax(x) for x in [saved_next] + rows[:kp-1]],
                  m = first mismatch; emitted = cands[:m] + [g[m]] (m < kp) or cands (m == kp).
vector_accept   : fast_spec_dec.py:246-256 -- g = argmax(cat(saved_next, rows[:kp-1])),
                  m = cumprod(g == cands).sum().
rows_accept     : the device kernel's contract on one sequence: g_j = argmax(row j) for every
                  given row, m = common prefix of g[:kp] and cands[:kp], next = g[m] (or -1),
                  len_after = len_before + keep_offset + m.
argmax follows torch.argmax: NaN is the maximum, the first index wins ties.
"""

from __future__ import annotations

import numpy as np


def argmax_torch_order(row) -> int:
    r = np.asarray(row, dtype=np.float32)
    nan = np.isnan(r)
    if nan.any():
        return int(np.argmax(nan))
    return int(np.argmax(r))  # numpy returns the first maximal index


def strict_accept(saved_next, rows, cands):
    kp = len(cands)
    g = [argmax_torch_order(x) for x in [saved_next] + [rows[j] for j in range(kp - 1)]]
    m = 0
    while m < kp and g[m] == cands[m]:
        m += 1
    emitted = list(cands[:m]) + [g[m]] if m < kp else list(cands)
    return g, m, emitted


def vector_accept(saved_next, rows, cands):
    kp = len(cands)
    stack = [saved_next] + [rows[j] for j in range(kp - 1)]
    g = np.array([argmax_torch_order(x) for x in stack])
    m = int(np.cumprod((g == np.asarray(cands)).astype(np.int64)).sum())
    return g.tolist(), m


def rows_accept(rows, cands, kp: int, len_before: int = 0, keep_offset: int = 0):
    g = [argmax_torch_order(r) for r in rows]
    m = 0
    while m < kp and g[m] == cands[m]:
        m += 1
    nxt = g[m] if m < len(g) else -1
    return g, m, nxt, len_before + keep_offset + m
