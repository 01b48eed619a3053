"""GPU: device greedy accept and rollback against the reference's vectorised accept
(golden cases) and the oracle, including ties, NaN and the full 151936 vocab."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as oacc
from oracle import spec_cache as osc

pytestmark = pytest.mark.gpu


def _ops():
    from specdec_b200.kernels import ops

    return ops


def _i32(x):
    return torch.tensor(x, dtype=torch.int32, device="cuda")


def test_accept_matches_golden_cases(golden):
    ops = _ops()
    cases = golden["accept"]
    B = len(cases)
    max_rows = max(c["stack"].shape[0] for c in cases)
    V = cases[0]["stack"].shape[1]
    rows = torch.cat([c["stack"] for c in cases], dim=0).cuda()
    n_rows = [c["stack"].shape[0] for c in cases]
    row0 = np.cumsum([0] + n_rows[:-1]).tolist()
    cands = torch.zeros(B, max_rows, dtype=torch.int32)
    for b, c in enumerate(cases):
        cands[b, : len(c["cands"])] = c["cands"].to(torch.int32)
    kp = [len(c["cands"]) for c in cases]
    g, m, nxt = ops.greedy_accept(rows, row0=_i32(row0), n_rows=_i32(n_rows), cands=cands.cuda(), kp=_i32(kp),
                                  max_rows=max_rows)
    torch.cuda.synchronize()
    g, m, nxt = g.cpu(), m.cpu(), nxt.cpu()
    for b, c in enumerate(cases):
        assert g[b, : n_rows[b]].tolist() == c["g"].tolist(), b
        assert int(m[b]) == c["m"], b
        want_next = c["g"][c["m"]].item() if c["m"] < n_rows[b] else -1
        assert int(nxt[b]) == want_next


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_accept_full_vocab_with_rollback(dtype):
    """Carry-forward verify blocks (pending + 4 candidates = 5 rows) over the target vocab."""
    ops = _ops()
    V, B, k = 151936, 6, 4
    gen = torch.Generator().manual_seed(4)
    logits = torch.randn(B * (k + 1), V, generator=gen).to(dtype)
    truth = logits.float().argmax(-1).view(B, k + 1)
    cands = torch.randint(0, V, (B, k), generator=gen, dtype=torch.int32)
    for b in range(B):
        mp = b % (k + 1)
        cands[b, :mp] = truth[b, :mp].to(torch.int32)
        if mp < k and cands[b, mp] == truth[b, mp]:
            cands[b, mp] += 1
    # a tie at the maximum in sequence 0 row 0 and a NaN in sequence 1 row 2
    logits[0, 12345] = logits[0].float().max().to(dtype)
    logits[0, 99] = logits[0, 12345]
    logits[1 * (k + 1) + 2, 777] = float("nan")
    pre = [100 + 10 * b for b in range(B)]
    len_after = torch.zeros(B, dtype=torch.int32, device="cuda")
    g, m, nxt = ops.greedy_accept(logits.cuda(), row0=_i32([b * (k + 1) for b in range(B)]),
                                  n_rows=_i32([k + 1] * B), cands=cands.cuda(), kp=_i32([k] * B), max_rows=k + 1,
                                  len_before=_i32(pre), len_after=len_after, keep_offset=1)
    torch.cuda.synchronize()
    lf = logits.float().numpy()
    for b in range(B):
        rows = [lf[b * (k + 1) + j] for j in range(k + 1)]
        og, om, onx, ol = oacc.rows_accept(rows, cands[b].tolist(), k, len_before=pre[b], keep_offset=1)
        assert g[b].cpu().tolist() == og
        assert int(m[b]) == om and int(nxt[b]) == onx and int(len_after[b]) == ol
    assert int(g[0, 0]) == 99  # first index wins the tie
    assert int(g[1, 2]) == 777  # NaN is the maximum


def test_accept_workspace_is_reusable_in_a_graph():
    ops = _ops()
    V, B = 32000, 3
    logits = torch.randn(B * 5, V, device="cuda", dtype=torch.bfloat16)
    args = dict(row0=_i32([0, 5, 10]), n_rows=_i32([5, 5, 5]), cands=torch.zeros(B, 4, dtype=torch.int32,
                                                                                  device="cuda"),
                kp=_i32([4, 4, 4]), max_rows=5)
    ws = ops.accept_workspace(B, 5, V)
    g1, m1, n1 = ops.greedy_accept(logits, workspace=ws, **args)
    g2, m2, n2 = ops.greedy_accept(logits, workspace=ws, **args)
    torch.cuda.synchronize()
    assert torch.equal(g1, g2) and torch.equal(m1, m2)
    assert torch.equal(g1, logits.float().argmax(-1).view(B, 5).to(torch.int32))
    # every ticket was reset by its last user: the ticket arrays (after the per-chunk
    # partials, 256-byte aligned) are zero again
    chunks = -(-V // 8192)
    rows = B * 5
    a256 = lambda x: -(-x // 256) * 256  # noqa: E731
    rt = a256(a256(rows * chunks * 4) + rows * chunks * 4)
    st = a256(rt + rows * 4)
    assert not ws[rt:rt + rows * 4].any() and not ws[st:st + B * 4].any()
    g3, m3, _ = ops.greedy_accept(logits, workspace=ws, **args)
    assert torch.equal(g1, g3) and torch.equal(m1, m3)


def test_device_trim_rule():
    from specdec_b200 import _lib

    ops = _ops()
    cur = [10, 10, 10, 5, 1]
    req = [3, 10, 0, 6, 1]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.trim_lengths(_i32(cur), _i32(req), status=status)
    want, err = osc.batched_trim(cur, req)
    assert out.cpu().tolist() == want
    assert bool(int(status.item()) & _lib.STATUS_TRIM_RANGE) == err


def test_paged_trim_view_semantics():
    from specdec_b200.engine import PagedKVCache, cache_length, trim_cache, trim_cache_device

    c = PagedKVCache.allocate(2, 1, 2, 128, 64, device="cuda")
    c.set_host_lengths([40])
    t = trim_cache(c, 25)
    assert cache_length(t) == 25 and cache_length(c) == 40
    assert t.pools is c.pools
    for bad in (0, -1, 41, True, 3.0):
        with pytest.raises(ValueError):
            trim_cache(c, bad)
    b = PagedKVCache.allocate(1, 3, 2, 128, 64, device="cuda")
    b.set_host_lengths([30, 20, 10])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    v = trim_cache_device(b, torch.tensor([29, 25, 1], device="cuda"), status=status)
    assert v.lengths.cpu().tolist() == [29, 20, 1] and int(status.item()) != 0
    assert b.lengths.cpu().tolist() == [30, 20, 10]
