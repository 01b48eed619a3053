"""GPU: the fused LM-head argmax (specdec_lmhead_argmax) against torch.argmax of the bf16
logits x @ W^T (model_self.py:857; the executors' argmax, spec_dec.py:230-236,
fast_spec_dec.py:246-249).

Bar: the chosen index equals torch.argmax of the cuBLAS bf16 logits, except where those
logits have a near-tie -- the top two within one bf16 ulp of each other, where a different
fp32 accumulation order may round either way; there the chosen logit must still be within
one bf16 ulp of the maximum.  Planted exact ties (identical weight rows) must pick the
first index, NaN logits count as the maximum, and every reported max value equals the
bf16 logit of the chosen index within one ulp."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from specdec_b200.kernels import ops

    return ops


def _bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """One bf16 unit in the last place at |x| (x float32)."""
    e = torch.floor(torch.log2(x.abs().clamp(min=2.0 ** -126)))
    return torch.exp2(e - 7)


def _check(idx, x, w, what, max_value=None):
    logits = (x @ w.t()).float()  # cuBLAS, stored in bf16 as the reference's LM head does
    want = logits.argmax(-1)
    got = idx.long()
    assert int(got.min()) >= 0 and int(got.max()) < w.shape[0], what
    top = logits.gather(1, want[:, None])[:, 0]
    mine = logits.gather(1, got[:, None])[:, 0]
    differ = got != want
    if bool(differ.any()):
        # only near-ties may differ: the chosen logit within one bf16 ulp of the maximum
        gap = (top - mine)[differ]
        assert bool((gap <= _bf16_ulp(top[differ]) * 1.001).all()), \
            f"{what}: {int(differ.sum())} rows differ beyond a near-tie (max gap {float(gap.max()):.3e})"
        assert float(differ.float().mean()) < 0.02, f"{what}: {int(differ.sum())} rows differ"
    if max_value is not None:
        assert bool(((max_value - mine).abs() <= _bf16_ulp(mine) * 1.001).all()), f"{what}: max values"
    return int(differ.sum())


@pytest.mark.parametrize("rows,vocab,hidden", [
    (5, 151936, 1536),    # one verify block, target LM head
    (256, 151936, 896),   # the draft's proposals of 256 sequences
    (1280, 151936, 1536),  # the target's verify rows of 256 sequences
    (129, 4099, 256),     # a vocab tail shorter than a tile, rows past one tile
    (1, 1000, 128),
])
def test_lmhead_argmax_matches_torch(rows, vocab, hidden):
    ops = _ops()
    g = torch.Generator(device="cuda").manual_seed(rows + vocab)
    x = torch.randn(rows, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    mv = torch.empty(rows, dtype=torch.float32, device="cuda")
    ws = ops.lmhead_workspace(rows)
    idx = ops.lmhead_argmax(x, w, max_value=mv, workspace=ws)
    torch.cuda.synchronize()
    _check(idx, x, w, f"rows={rows} vocab={vocab}", mv)
    # the workspace is left zeroed: a second call on other inputs is right too
    x2 = torch.randn(rows, hidden, generator=g, device="cuda").to(torch.bfloat16)
    idx2 = ops.lmhead_argmax(x2, w, workspace=ws)
    torch.cuda.synchronize()
    _check(idx2, x2, w, f"rows={rows} vocab={vocab} second call")
    assert int(ws.count_nonzero()) == 0


def test_lmhead_argmax_ties_and_zero_rows():
    """Identical weight rows (exact ties) give the first index, within a tile and across
    tiles; an all-zero hidden row (every logit +-0, all equal) gives index 0."""
    ops = _ops()
    vocab, hidden = 151936, 1536
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    x = torch.randn(4, hidden, generator=g, device="cuda").to(torch.bfloat16)
    for r, (a, b) in enumerate(((300, 301), (5, 150000))):
        w[a] = x[r] * 0.2
        w[b] = w[a]
    x[2] = 0
    idx = ops.lmhead_argmax(x, w)
    torch.cuda.synchronize()
    want = (x @ w.t()).argmax(-1)
    assert int(idx[0]) == 300 and int(want[0]) == 300
    assert int(idx[1]) == 5 and int(want[1]) == 5
    assert int(idx[2]) == 0 and int(want[2]) == 0
    _check(idx[3:], x[3:], w, "plain row")


def test_lmhead_argmax_nan_is_the_maximum():
    """A NaN logit wins (the first NaN index, as torch.argmax): one weight row with a NaN
    makes that vocab entry NaN for every row whose hidden value there is used."""
    ops = _ops()
    vocab, hidden = 40000, 896
    g = torch.Generator(device="cuda").manual_seed(6)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    x = torch.randn(3, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w[777, 10] = float("nan")
    w[31000, 3] = float("nan")
    idx = ops.lmhead_argmax(x, w)
    torch.cuda.synchronize()
    want = (x @ w.t()).argmax(-1)
    assert idx.tolist() == [777, 777, 777] and want.tolist() == [777, 777, 777]


def test_lmhead_argmax_strided_rows():
    """Rows taken from a wider buffer (row stride > hidden), as the engine gathers last rows."""
    ops = _ops()
    g = torch.Generator(device="cuda").manual_seed(9)
    big = torch.randn(40, 1024, generator=g, device="cuda").to(torch.bfloat16)
    x = big[:, :896]
    w = (torch.randn(32000, 896, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    idx = ops.lmhead_argmax(x, w)
    torch.cuda.synchronize()
    _check(idx, x.contiguous(), w, "strided")
