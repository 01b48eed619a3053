"""GPU: RMSNorm / RoPE / SwiGLU against the reference's own outputs (golden vectors of
reference.rmsnorm / apply_rope / swiglu, specdec/kernels/reference.py:14-31, made by
tests/golden/make_golden.py).  The kernels follow the reference's rounding steps, so the
bar is one unit in the last place: 1 bf16 ulp for bf16; for fp32, 4 ulps for RoPE and
SwiGLU (the exponential of silu differs from the CPU's by an ulp or two) and a relative
2e-6 for RMSNorm, whose fp32 sum of squares runs in another order than torch's CPU
reduction (the reference's own fp32 check is 1e-4 absolute, sample_experiment.py:21)."""

from __future__ import annotations

import pytest
import torch

from oracle import elementwise as oel

pytestmark = pytest.mark.gpu

BF16_ULPS = 1
F32_ULPS = 4


def _ops():
    from specdec_b200.kernels import ops

    return ops


def _ordered(t: torch.Tensor) -> torch.Tensor:
    """Bit patterns mapped to integers that order like the values (adjacent floats differ by 1)."""
    if t.dtype == torch.bfloat16:
        b = t.contiguous().view(torch.int16).long()
        return torch.where(b < 0, -(b & 0x7FFF), b)
    b = t.float().contiguous().view(torch.int32).long()
    return torch.where(b < 0, -(b & 0x7FFFFFFF), b)


def ulps(got: torch.Tensor, want: torch.Tensor) -> int:
    got = got.cpu().to(want.dtype)
    assert torch.isfinite(want.float()).all()
    return int((_ordered(got) - _ordered(want)).abs().max())


def _bar(dtype):
    return BF16_ULPS if dtype == torch.bfloat16 else F32_ULPS


def _rmsnorm_ok(got, want):
    if want.dtype == torch.bfloat16:
        return ulps(got, want) <= BF16_ULPS
    torch.testing.assert_close(got.cpu(), want, rtol=2e-6, atol=1e-7)
    return True


def test_rmsnorm_matches_reference(golden):
    ops = _ops()
    n = 0
    for name, c in golden["elementwise"].items():
        if not name.startswith("rmsnorm"):
            continue
        got = ops.rmsnorm(c["x"].cuda(), c["w"].cuda())
        assert _rmsnorm_ok(got, c["out"]), name
        n += 1
    assert n == 6


def test_rope_matches_reference(golden):
    ops = _ops()
    n = 0
    for name, c in golden["elementwise"].items():
        if not name.startswith("rope"):
            continue
        got = ops.apply_rope(c["x"].cuda(), c["cos"].cuda(), c["sin"].cuda())
        assert ulps(got, c["out"]) <= _bar(c["out"].dtype), name
        n += 1
    assert n == 6


def test_swiglu_matches_reference(golden):
    ops = _ops()
    n = 0
    for name, c in golden["elementwise"].items():
        if not name.startswith("swiglu"):
            continue
        got = ops.swiglu(c["gate"].cuda(), c["up"].cuda())
        assert ulps(got, c["out"]) <= _bar(c["out"].dtype), name
        if c["out"].dtype == torch.bfloat16:
            gu = torch.cat([c["gate"], c["up"]], dim=1)
            assert ulps(ops.swiglu_packed(gu.cuda()), c["out"]) <= BF16_ULPS, name + " (packed)"
        n += 1
    assert n == 4


def test_rope_strided_input():
    """A strided (transposed) input view, against the oracle (pinned to the reference)."""
    ops = _ops()
    x = torch.randn(1, 32, 12, 128).to(torch.bfloat16).transpose(1, 2)  # (1, 12, 32, 128), strided
    cos = torch.randn(1, 1, 32, 128).to(torch.bfloat16)
    sin = torch.randn_like(cos)
    got = ops.apply_rope(x.cuda(), cos.cuda(), sin.cuda())
    assert ulps(got, oel.apply_rope(x, cos, sin)) <= BF16_ULPS


def test_swiglu_packed_large():
    ops = _ops()
    gu = torch.randn(33, 2 * 4864).to(torch.bfloat16)
    got = ops.swiglu_packed(gu.cuda())
    assert ulps(got, oel.swiglu(gu[:, :4864], gu[:, 4864:])) <= BF16_ULPS


@pytest.mark.parametrize("hidden", [896, 1536, 1000, 4096])
def test_rmsnorm_engine_sizes(hidden):
    """bf16 rows of the model sizes (one warp per row) and of a size that is not a
    multiple of 8 (one block per row), against the oracle (pinned to the reference)."""
    ops = _ops()
    x = torch.randn(37, hidden).to(torch.bfloat16)
    w = torch.randn(hidden).to(torch.bfloat16)
    assert ulps(ops.rmsnorm(x.cuda(), w.cuda()), oel.rmsnorm(x, w)) <= BF16_ULPS
    x32 = torch.randn(5, hidden)
    w32 = torch.randn(hidden)
    assert _rmsnorm_ok(ops.rmsnorm(x32.cuda(), w32.cuda()), oel.rmsnorm(x32, w32))
