"""GPU: RMSNorm / RoPE / SwiGLU against the reference formulas (reference.py:14-31) with the
sample experiment's tolerances (fp32 1e-4 absolute; bf16 2e-2 or 2 % of the magnitude)."""

from __future__ import annotations

import pytest
import torch

from oracle import elementwise as oel

pytestmark = pytest.mark.gpu


def _ops():
    from specdec_b200.kernels import ops

    return ops


def _bf16_ok(got, ref):
    err = (got.float().cpu() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item()
    return err <= 2e-2 or err <= 0.02 * max(scale, 1e-6)


def test_rmsnorm():
    ops = _ops()
    x = torch.randn(4, 128, 1536)
    w = torch.randn(1536)
    got = ops.rmsnorm(x.cuda(), w.cuda())
    torch.testing.assert_close(got.cpu(), oel.rmsnorm(x, w), rtol=0, atol=1e-4)
    xb, wb = x.to(torch.bfloat16), w.to(torch.bfloat16)
    assert _bf16_ok(ops.rmsnorm(xb.cuda(), wb.cuda()), oel.rmsnorm(xb, wb))


def test_rope_strided_input():
    ops = _ops()
    x = torch.randn(1, 32, 12, 128).to(torch.bfloat16).transpose(1, 2)  # (1, 12, 32, 128), strided
    cos = torch.randn(1, 1, 32, 128).to(torch.bfloat16)
    sin = torch.randn_like(cos)
    got = ops.apply_rope(x.cuda(), cos.cuda(), sin.cuda())
    assert _bf16_ok(got, oel.apply_rope(x, cos, sin))


def test_swiglu():
    ops = _ops()
    g = torch.randn(2, 32, 8960).to(torch.bfloat16)
    u = torch.randn_like(g)
    assert _bf16_ok(ops.swiglu(g.cuda(), u.cuda()), oel.swiglu(g, u))
    g32, u32 = g.float(), u.float()
    torch.testing.assert_close(ops.swiglu(g32.cuda(), u32.cuda()).cpu(), oel.swiglu(g32, u32), rtol=0, atol=1e-4)


def test_swiglu_packed_matches_swiglu():
    """Fused gate|up SwiGLU: the reference formula's tolerance, and within one bf16 ulp of
    the unpacked kernel (its silu uses the hardware exponential and reciprocal)."""
    ops = _ops()
    gu = torch.randn(33, 2 * 4864).to(torch.bfloat16)
    got = ops.swiglu_packed(gu.cuda()).cpu()
    assert _bf16_ok(got, oel.swiglu(gu[:, :4864], gu[:, 4864:]))
    want = ops.swiglu(gu[:, :4864].contiguous().cuda(), gu[:, 4864:].contiguous().cuda()).cpu()
    ulp = (got.view(torch.int16).int() - want.view(torch.int16).int()).abs()
    assert int(ulp.max()) <= 1
    assert float((ulp == 0).float().mean()) > 0.99


@pytest.mark.parametrize("hidden", [896, 1536, 1000, 4096])
def test_rmsnorm_engine_sizes(hidden):
    """bf16 rows of the model sizes (one warp per row) and of a size that is not a
    multiple of 8 (one block per row)."""
    ops = _ops()
    x = torch.randn(37, hidden).to(torch.bfloat16)
    w = torch.randn(hidden).to(torch.bfloat16)
    assert _bf16_ok(ops.rmsnorm(x.cuda(), w.cuda()), oel.rmsnorm(x, w))
