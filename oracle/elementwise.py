"""Elementwise oracle (test infrastructure): reference.rmsnorm / apply_rope / swiglu
(specdec/kernels/reference.py:14-31) restated with torch CPU ops."""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rmsnorm(x, weight, eps=1e-6):
    x = x.cpu()
    x32 = x.float()
    normed = x32 * torch.rsqrt(torch.mean(x32 * x32, dim=-1, keepdim=True) + eps)
    return weight.cpu() * normed.to(x.dtype)


def apply_rope(x, cos, sin):
    x, cos, sin = x.cpu(), cos.cpu(), sin.cpu()
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rotated * sin


def swiglu(gate, up):
    return F.silu(gate.cpu()) * up.cpu()
