"""FP8 E4M3 oracle (test infrastructure): numpy restatement of the V-only quantiser.

quantize_v follows quantize_kv_fp8(x, group_size=GROUP_V=128) (specdec/engine/model_self.py:304-314):
    m = max |x| over the group (fp32);  s = m / 448;  s = 1 where s == 0;
    q = float8_e4m3fn(x / s)
E4M3_MAX = 448 and GROUP_V = 128 are model_self.py:300-302.

The fp32 -> float8_e4m3fn conversion restates PyTorch's (the reference's
arithmetic dependency, torch >= 2.3 pinned in requirements-local.txt; c10
Float8_e4m3fn): round to nearest even on the 3-bit mantissa, subnormal step
2^-9, sign kept (including -0), and any magnitude above 464 (which would round
to the 0x7F NaN pattern) or NaN becomes NaN 0x7F | sign.  This module is pinned
against torch's own cast and the golden vectors of tests/golden.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = np.float32(448.0)
GROUP_V = 128


def f32_to_e4m3(x) -> np.ndarray:
    """Vectorised RNE float32 -> E4M3 (fn variant) codes as uint8."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = x.view(np.uint32)
    sign = ((bits >> 31) & 1).astype(np.uint32)
    a = bits & np.uint32(0x7FFFFFFF)
    out = np.zeros(a.shape, dtype=np.uint32)

    nan_or_big = a > np.uint32(0x43E80000)  # NaN, inf, and |x| > 464
    sub = a < np.uint32(0x3C800000)  # |x| < 2^-6: E4M3 subnormal range
    norm = ~(nan_or_big | sub)

    # subnormals: m * 2^-9, m = rne(|x| * 2^9) in 0..8 (8 is the smallest normal, code 0x08)
    af = a.view(np.float32)
    m = np.rint(af[sub] * np.float32(512.0)).astype(np.uint32)
    out[sub] = m

    # normals: keep 3 mantissa bits with round-to-nearest-even on the 20 dropped bits
    an = a[norm]
    q = an >> 20
    low = an & np.uint32(0xFFFFF)
    up = (low > 0x80000) | ((low == 0x80000) & ((q & 1) == 1))
    q = q + up.astype(np.uint32)
    out[norm] = q - np.uint32(120 << 3)  # rebias exponent 127 -> 7

    out[nan_or_big] = 0x7F
    out |= sign << 7
    return out.astype(np.uint8)


def e4m3_to_f32(codes) -> np.ndarray:
    """Exact decode of E4M3 codes (0x7F / 0xFF are NaN)."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    s = np.where((c >> 7) & 1, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    val = np.where((c & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


def quantize_v(x, group_size: int = GROUP_V):
    """(codes uint8 same shape as x, scale float32 shape x.shape[:-1] + (groups,))."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    if d % group_size:
        raise ValueError(f"head_dim {d} % group_size {group_size} != 0")
    g = d // group_size
    xg = x.reshape(*x.shape[:-1], g, group_size)
    m = np.abs(xg).max(axis=-1, keepdims=True)
    s = (m / E4M3_MAX).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    q = f32_to_e4m3((xg / s).astype(np.float32))
    return q.reshape(x.shape), s[..., 0]


def dequantize_v(codes, scale, group_size: int = GROUP_V) -> np.ndarray:
    """f32(code) * scale in fp32 (model_self.py:316-320 before its final dtype cast)."""
    c = e4m3_to_f32(codes)
    d = c.shape[-1]
    g = d // group_size
    cg = c.reshape(*c.shape[:-1], g, group_size)
    return (cg * np.asarray(scale, dtype=np.float32)[..., None]).reshape(c.shape).astype(np.float32)


def outlier_v(shape, seed: int, frac: float = 0.01, sigma: float = 8.0):
    """Synthetic V of the FP8 config: N(0,1) with a `frac` share of entries replaced by +-sigma."""
    rng = np.random.default_rng(seed)
    v = rng.standard_normal(shape).astype(np.float32)
    hit = rng.random(shape) < frac
    sgn = np.where(rng.random(shape) < 0.5, -1.0, 1.0).astype(np.float32)
    v[hit] = sigma * sgn[hit]
    return v
