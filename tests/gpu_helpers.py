"""Helpers of the GPU parity tests: seeded inputs, oracle-built pools, comparisons.

Pools are built by the oracle (numpy) and uploaded, so attention parity does not
depend on the append kernel; the append kernel is checked separately against
the same oracle pools."""

from __future__ import annotations

import numpy as np
import torch

from oracle import attention as oatt
from oracle import fp8 as ofp8
from oracle import paged as opg

RTOL, ATOL = 2e-2, 1e-2  # north-star tolerance for bf16 attention outputs


def seeded_kv(lens, KV, D, seed, fp8=False):
    """Per-sequence bf16 K and V (KV, T_b, D); V with 1 % outliers at +-8 sigma when fp8."""
    g = torch.Generator().manual_seed(seed)
    ks, vs = [], []
    for i, n in enumerate(lens):
        ks.append(torch.randn(KV, n, D, generator=g).to(torch.bfloat16))
        if fp8:
            vs.append(torch.from_numpy(ofp8.outlier_v((KV, n, D), seed * 1000 + i)).to(torch.bfloat16))
        else:
            vs.append(torch.randn(KV, n, D, generator=g).to(torch.bfloat16))
    return ks, vs


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def oracle_pools(ks, vs, pt, num_pages, fp8):
    """Oracle pools of per-sequence bf16 K/V: (k_pool, v_pool, scale_pool, v_ref list)."""
    if fp8:
        cs, ss, vref = [], [], []
        for v in vs:
            c, s = ofp8.quantize_v(v.float().numpy())
            cs.append(c)
            ss.append(s[..., 0])
            vref.append(torch.from_numpy(ofp8.dequantize_v(c, s)).to(torch.bfloat16))
        kp, vp, sp = opg.build_pools([u16(k) for k in ks], cs, pt, num_pages, ss)
    else:
        kp, vp, sp = opg.build_pools([u16(k) for k in ks], [u16(v) for v in vs], pt, num_pages)
        vref = vs
    return kp, vp, sp, vref


def build_cache(lens, KV, D, *, fp8, seed, over_provision=4, num_layers=1, capacity=None):
    """A PagedKVCache (device) holding seeded K/V, plus the reference-layout tensors
    the oracle attends over: (cache, k_list, v_ref_list) with v_ref = dequantised V for fp8."""
    ks, vs = seeded_kv(lens, KV, D, seed, fp8)
    cache, vref = cache_from_kv(ks, vs, KV, D, fp8=fp8, seed=seed, over_provision=over_provision,
                                num_layers=num_layers, capacity=capacity or max(lens))
    return cache, ks, vref


def cache_from_kv(ks, vs, KV, D, *, fp8, seed, capacity, over_provision=4, num_layers=1):
    from specdec_b200.engine.paged_cache import PagedKVCache

    lens = [k.shape[1] for k in ks]
    cap = capacity
    max_pages = (cap + 15) // 16
    num_pages = len(lens) * max_pages * over_provision
    pt = opg.random_page_table(len(lens), max_pages, num_pages, seed)
    kp, vp, sp, vref = oracle_pools(ks, vs, pt, num_pages, fp8)
    cache = PagedKVCache.allocate(num_layers, len(lens), KV, D, cap, v_dtype="e4m3" if fp8 else "bf16",
                                  device="cuda", num_pages=num_pages)
    cache.page_table.copy_(torch.from_numpy(pt))
    for pool in cache.pools:
        pool.k.copy_(torch.from_numpy(kp.view(np.int16)).view(torch.bfloat16))
        if fp8:
            pool.v.copy_(torch.from_numpy(vp))
            pool.v_scale.copy_(torch.from_numpy(sp))
        else:
            pool.v.copy_(torch.from_numpy(vp.view(np.int16)).view(torch.bfloat16))
    cache.set_host_lengths(list(lens))
    return cache, vref


def oracle_rows(q_rows, ks, vrefs, q_lens, eager=False):
    return oatt.ragged_attention(q_rows.cpu(), ks, vrefs, q_lens, fp32=not eager)


def assert_close_attention(got, ref, what=""):
    """Elementwise bar against the fp32 formula (reference.attention_fp32)."""
    ok, max_err, excess = oatt.within_tolerance(got, ref, RTOL, ATOL)
    assert ok, f"{what}: max |err| {max_err:.3e}, worst excess over tolerance {excess:.3e}"
    return max_err


def assert_close_eager(got, ref, what=""):
    """Bar against the eager engine path (reference.attention), whose scores are rounded to
    bf16 before the softmax: the reference's own bf16 check (sample_experiment.py:45-47),
    max |err| <= 2e-2 or <= 2 % of the output magnitude."""
    err = (got.float().cpu() - ref.float().cpu()).abs().max().item()
    scale = ref.float().abs().max().item()
    assert torch.isfinite(got.float()).all(), f"{what}: non-finite output"
    assert err <= 2e-2 or err <= 0.02 * max(scale, 1e-6), f"{what}: max |err| {err:.3e} (scale {scale:.3e})"
    return err
