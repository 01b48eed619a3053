"""GPU: quantise-on-append writes exactly the oracle's pool bytes (FP8 codes, scales,
bf16 K/V, page placement) -- the reference's quantize_kv_fp8 contract, bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_helpers import cache_from_kv, oracle_pools, seeded_kv, u16
from oracle import paged as opg

pytestmark = pytest.mark.gpu


def _ops():
    from specdec_b200.kernels import ops

    return ops


@pytest.mark.parametrize("fp8,D", [(True, 128), (False, 128), (False, 64)])
def test_append_matches_oracle_pools(fp8, D):
    ops = _ops()
    KV = 2
    before = [1, 13, 100, 16, 250]
    n_new = [16, 5, 1, 33, 0]
    cap = 320
    ks_old, vs_old = seeded_kv(before, KV, D, seed=21, fp8=fp8)
    ks_new, vs_new = seeded_kv(n_new, KV, D, seed=22, fp8=fp8)
    if fp8:
        # a NaN in one V row: torch's amax keeps it, so that row's scale and codes are NaN
        vs_new[1][1, 2, 17] = float("nan")
    cache, _ = cache_from_kv(ks_old, vs_old, KV, D, fp8=fp8, seed=23, capacity=cap)
    # packed new rows (rows, KV, D)
    k_rows = torch.cat([k.permute(1, 0, 2) for k in ks_new], dim=0).contiguous().cuda()
    v_rows = torch.cat([v.permute(1, 0, 2) for v in vs_new], dim=0).contiguous().cuda()
    row0 = torch.tensor(np.cumsum([0] + n_new[:-1]), dtype=torch.int32, device="cuda")
    nn = torch.tensor(n_new, dtype=torch.int32, device="cuda")
    pos0 = torch.tensor(before, dtype=torch.int32, device="cuda")
    len_out = torch.zeros(len(before), dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.append_kv(k_rows, v_rows, cache, 0, row0=row0, n_new=nn, pos0=pos0, max_new=max(n_new), len_out=len_out,
                  status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert len_out.cpu().tolist() == [a + b for a, b in zip(before, n_new)]

    ks_all = [torch.cat([a, b], dim=1) for a, b in zip(ks_old, ks_new)]
    vs_all = [torch.cat([a, b], dim=1) for a, b in zip(vs_old, vs_new)]
    pt = cache.page_table.cpu().numpy()
    kp, vp, sp, _ = oracle_pools(ks_all, vs_all, pt, cache.num_pages, fp8)
    pool = cache.pools[0]
    np.testing.assert_array_equal(pool.k.cpu().view(torch.int16).numpy().view(np.uint16), kp)
    if fp8:
        np.testing.assert_array_equal(pool.v.cpu().numpy(), vp)
        np.testing.assert_array_equal(pool.v_scale.cpu().numpy().view(np.uint32), sp.view(np.uint32))
    else:
        np.testing.assert_array_equal(pool.v.cpu().view(torch.int16).numpy().view(np.uint16), vp)


def test_append_full_history_fp8_8k():
    """Quantise an 8192-token V history (the FP8 config) and gather it back bit-exactly."""
    ops = _ops()
    from oracle import fp8 as ofp8
    from specdec_b200.engine.paged_cache import PagedKVCache

    T, KV, D = 8192, 2, 128
    ks, vs = seeded_kv([T], KV, D, seed=31, fp8=True)
    cache = PagedKVCache.allocate(1, 1, KV, D, T, v_dtype="e4m3", device="cuda", page_order_seed=5)
    ops.append_kv(ks[0].permute(1, 0, 2).contiguous().cuda(), vs[0].permute(1, 0, 2).contiguous().cuda(), cache, 0,
                  row0=torch.zeros(1, dtype=torch.int32, device="cuda"),
                  n_new=torch.tensor([T], dtype=torch.int32, device="cuda"),
                  pos0=torch.zeros(1, dtype=torch.int32, device="cuda"), max_new=T)
    got = cache.gather_layer(0, 0, T)
    codes, scale = ofp8.quantize_v(vs[0].float().numpy())
    np.testing.assert_array_equal(got["v"][0].view(torch.uint8).cpu().numpy(), codes)
    np.testing.assert_array_equal(got["v_scale"][0, :, :, 0].cpu().numpy().view(np.uint32),
                                  scale[..., 0].view(np.uint32))
    assert torch.equal(got["k"][0].cpu().view(torch.int16), ks[0].view(torch.int16))


def test_append_bad_position_sets_status():
    from specdec_b200 import _lib

    ops = _ops()
    ks, vs = seeded_kv([4], 2, 128, seed=3, fp8=True)
    cache, _ = cache_from_kv(ks, vs, 2, 128, fp8=True, seed=4, capacity=16)
    k = torch.zeros(1, 2, 128, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    one = torch.ones(1, dtype=torch.int32, device="cuda")
    ops.append_kv(k, k, cache, 0, row0=torch.zeros_like(one), n_new=one, pos0=one * 16, max_new=1, status=status)
    assert int(status.item()) & _lib.STATUS_PAGE_OVERFLOW


def test_gather_layer_round_trip():
    ks, vs = seeded_kv([77, 3], 2, 128, seed=9, fp8=False)
    cache, _ = cache_from_kv(ks, vs, 2, 128, fp8=False, seed=10, capacity=80)
    for b, n in enumerate([77, 3]):
        got = cache.gather_layer(0, b, n)
        assert torch.equal(got["k"][0].cpu().view(torch.int16), ks[b].view(torch.int16))
        assert torch.equal(got["v"][0].cpu().view(torch.int16), vs[b].view(torch.int16))
    k_np, _, _ = opg.gather(cache.pools[0].k.cpu().view(torch.int16).numpy().view(np.uint16),
                            cache.pools[0].v.cpu().view(torch.int16).numpy().view(np.uint16), None,
                            cache.page_table.cpu().numpy(), 0, 77)
    np.testing.assert_array_equal(k_np, u16(ks[0]))


@pytest.mark.parametrize("fp8,H,D", [(True, 12, 128), (False, 12, 128), (False, 14, 64)])
def test_rope_append_matches_oracle(fp8, H, D):
    """The fused step seam (one launch after the QKV projection) against the oracle: the
    rotated queries equal reference.apply_rope (specdec/kernels/reference.py:23-27) of q,
    bit for bit, and the pool holds apply_rope of k and the quantize_kv_fp8 codes and scales
    of v (model_self.py:304-314) at the appended positions, bit for bit.  The unfused
    kernels (apply_rope, then append_kv) write the same bytes."""
    from oracle import elementwise as oel
    from oracle import fp8 as ofp8
    from specdec_b200.engine.paged_cache import PagedKVCache

    ops = _ops()
    KV, B, qmax = 2, 5, 5
    before = [1, 13, 100, 16, 250]
    q_len = [5, 1, 3, 5, 0]
    rows = B * qmax
    g = torch.Generator().manual_seed(31)
    qkv_h = (torch.randn(rows, H + 2 * KV, D, generator=g) * 2.0).to(torch.bfloat16)
    # the engine's tables: cos / sin of fp32 angles at each row's position, rounded to bf16
    pos = torch.tensor([before[r // qmax] + min(r % qmax, max(q_len[r // qmax] - 1, 0)) for r in range(rows)],
                       dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.outer(pos, inv)
    cos_h = torch.cat([ang.cos(), ang.cos()], -1).to(torch.bfloat16)
    sin_h = torch.cat([ang.sin(), ang.sin()], -1).to(torch.bfloat16)
    qkv, cos, sin = qkv_h.cuda(), cos_h.cuda(), sin_h.cuda()
    row0 = torch.arange(B, dtype=torch.int32, device="cuda") * qmax
    nn = torch.tensor(q_len, dtype=torch.int32, device="cuda")
    pos0 = torch.tensor(before, dtype=torch.int32, device="cuda")
    caches = [PagedKVCache.allocate(1, B, KV, D, 320, v_dtype="e4m3" if fp8 else "bf16", device="cuda",
                                    page_order_seed=4) for _ in range(2)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    q_fused = ops.rope_append(qkv, cos, sin, caches[0], 0, num_q_heads=H, row0=row0, n_new=nn, pos0=pos0,
                              max_new=qmax, status=status)
    # unfused: rope of q and k as (1, heads, rows, D) views, then append
    k_rot = ops.apply_rope(qkv[:, H:H + KV].transpose(0, 1).unsqueeze(0), cos, sin)[0].transpose(0, 1)
    ops.append_kv(k_rot.contiguous(), qkv[:, H + KV:].contiguous(), caches[1], 0, row0=row0, n_new=nn, pos0=pos0,
                  max_new=qmax, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0

    # oracle: the reference formula on (heads, rows, D) views, per-row cos / sin
    c4, s4 = cos_h.unsqueeze(0), sin_h.unsqueeze(0)
    q_ref = oel.apply_rope(qkv_h[:, :H].transpose(0, 1), c4, s4).transpose(0, 1)
    k_ref = oel.apply_rope(qkv_h[:, H:H + KV].transpose(0, 1), c4, s4)  # (KV, rows, D)
    v_in = qkv_h[:, H + KV:].transpose(0, 1)                             # (KV, rows, D)
    assert torch.equal(q_fused.cpu().view(torch.int16), q_ref.contiguous().view(torch.int16))
    for b in range(B):
        n = q_len[b]
        if n == 0:
            continue
        sl = slice(b * qmax, b * qmax + n)
        got = caches[0].gather_layer(0, b, before[b] + n)
        assert torch.equal(got["k"][0, :, before[b]:].cpu().view(torch.int16), k_ref[:, sl].contiguous().view(torch.int16))
        if fp8:
            codes, scale = ofp8.quantize_v(v_in[:, sl].float().numpy())
            np.testing.assert_array_equal(got["v"][0, :, before[b]:].view(torch.uint8).cpu().numpy(), codes)
            np.testing.assert_array_equal(got["v_scale"][0, :, before[b]:, 0].cpu().numpy().view(np.uint32),
                                          scale[..., 0].view(np.uint32))
        else:
            assert torch.equal(got["v"][0, :, before[b]:].cpu().view(torch.int16), v_in[:, sl].contiguous().view(torch.int16))
    a, b2 = caches[0].pools[0], caches[1].pools[0]
    assert torch.equal(a.k.view(torch.int16), b2.k.view(torch.int16))
    assert torch.equal(a.v.view(torch.uint8), b2.v.view(torch.uint8))
    if fp8:
        assert torch.equal(a.v_scale, b2.v_scale)
