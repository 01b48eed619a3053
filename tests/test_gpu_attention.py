"""GPU parity of the attention kernels against the oracle and the reference's golden outputs.

Tolerance: against the fp32 formula (reference.attention_fp32) every bf16 output element
satisfies |got - ref| <= 1e-2 + 2e-2 * |ref| (north star); against the eager engine path
(reference.attention, bf16-rounded scores) the reference's own bf16 check applies
(max |err| <= 2e-2 or <= 2 % of the output magnitude, sample_experiment.py:45-47);
the fp32 contiguous op is held to 1e-4 absolute (sample_experiment.py:21)."""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close_attention, assert_close_eager, build_cache, oracle_rows
from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _ops():
    from specdec_b200.kernels import ops

    return ops


def test_contiguous_attention_matches_golden(golden):
    ops = _ops()
    for name, case in golden["attention"].items():
        q, k, v = (case[x].cuda() for x in ("q", "k", "v"))
        got = ops.attention(q, k, v, backend="cuda").cpu()
        if q.dtype == torch.float32:
            torch.testing.assert_close(got, case["fp32"], rtol=0, atol=1e-4, msg=name)
            continue
        assert_close_eager(got, case["eager"], f"{name} vs eager")
        assert_close_attention(got, case["fp32"], f"{name} vs fp32")


@pytest.mark.parametrize("B,S,T", [(1, 1, 1), (1, 5, 5), (2, 5, 77), (1, 1, 300), (1, 5, 2048), (1, 5, 8192),
                                   (2, 2, 4093)])
def test_contiguous_attention_fp8v(B, S, T):
    """The contiguous op over a V-only FP8 dict cache's codes and scales (the patched forward's
    path) against the fp32 formula on the dequantised V (reference.attention_fp32 after
    dequantize_kv_fp8), including lengths that are not multiples of the 16-token page."""
    from oracle import engine as oeng
    from oracle import fp8 as ofp8

    ops = _ops()
    H, KV, D = 12, 2, 128
    g = torch.Generator().manual_seed(B * 100 + S + T)
    q = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, KV, T, D, generator=g).to(torch.bfloat16)
    v = torch.from_numpy(ofp8.outlier_v((B, KV, T, D), T + S)).to(torch.bfloat16)
    codes, scale = oeng.quantize_kv_fp8(v, 128)
    got = ops.attention_fp8v(q.cuda(), k.cuda(), codes.cuda(), scale.cuda()).cpu()
    vd = oeng.dequantize_kv_fp8(codes, scale, torch.bfloat16)
    assert_close_attention(got, oatt.attention_fp32(q, k, vd), f"fp8v B={B} S={S} T={T}")


@pytest.mark.parametrize("S,T", [(1, 1), (1, 15), (1, 16), (1, 17), (5, 5), (5, 21), (2, 300), (5, 2048), (64, 64)])
@pytest.mark.parametrize("H,KV,D", [(12, 2, 128), (14, 2, 64)])
def test_contiguous_attention_shapes(S, T, H, KV, D):
    ops = _ops()
    g = torch.Generator().manual_seed(S * 1000 + T + H)
    q = torch.randn(2, H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(2, KV, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(2, KV, T, D, generator=g).to(torch.bfloat16)
    got = ops.attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    assert_close_attention(got, oatt.attention_fp32(q, k, v), f"S={S} T={T}")
    assert_close_eager(got, oatt.eager_attention(q, k, v), f"S={S} T={T} eager")


def _paged_case(lens, q_lens, H, KV, D, fp8, seed):
    ops = _ops()
    cache, ks, vrefs = build_cache(lens, KV, D, fp8=fp8, seed=seed)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    g = torch.Generator().manual_seed(seed + 7)
    q = torch.randn(batch.total_rows, H, D, generator=g).to(torch.bfloat16)
    out = ops.paged_attention(q.cuda(), cache, 0, batch)
    torch.cuda.synchronize()
    return out.cpu(), oracle_rows(q, ks, vrefs, q_lens), q, ks, vrefs


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("S", [1, 2, 5])
@pytest.mark.parametrize("T", [5, 16, 17, 100, 2048, 4096, 8192])
def test_paged_attention_single_sequence(fp8, S, T):
    got, ref, *_ = _paged_case([T], [S], 12, 2, 128, fp8, seed=T * 10 + S)
    assert_close_attention(got, ref, f"fp8={fp8} S={S} T={T}")


@pytest.mark.parametrize("S", [1, 2, 5])
def test_paged_attention_draft_geometry(S):
    got, ref, *_ = _paged_case([333, 64], [S, S], 14, 2, 64, False, seed=3 + S)
    assert_close_attention(got, ref, f"14:2 d64 S={S}")


@pytest.mark.parametrize("H,KV", [(28, 4), (20, 2), (8, 1), (34, 2)])
@pytest.mark.parametrize("S", [1, 3])
def test_paged_attention_d64_head_pairs(H, KV, S):
    """head_dim 64 runs KV-head pairs as 128-dim groups (both heads' page blocks in one tile,
    each query row's dims in its own head's half) when the KV heads pair up and a pair's query
    rows fit the 32-row tile -- 28:4 (two pairs) and 20:2 -- and the 64-dim kernel otherwise
    (8:1, 34:2); every form against the oracle."""
    got, ref, *_ = _paged_case([900, 130, 8192], [S, S, S], H, KV, 64, False, seed=H * 10 + KV + S)
    assert_close_attention(got, ref, f"{H}:{KV} d64 S={S}")


def test_paged_attention_matches_eager_reference_fp8():
    got, _, q, ks, vrefs = _paged_case([2048], [5], 12, 2, 128, True, seed=99)
    ref = oracle_rows(q, ks, vrefs, [5], eager=True)
    assert_close_eager(got, ref, "fp8 vs eager")


@pytest.mark.parametrize("fp8", [False, True])
def test_ragged_batch_mixed_rows(fp8):
    """Mixed decode (q=1) and verify (q=5) rows, ragged lengths, one idle sequence, one launch."""
    rng = torch.Generator().manual_seed(5)
    lens = [int(x) for x in torch.randint(1, 3000, (15,), generator=rng)] + [40]
    q_lens = [1 if i % 2 else 5 for i in range(15)] + [0]
    lens = [max(n, q) for n, q in zip(lens, q_lens)]
    got, ref, *_ = _paged_case(lens, q_lens, 12, 2, 128, fp8, seed=17)
    assert_close_attention(got, ref, f"ragged fp8={fp8}")


@pytest.mark.parametrize("fp8,H,D", [(False, 12, 128), (True, 12, 128), (False, 14, 64), (False, 16, 128)])
def test_ragged_decode_rows(fp8, H, D):
    """Decode-only batches (at most 8 query rows per item: two warp groups on alternate
    tiles): one-tile items, CTAs with several items, direct and split items."""
    rng = torch.Generator().manual_seed(11 + H + D)
    lens = [int(x) for x in torch.randint(1, 5000, (40,), generator=rng)] + [1, 16, 17, 128, 129, 8192]
    q_lens = [1] * len(lens)
    got, ref, *_ = _paged_case(lens, q_lens, H, 2, D, fp8, seed=21)
    assert_close_attention(got, ref, f"decode rows fp8={fp8} H={H} D={D}")


@pytest.mark.parametrize("num_sms", [148, 97, 33, 8, 1])
@pytest.mark.parametrize("fp8", [False, True])
def test_grid_sizes(num_sms, fp8):
    """The same ragged batch on grids of every size: the plan's whole-tile CTA count for small
    calls with the blocks that get no pages placed first, grids with fewer CTAs than split
    rows (several merge rounds) and a single CTA that takes every item."""
    import ctypes

    from specdec_b200 import _lib

    ops = _ops()
    lens, q_lens = [8192, 3000, 77, 1, 640], [5, 1, 5, 1, 2]
    cache, ks, vrefs = build_cache(lens, 2, 128, fp8=fp8, seed=41)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    g = torch.Generator().manual_seed(43)
    q = torch.randn(batch.total_rows, 12, 128, generator=g).to(torch.bfloat16)
    qc = q.cuda()
    out = torch.empty_like(qc)
    args = ops.attn_args(qc, out, cache, 0, batch, ops.attn_workspace(batch, 12, cache))
    args.num_sms = num_sms
    _lib.check(ops._lib_handle().specdec_paged_attention(ctypes.byref(args), ops._stream()), "paged_attention")
    torch.cuda.synchronize()
    assert_close_attention(out.cpu(), oracle_rows(q, ks, vrefs, q_lens), f"num_sms={num_sms} fp8={fp8}")


def test_ragged_config4_full_size():
    """The ragged config at its full size (64 sequences, T ~ U[1024, 8192], q_len 1 and 5
    in a 1:1 seeded shuffle, E4M3 V): every output row against the oracle."""
    g = torch.Generator().manual_seed(4)
    lens = [int(x) for x in torch.randint(1024, 8193, (64,), generator=g)]
    q_lens = [1, 5] * 32
    perm = torch.randperm(64, generator=g).tolist()
    q_lens = [q_lens[i] for i in perm]
    ops = _ops()
    cache, ks, vrefs = build_cache(lens, 2, 128, fp8=True, seed=4, over_provision=1)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, 12, 128, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    got = ops.paged_attention(q.cuda(), cache, 0, batch).cpu()
    assert_close_attention(got, oracle_rows(q, ks, vrefs, q_lens), "ragged config 4")


def test_ragged_config4_verify_accept_trim_cycle():
    """The ragged config's whole cycle (64 sequences, T ~ U[1024, 8192], q_len 1 and 5 in a
    1:1 seeded shuffle, E4M3 V), for 4 rounds: append each sequence's q_len new tokens
    (append_kv: bf16 K, E4M3 V), attention over the grown history, then for every verify
    row an accepted count m ~ min(Geometric(0.5) - 1, 4) and the device rollback of the
    rejected tail (trim_lengths to len + 1 + m: the verify block's pending token plus the
    m accepted candidates, spec_dec.py:235-243); decode rows keep their token.  After every
    round the lengths, the page table and the FP8 codes / scales and bf16 K of every kept
    token are bit-exact against the oracle's restatement of the same cycle, and every
    output row is within the attention tolerance of the oracle's attention."""
    from oracle import fp8 as ofp8

    ops = _ops()
    g = torch.Generator().manual_seed(4)
    lens = [int(x) for x in torch.randint(1024, 8193, (64,), generator=g)]
    q_lens = [1, 5] * 32
    perm = torch.randperm(64, generator=g).tolist()
    q_lens = [q_lens[i] for i in perm]
    rounds, KV, D, H = 4, 2, 128, 12
    cache, ks, _ = build_cache(lens, KV, D, fp8=True, seed=4, over_provision=1, capacity=max(lens) + 5 * rounds)
    # the oracle keeps the bf16 K / V token lists of every sequence
    from gpu_helpers import seeded_kv

    _, vs = seeded_kv(lens, KV, D, 4, True)
    ks, vs = list(ks), list(vs)
    pt0 = cache.page_table.clone()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    batch = None
    for r in range(rounds):
        gr = torch.Generator().manual_seed(100 + r)
        n_rows = sum(q_lens)
        k_rows = torch.randn(n_rows, KV, D, generator=gr).to(torch.bfloat16)
        v_rows = torch.from_numpy(ofp8.outlier_v((n_rows, KV, D), 200 + r)).to(torch.bfloat16)
        row0 = [sum(q_lens[:b]) for b in range(64)]
        i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")  # noqa: E731
        ops.append_kv(k_rows.cuda(), v_rows.cuda(), cache, 0, row0=i32(row0), n_new=i32(q_lens), pos0=i32(lens),
                      max_new=5, len_out=cache.lengths, status=status)
        for b in range(64):
            sl = slice(row0[b], row0[b] + q_lens[b])
            ks[b] = torch.cat([ks[b], k_rows[sl].transpose(0, 1)], dim=1)
            vs[b] = torch.cat([vs[b], v_rows[sl].transpose(0, 1)], dim=1)
        grown = [n + q for n, q in zip(lens, q_lens)]
        batch = ops.RaggedBatch.from_lengths(q_lens, grown)
        q = torch.randn(batch.total_rows, H, D, generator=gr).to(torch.bfloat16)
        got = ops.paged_attention(q.cuda(), cache, 0, batch, status=status).cpu()
        vrefs = []
        for v in vs:
            c, sc = ofp8.quantize_v(v.float().numpy())
            vrefs.append(torch.from_numpy(ofp8.dequantize_v(c, sc)).to(torch.bfloat16))
        assert_close_attention(got, oracle_rows(q, ks, vrefs, q_lens), f"cycle round {r}")
        # accept + rollback of the verify rows
        m = []
        for b in range(64):
            u = torch.rand(1, generator=gr).item()
            geo = 0
            while u < 0.5 ** (geo + 1) and geo < 4:  # P(m >= j) = 0.5 ** j, truncated at 4
                geo += 1
            m.append(geo)
        new_len = [n + 1 + mm if q == 5 else n + 1 for n, q, mm in zip(lens, q_lens, m)]
        ops.trim_lengths(cache.lengths, i32(new_len), out=cache.lengths, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"round {r}: status {int(status.item()):#x}"
        lens = new_len
        ks = [k[:, :n] for k, n in zip(ks, lens)]
        vs = [v[:, :n] for v, n in zip(vs, lens)]
        assert cache.lengths.cpu().tolist() == lens
        assert torch.equal(cache.page_table, pt0)
        for b in range(0, 64, 7 if r < rounds - 1 else 1):
            kept = cache.gather_layer(0, b, lens[b])
            codes, sc = ofp8.quantize_v(vs[b].float().numpy())
            assert torch.equal(kept["k"][0].cpu().view(torch.int16), ks[b].view(torch.int16)), f"K seq {b} round {r}"
            assert (kept["v"][0].view(torch.uint8).cpu().numpy() == codes).all(), f"codes seq {b} round {r}"
            assert (kept["v_scale"][0, :, :, 0].cpu().numpy().view("u4") == sc[..., 0].view("u4")).all(), \
                f"scales seq {b} round {r}"


def test_draft_decode_full_size():
    """The draft model's decode attention at the bench's size (64 sequences x 8192, q_len 1,
    14:2 heads, head_dim 64, bf16 K/V): every output row against the oracle."""
    ops = _ops()
    lens, q_lens = [8192] * 64, [1] * 64
    cache, ks, vrefs = build_cache(lens, 2, 64, fp8=False, seed=5, over_provision=1)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, 14, 64, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    got = ops.paged_attention(q.cuda(), cache, 0, batch).cpu()
    assert_close_attention(got, oracle_rows(q, ks, vrefs, q_lens), "draft decode 64 x 8K")


@pytest.mark.parametrize("cluster_size", [1, 8, 16])
@pytest.mark.parametrize("lens,q_lens,fp8,H,D", [
    ([8192], [5], False, 12, 128),
    ([8192], [1], True, 12, 128),
    ([4096], [5], True, 12, 128),
    ([2048], [2], False, 14, 64),
    ([100], [5], False, 12, 128),
    ([5], [5], True, 12, 128),
    ([3000, 77, 1, 640], [5, 1, 5, 2], True, 12, 128),
    ([8192, 0, 2500], [1, 0, 1], False, 14, 64),
    ([1024], [1], False, 12, 128),
    ([1024, 1024], [5, 1], True, 12, 128),
])
def test_small_batches_on_clusters(cluster_size, lens, q_lens, fp8, H, D):
    """Small batches with every (sequence, query tile, KV head) group on thread-block clusters
    of its own (8 or 16 CTAs: the split partials reduced in distributed shared memory, groups
    spread over several clusters joined by per-row tickets) and on the persistent grid (1),
    against the oracle; a plan reused by the following calls of a step gives the same rows.
    On the persistent grid most of these calls take the spare-block merge (blocks without
    pages merge the split rows, wide and narrow); 3000/77/1/640 does not fit it."""
    ops = _ops()
    lens = [max(n, q) for n, q in zip(lens, q_lens)]
    lens_cache = [max(n, 1) for n in lens]
    cache, ks, vrefs = build_cache(lens_cache, 2, D, fp8=fp8, seed=sum(lens) + cluster_size, num_layers=2)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, H, D, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    qc = q.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = ops.attn_workspace(batch, H, cache)
    ops.ragged_plan(qc, cache, batch, ws, status=status, cluster_size=cluster_size)
    outs = [ops.paged_attention(qc, cache, layer, batch, workspace=ws, reuse_plan=True, status=status,
                                history_ready=layer > 0, cluster_size=cluster_size) for layer in range(2)]
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    keep = [i for i, n in enumerate(q_lens) if n > 0]
    row0 = [sum(q_lens[:i]) for i in range(len(q_lens))]
    rows = torch.cat([torch.arange(row0[i], row0[i] + q_lens[i]) for i in keep])
    ref = oracle_rows(q[rows], [ks[i] for i in keep], [vrefs[i] for i in keep], [q_lens[i] for i in keep])
    for o in outs:
        assert_close_attention(o.cpu()[rows], ref, f"clusters={cluster_size} lens={lens} q={q_lens}")
    assert torch.equal(outs[0], outs[1])


def test_library_cluster_choice():
    """The library's own choice (cluster_size 0): clusters only for a small batch whose host-known
    context bound puts every group on one cluster at one tile per CTA; the persistent grid for
    long contexts, for an unknown bound and for large batches."""
    ops = _ops()
    cache, *_ = build_cache([16], 2, 128, fp8=False, seed=1)
    q = torch.zeros(5, 12, 128, dtype=torch.bfloat16, device="cuda")

    def shape(q_lens, ctx, known=True):
        batch = ops.RaggedBatch.from_lengths(q_lens, ctx)
        if not known:
            batch.max_ctx_len = 0
        return ops.launch_shape(q, cache, batch, ops.attn_workspace(batch, 12, cache))

    grid, cs = shape([5], [2048])
    assert cs in (8, 16) and grid % cs == 0
    assert shape([5], [8192])[1] == 0
    assert shape([5], [2048], known=False)[1] == 0
    assert shape([1] * 64, [1024] * 64)[1] == 0


def test_plan_built_for_another_launch_shape_is_refused():
    """A plan reused by a call that would launch another grid (clusters of 8 against clusters
    of 16, or the persistent grid) is detected on the device: the call sets
    SPECDEC_STATUS_PLAN_MISMATCH and computes nothing, in every CTA alike."""
    from specdec_b200 import _lib

    ops = _ops()
    cache, ks, vrefs = build_cache([4096], 2, 128, fp8=False, seed=3)
    batch = ops.RaggedBatch.from_lengths([5], [4096])
    q = torch.randn(5, 12, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    ws = ops.attn_workspace(batch, 12, cache)
    for planned, used in ((8, 16), (16, 1), (1, 8)):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        ops.ragged_plan(q, cache, batch, ws, cluster_size=planned)
        ops.paged_attention(q, cache, 0, batch, workspace=ws, reuse_plan=True, status=status, cluster_size=used)
        torch.cuda.synchronize()
        assert int(status.item()) & _lib.STATUS_PLAN_MISMATCH, (planned, used)
    # and the matching plan still works afterwards
    ops.ragged_plan(q, cache, batch, ws, cluster_size=16)
    out = ops.paged_attention(q, cache, 0, batch, workspace=ws, reuse_plan=True, cluster_size=16)
    assert_close_attention(out.cpu(), oracle_rows(q.cpu(), ks, vrefs, [5]), "matching plan")


def test_plan_reuse_across_layers():
    """One plan serves every layer: reuse_plan=True gives the same output as a fresh plan."""
    ops = _ops()
    lens, q_lens = [700, 1500, 64], [5, 1, 5]
    cache, ks, vrefs = build_cache(lens, 2, 128, fp8=True, seed=8, num_layers=2)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, 12, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    ws = ops.attn_workspace(batch, 12, cache)
    ops.ragged_plan(q, cache, batch, ws)
    a = ops.paged_attention(q, cache, 1, batch, workspace=ws, reuse_plan=True)
    b = ops.paged_attention(q, cache, 1, batch)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("fp8,D,q_lens", [(False, 128, [5, 1, 2, 5]), (True, 128, [5, 1, 2, 5]),
                                          (False, 64, [5, 1, 2, 5]), (True, 128, [1, 1, 1, 1]),
                                          (False, 64, [1, 2, 1, 1])])
def test_history_ready_gives_identical_results(fp8, D, q_lens):
    """Loading the plan, page table and KV history before the dependency wait changes
    no result: a layer stack with history_ready equals the same calls without it (verify
    rows, decode rows, and the draft's q = 2 catch-up)."""
    ops = _ops()
    lens = [900, 4100, 33, 2000]
    H = 12 if D == 128 else 14
    cache, ks, vrefs = build_cache(lens, 2, D, fp8=fp8, seed=9, num_layers=3)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, H, D, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    ws = ops.attn_workspace(batch, H, cache)
    ops.ragged_plan(q, cache, batch, ws)
    early = [ops.paged_attention(q, cache, layer, batch, workspace=ws, reuse_plan=True, history_ready=layer > 0)
             for layer in range(3)]
    plain = [ops.paged_attention(q, cache, layer, batch) for layer in range(3)]
    torch.cuda.synchronize()
    for a, b in zip(early, plain):
        assert torch.equal(a, b)


def test_bad_page_id_sets_status_without_fault():
    """A corrupted page table (host-side) is caught by the producer's bounds check."""
    from specdec_b200 import _lib

    ops = _ops()
    cache, ks, vrefs = build_cache([100], 2, 128, fp8=False, seed=4)
    cache.page_table[0, 2] = cache.num_pages + 5
    batch = ops.RaggedBatch.from_lengths([1], [100])
    q = torch.randn(1, 12, 128, device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.paged_attention(q, cache, 0, batch, status=status)
    assert int(status.item()) & _lib.STATUS_BAD_PAGE


def test_length_overflow_sets_status():
    from specdec_b200 import _lib

    ops = _ops()
    cache, *_ = build_cache([32], 2, 128, fp8=False, seed=6)
    batch = ops.RaggedBatch.from_lengths([1, 5], [10 ** 6, 2])  # beyond the page table; ctx < q_len
    from specdec_b200.engine.paged_cache import PagedKVCache

    big = PagedKVCache.allocate(1, 2, 2, 128, 32, device="cuda")
    q = torch.zeros(6, 12, 128, device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.paged_attention(q, big, 0, batch, status=status)
    s = int(status.item())
    assert s & _lib.STATUS_PAGE_OVERFLOW and s & _lib.STATUS_BAD_LENGTH
    del cache


def test_cuda_graph_replay_matches_eager():
    ops = _ops()
    lens, q_lens = [1000, 2500], [5, 5]
    cache, ks, vrefs = build_cache(lens, 2, 128, fp8=True, seed=12)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, 12, 128, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    ws = ops.attn_workspace(batch, 12, cache)
    out = torch.empty_like(q)
    ops.paged_attention(q, cache, 0, batch, out=out, workspace=ws)  # warm-up outside capture
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            ops.paged_attention(q, cache, 0, batch, out=out, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert_close_attention(out.cpu(), oracle_rows(q.cpu(), ks, vrefs, q_lens), "graph replay")
