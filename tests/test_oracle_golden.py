"""The CPU oracle is pinned against golden vectors produced by the live reference
(tests/golden/make_golden.py) and against torch's own float8 cast."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as oacc
from oracle import attention as oatt
from oracle import fp8 as ofp8
from oracle import paged as opg
from oracle import spec_cache as osc


def test_attention_oracle_matches_reference(golden):
    for name, case in golden["attention"].items():
        q, k, v = case["q"], case["k"], case["v"]
        eager = oatt.eager_attention(q, k, v)
        assert eager.dtype == case["eager"].dtype
        # same torch ops on the same inputs: identical bits expected; allow 1 bf16 ulp for a
        # different CPU kernel path
        torch.testing.assert_close(eager.float(), case["eager"].float(), rtol=8e-3, atol=1e-3, msg=name)
        fp32 = oatt.attention_fp32(q, k, v)
        torch.testing.assert_close(fp32.float(), case["fp32"].float(), rtol=8e-3, atol=1e-4, msg=name)


def test_mask_rule():
    m = oatt.offset_causal_mask(5, 8)
    # row i sees j <= i + 3
    for i in range(5):
        assert m[i].tolist() == [j > i + 3 for j in range(8)]
    assert not oatt.offset_causal_mask(1, 9).any()  # decode sees every key


def test_fp8_oracle_matches_reference_bit_exact(golden):
    for name, case in golden["fp8"].items():
        codes, scale = ofp8.quantize_v(case["x"].float().numpy())
        np.testing.assert_array_equal(codes, case["codes"].numpy(), err_msg=name)
        np.testing.assert_array_equal(scale.view(np.uint32), case["scale"].float().numpy().view(np.uint32),
                                      err_msg=name)
        deq = torch.from_numpy(ofp8.dequantize_v(codes, scale)).to(torch.bfloat16)
        assert torch.equal(deq.view(torch.int16), case["deq"].view(torch.int16)), name


def test_fp8_edge_semantics(golden):
    e = golden["fp8"]["edge"]
    codes, scale = e["codes"].numpy(), e["scale"].numpy()
    assert scale[0, 0, 0, 0] == 1.0 and not codes[0, 0, 0].any()  # zero group: scale 1, codes 0
    assert codes[0, 0, 1, 3] == 0x7E  # the max element maps to 448
    assert (codes[0, 0, 2] == 0x80).all()  # -0.0 keeps its sign


def test_e4m3_conversion_matches_torch_cast():
    rng = np.random.default_rng(3)
    x = np.concatenate([
        rng.uniform(-470, 470, 200_000),
        rng.standard_normal(200_000) * 1e-2,
        (np.arange(65536, dtype=np.uint32) << 16).view(np.float32),
    ]).astype(np.float32)
    ours = ofp8.f32_to_e4m3(x)
    ref = torch.from_numpy(x.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, ref)


def test_spec_cache_oracle_matches_reference(golden):
    def mk(n):
        return [{"k": torch.zeros(1, 2, n, 4), "v": torch.zeros(1, 2, n, 4), "fmt": "fp16"} for _ in range(2)]

    for rec in golden["spec_cache"]["trim"]:
        cache = mk(rec["cur"]) if rec["cur"] is not None else None
        if rec["ok"]:
            t = osc.trim_cache(cache, rec["req"])
            assert osc.cache_length(t) == rec["new_len"]
            assert osc.cache_length(cache) == rec["orig_len"]
        else:
            with pytest.raises(ValueError):
                osc.trim_cache(cache, rec["req"])
    shapes = [((1, 2, 8, 4), 8), ((1, 2, 7, 4), 8), ((1, 2, 8, 4), 6)]
    for (shape_v, layer2), ok in zip(shapes, golden["spec_cache"]["consistent"]):
        c = [{"k": torch.zeros(1, 2, 8, 4), "v": torch.zeros(*shape_v)},
             {"k": torch.zeros(1, 2, layer2, 4), "v": torch.zeros(1, 2, layer2, 4)}]
        if ok:
            osc.check_consistent(c)
        else:
            with pytest.raises(RuntimeError):
                osc.check_consistent(c)


def test_accept_oracle_matches_reference(golden):
    for case in golden["accept"]:
        stack = case["stack"].float().numpy()
        cands = case["cands"].tolist()
        g, m = oacc.vector_accept(stack[0], stack[1:], cands)
        assert g == case["g"].tolist()
        assert m == case["m"]
        g2, m2, nxt, la = oacc.rows_accept(list(stack), cands, len(cands), len_before=10, keep_offset=1)
        assert g2 == case["g"].tolist() and m2 == case["m"] and la == 11 + m2


def test_accept_trace_rules(golden):
    """Control traces of the reference executors obey the accept/rollback rules the kernels implement."""
    for tr in golden["traces"]:
        assert tr["gen"] == tr["fast_gen"]
        for row in tr["control"]:
            kp, m, g, cands = row["Kp"], row["m"], row["g"], row["cands"]
            mm = 0
            while mm < kp and g[mm] == cands[mm]:
                mm += 1
            assert mm == m
            if m < kp:
                assert row["emitted"] == cands[:m] + [g[m]]
                assert row["tgt_len"] == row["pre"] + m + 1 and row["drf_len"] == row["pre"] + m + 1
            else:
                assert row["emitted"] == cands and row["tgt_len"] == row["pre"] + kp


def test_paged_pack_gather_round_trip():
    rng = np.random.default_rng(5)
    KV, D = 2, 128
    lens = [37, 16, 1]
    max_pages = 3
    pt = opg.random_page_table(3, max_pages, 12, seed=2)
    ks = [rng.integers(0, 65535, (KV, n, D), dtype=np.uint16) for n in lens]
    vs = [rng.integers(0, 255, (KV, n, D), dtype=np.uint8) for n in lens]
    ss = [rng.random((KV, n)).astype(np.float32) for n in lens]
    kp, vp, sp = opg.build_pools(ks, vs, pt, 12, ss)
    for b, n in enumerate(lens):
        k, v, s = opg.gather(kp, vp, sp, pt, b, n)
        np.testing.assert_array_equal(k, ks[b])
        np.testing.assert_array_equal(v, vs[b])
        np.testing.assert_array_equal(s, ss[b])


def test_product_layout_matches_oracle_layout():
    from specdec_b200.engine import paged_cache as pc

    for D in (64, 128):
        assert pc.kblock_index(D).tolist() == opg.kblock_perm(D).tolist()
    assert pc.vblock_index(128).tolist() == opg.vblock_perm(128).tolist()
    # the bf16 block permutation is a bijection onto the block
    assert sorted(opg.kblock_perm(128).tolist()) == list(range(16 * 128))


def test_elementwise_oracle_matches_reference(golden):
    """oracle/elementwise.py against reference.rmsnorm / apply_rope / swiglu
    (specdec/kernels/reference.py:14-31): the same torch ops, bit-identical results."""
    from oracle import elementwise as oel

    cases = golden["elementwise"]
    assert len(cases) == 16
    for name, c in cases.items():
        if name.startswith("rmsnorm"):
            got = oel.rmsnorm(c["x"], c["w"])
        elif name.startswith("rope"):
            got = oel.apply_rope(c["x"], c["cos"], c["sin"])
        else:
            got = oel.swiglu(c["gate"], c["up"])
        assert got.dtype == c["out"].dtype, name
        assert torch.equal(got, c["out"]), name


def _golden_model(golden):
    import oracle.engine as oeng

    g = golden["model"]
    c = g["config"]
    m = oeng.QwenLM(c["vocab"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["intermediate"], c["layers"],
                    rope_theta=c["rope_theta"], attn_bias=c["attn_bias"]).to(torch.bfloat16)
    m.load_state_dict(g["state"], strict=True)
    return m.eval(), g


@pytest.mark.parametrize("fmt", ["fp16", "v_fp8"])
def test_engine_oracle_matches_reference_model(golden, fmt):
    """oracle/engine.py (the model-level restatement the engine tests use) against a tiny
    reference QwenLM (model_self.py:835-931) with the same weights: prompt-pass logits,
    a 5-token verify block on the prompt's dict cache, and greedy decoding, for the bf16
    and V-only FP8 cache formats.  Same torch CPU ops: identical bits."""
    import oracle.engine as oeng

    m, g = _golden_model(golden)
    m.set_kv_format(fmt)
    want = g[fmt]
    with torch.inference_mode():
        lg, cache = m._run(m.embed_tokens(g["prompt"]), None)
        assert torch.equal(lg[0, -1], want["prompt_logits"])
        vb, _ = m._run(m.embed_tokens(g["block"]), cache)
        assert torch.equal(vb[0], want["verify_logits"])
        toks, _ = oeng.greedy_decode(m, g["prompt"], len(want["greedy"]))
    assert toks == want["greedy"]


def test_specdec_oracle_replays_reference_executor_traces(golden):
    """oracle/specdec.py (the strict executor restated, spec_dec.py:189-275) on the toy models
    the golden traces were recorded with: the same emitted tokens and, round by round, the
    same candidates, argmaxes, accepted counts, emitted tokens and cache lengths."""
    import importlib.util
    from pathlib import Path

    from oracle import specdec as osd

    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    for tr in golden["traces"]:
        tgt = mg.ToyLM(tr["vocab"], tr["hidden"], tr["seed"])
        drf = mg.ToyLM(tr["vocab"], tr["hidden"], tr["seed"] + 50, like=tgt, noise=tr["noise"])
        log = []
        res = osd.spec_decode_greedy(tgt, drf, tr["prompt"], tr["max_new"], k=4, log=log.append)
        assert res["gen"] == tr["gen"]
        assert len(log) == len(tr["control"])
        for mine, ref in zip(log, tr["control"]):
            for key in ("Kp", "m", "pre", "tgt_len", "drf_len", "cands", "g", "emitted"):
                assert mine[key] == ref[key], (tr["seed"], key)
