"""Generate the golden fixtures of tests/golden from the live reference.

Run in a checkout that has the reference repository importable:

    REFERENCE_ROOT=/path/to/SpecDec-Context-Scaling python tests/golden/make_golden.py

It imports the reference's own functions (specdec.kernels.reference.attention /
attention_fp32 / rmsnorm / apply_rope / swiglu, specdec.engine.model_self.quantize_kv_fp8 /
dequantize_kv_fp8 / QwenLM, specdec.engine.spec_cache,
specdec.engine.spec_dec.spec_decode_greedy and
experiments.execution_optimization.fast_spec_dec.spec_decode_greedy_optimized)
on seeded synthetic inputs and stores inputs and outputs in golden_v1.pt.
The GPU box never needs the reference: tests compare against this file.
REFERENCE_ROOT must be set; there is no default location.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ["REFERENCE_ROOT"]) if os.environ.get("REFERENCE_ROOT") else None


def _import_reference():
    if REF is None or not (REF / "specdec").exists():
        raise SystemExit(f"set REFERENCE_ROOT to a checkout of the reference (got {REF})")
    sys.path.insert(0, str(REF))
    from specdec.kernels import reference as kref  # noqa: E402
    from specdec.engine import model_self, spec_cache, spec_dec  # noqa: E402
    from experiments.execution_optimization import fast_spec_dec  # noqa: E402

    return kref, model_self, spec_cache, spec_dec, fast_spec_dec


def attention_cases(kref):
    """(name, q, k, v) seeded N(0,1); shapes cover decode, verify, ragged-length and draft geometry."""
    specs = [
        ("decode_12x2_d128_t128", 1, 12, 2, 1, 128, 128, torch.bfloat16),
        ("verify_12x2_d128_s5_t77", 1, 12, 2, 5, 77, 128, torch.bfloat16),
        ("verify_12x2_d128_s5_t16", 1, 12, 2, 5, 16, 128, torch.bfloat16),
        ("decode_12x2_d128_b2_t33", 2, 12, 2, 1, 33, 128, torch.bfloat16),
        ("verify_14x2_d64_s5_t50", 1, 14, 2, 5, 50, 64, torch.bfloat16),
        ("decode_14x2_d64_t1", 1, 14, 2, 1, 1, 64, torch.bfloat16),
        ("prefill_12x2_d128_s40_t40", 1, 12, 2, 40, 40, 128, torch.bfloat16),
        ("fp32_4x2_d64_s64_t64", 1, 4, 2, 64, 64, 64, torch.float32),
    ]
    out = {}
    for i, (name, B, H, KV, S, T, D, dt) in enumerate(specs):
        g = torch.Generator().manual_seed(1000 + i)
        q = torch.randn(B, H, S, D, generator=g).to(dt)
        k = torch.randn(B, KV, T, D, generator=g).to(dt)
        v = torch.randn(B, KV, T, D, generator=g).to(dt)
        out[name] = dict(q=q, k=k, v=v, eager=kref.attention(q, k, v), fp32=kref.attention_fp32(q, k, v))
    return out


def fp8_cases(model_self):
    g = torch.Generator().manual_seed(7)
    v = torch.randn(1, 2, 48, 128, generator=g)
    hit = torch.rand(v.shape, generator=g) < 0.01
    sign = torch.where(torch.rand(v.shape, generator=g) < 0.5, -1.0, 1.0)
    v = torch.where(hit, 8.0 * sign, v).to(torch.bfloat16)
    # edge rows: all zero, one 448-sized element, negative zeros, tiny values, a single max
    edge = torch.zeros(1, 2, 6, 128)
    edge[0, 0, 1, 3] = 448.0
    edge[0, 0, 2] = -0.0
    edge[0, 0, 3] = torch.linspace(-1e-6, 1e-6, 128)
    edge[0, 1, 0] = torch.linspace(-3.0, 5.0, 128)
    edge[0, 1, 1, 0] = -2.5
    edge[0, 1, 2] = 1e-30
    edge[0, 1, 3] = torch.arange(128) * 0.37 - 20.0
    edge[0, 1, 4] = 65504.0 * torch.sign(torch.arange(128) - 63.5)
    edge[0, 1, 5] = torch.randn(128, generator=g) * 1e-3
    edge = edge.to(torch.bfloat16)
    # a NaN in a V row: the reference's amax propagates it, so that row's scale and every
    # code of the row are NaN
    nan_rows = torch.randn(1, 2, 3, 128, generator=g)
    nan_rows[0, 1, 1, 17] = float("nan")
    nan_rows = nan_rows.to(torch.bfloat16)
    res = {}
    for name, x in (("outlier", v), ("edge", edge), ("nan_row", nan_rows)):
        qv, sv = model_self.quantize_kv_fp8(x, model_self.GROUP_V)
        deq = model_self.dequantize_kv_fp8(qv, sv, torch.bfloat16)
        res[name] = dict(x=x, codes=qv.view(torch.uint8).clone(), scale=sv.clone(), deq=deq)
    return res


def spec_cache_cases(spec_cache):
    def mk(n):
        return [{"k": torch.zeros(1, 2, n, 4), "v": torch.zeros(1, 2, n, 4), "fmt": "fp16"} for _ in range(2)]

    rec = []
    for cur, req in [(8, 3), (8, 8), (8, 1), (8, 0), (8, -1), (8, 9), (8, True), (8, 2.0), (None, 0), (None, 1)]:
        cache = mk(cur) if cur is not None else None
        try:
            t = spec_cache.trim_cache(cache, req)
            rec.append(dict(cur=cur, req=req, ok=True, new_len=spec_cache.cache_length(t),
                            orig_len=spec_cache.cache_length(cache), fmt_kept=(t is None or t[0]["fmt"] == "fp16")))
        except ValueError:
            rec.append(dict(cur=cur, req=req, ok=False))
    cons = []
    for shape_v, layer2 in [((1, 2, 8, 4), 8), ((1, 2, 7, 4), 8), ((1, 2, 8, 4), 6)]:
        c = [{"k": torch.zeros(1, 2, 8, 4), "v": torch.zeros(*shape_v)},
             {"k": torch.zeros(1, 2, layer2, 4), "v": torch.zeros(1, 2, layer2, 4)}]
        try:
            spec_cache.check_consistent(c)
            cons.append(True)
        except RuntimeError:
            cons.append(False)
    return dict(trim=rec, consistent=cons)


def accept_cases():
    """Rows + candidates -> (g, m) by the vectorised accept expressions of fast_spec_dec.py:246-249."""
    g = torch.Generator().manual_seed(11)
    cases = []
    V = 1000
    for i in range(24):
        kp = 1 + i % 4
        saved = torch.randn(1, V, generator=g).to(torch.bfloat16)
        rows = torch.randn(kp, V, generator=g).to(torch.bfloat16)
        stack = torch.cat([saved.reshape(1, -1), rows[: kp - 1]], dim=0)
        truth = stack.float().argmax(-1)
        m_plant = i % (kp + 1)
        cands = torch.randint(0, V, (kp,), generator=g)
        cands[:m_plant] = truth[:m_plant]
        if m_plant < kp and cands[m_plant] == truth[m_plant]:
            cands[m_plant] = (truth[m_plant] + 1) % V
        if i % 6 == 5:  # exact ties: the first index must win
            stack[0, 10] = stack[0].max()
            stack[0, 900] = stack[0, 10]
        if i % 8 == 7:  # NaN counts as the maximum in torch.argmax
            stack[min(1, kp - 1), 500] = float("nan")
        g_t = stack.argmax(dim=-1)
        eq = g_t == cands
        m_t = eq.to(torch.int64).cumprod(0).sum()
        cases.append(dict(stack=stack.clone(), cands=cands.clone(), g=g_t.clone(), m=int(m_t)))
    return cases


class ToyLM(torch.nn.Module):
    """Deterministic toy causal LM with the reference engine's dict-cache interface.

    logits(token t at position p) = (E[t] + P[p]) @ W^T; the cache stores one
    scalar per position so trims and cache lengths are observable."""

    def __init__(self, vocab, hidden, seed, like=None, noise=0.0, max_pos=96):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.E = torch.nn.functional.normalize(torch.randn(vocab, hidden, generator=g), dim=1)
        self.P = 0.5 * torch.randn(max_pos, hidden, generator=g)
        base = torch.randn(vocab, hidden, generator=g) / hidden ** 0.5
        if like is not None:
            base = like.W + noise * torch.randn(vocab, hidden, generator=g) / hidden ** 0.5
            self.E, self.P = like.E, like.P
        self.W = base
        self.kv_format = "fp16"
        self.head_dim = hidden

    def set_kv_format(self, fmt):
        self.kv_format = fmt

    def embed_tokens(self, ids):
        return torch.nn.functional.embedding(ids, self.E)

    def _run(self, x, cache=None, need_logits=True):
        b, s, _ = x.shape
        t0 = cache[0]["k"].shape[2] if cache else 0
        h = x + self.P[t0:t0 + s].unsqueeze(0)
        logits = h @ self.W.T
        kn = x[:, :, :1].transpose(1, 2).unsqueeze(-1)
        if cache is None:
            cache = [{"k": kn, "v": kn.clone()}]
        else:
            cache[0]["k"] = torch.cat([cache[0]["k"], kn], dim=2)
            cache[0]["v"] = torch.cat([cache[0]["v"], kn.clone()], dim=2)
        return (logits if need_logits else None), cache


def elementwise_cases(kref):
    """reference.rmsnorm / apply_rope / swiglu (specdec/kernels/reference.py:14-31) at bf16 and
    fp32, on the engine's shapes: hidden 1536 and 896 rows, (B, H, S, 128) and (B, H, S, 64)
    rotary inputs with the engine's cos / sin tables, and the FFN widths 8960 and 4864."""
    out = {}
    for dt_name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        g = torch.Generator().manual_seed(300 if dt is torch.bfloat16 else 301)
        for hidden in (1536, 896, 1000):
            x = (torch.randn(13, hidden, generator=g) * 3.0).to(dt)
            w = torch.randn(hidden, generator=g).to(dt)
            out[f"rmsnorm_{dt_name}_{hidden}"] = dict(x=x, w=w, out=kref.rmsnorm(x, w))
        for H, S, D in ((12, 5, 128), (14, 2, 64), (2, 9, 128)):
            x = torch.randn(1, H, S, D, generator=g).to(dt)
            pos = torch.arange(8190, 8190 + S, dtype=torch.float32)
            inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
            ang = torch.outer(pos, inv)
            cos = torch.cat([ang.cos(), ang.cos()], -1)[None, None].to(dt)
            sin = torch.cat([ang.sin(), ang.sin()], -1)[None, None].to(dt)
            out[f"rope_{dt_name}_{H}x{S}x{D}"] = dict(x=x, cos=cos, sin=sin, out=kref.apply_rope(x, cos, sin))
        for inter in (8960, 4864):
            gate = (torch.randn(3, inter, generator=g) * 2.0).to(dt)
            up = torch.randn(3, inter, generator=g).to(dt)
            out[f"swiglu_{dt_name}_{inter}"] = dict(gate=gate, up=up, out=kref.swiglu(gate, up))
    return out


def model_cases(model_self):
    """A tiny random-init reference QwenLM (model_self.py:835-931) in bf16 on the CPU: the
    target geometry's heads (12 query : 2 KV heads, head_dim 128) at width 128, 2 layers,
    Qwen2 q/k/v biases.  For the bf16 ("fp16") and V-only FP8 ("v_fp8") cache formats: the
    prompt pass's last-row logits, the logits of a 5-token verify block on top of the prompt,
    and 6 greedy tokens decoded one at a time from the prompt (QwenLM._run with dict caches),
    with the weights as a state dict."""
    torch.manual_seed(123)
    m = model_self.QwenLM(vocab_size=512, hidden=128, heads=12, kv_heads=2, head_dim=128, intermediate=256,
                          num_layers=2, rope_theta=1_000_000.0, rms_eps=1e-6, attn_bias=True)
    # the constructor's own seeded init, rescaled so that greedy decoding does not just repeat
    # the last token (tied embeddings at N(0,1) dominate the residual stream), and norm
    # weights that are not all ones
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name:
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            elif "embed" in name:
                p.mul_(0.05)
            else:
                p.mul_(3.0)
    m = m.to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(124)
    prompt = torch.randint(0, 512, (1, 37), generator=g)
    block = torch.randint(0, 512, (1, 5), generator=g)
    res = dict(config=dict(vocab=512, hidden=128, heads=12, kv_heads=2, head_dim=128, intermediate=256, layers=2,
                           rope_theta=1_000_000.0, eps=1e-6, attn_bias=True),
               state={k: v.clone() for k, v in m.state_dict().items()}, prompt=prompt, block=block)
    with torch.no_grad():
        for fmt in ("fp16", "v_fp8"):
            m.set_kv_format(fmt)
            lg, cache = m._run(m.embed_tokens(prompt), None)
            prompt_logits = lg[0, -1].clone()
            vb, _ = m._run(m.embed_tokens(block), cache)
            # greedy decode from a fresh prompt pass
            lg, cache = m._run(m.embed_tokens(prompt), None)
            toks, step_logits = [], []
            for _ in range(6):
                t = int(lg[0, -1].argmax())
                toks.append(t)
                step_logits.append(lg[0, -1].clone())
                lg, cache = m._run(m.embed_tokens(torch.tensor([[t]])), cache)
            res[fmt] = dict(prompt_logits=prompt_logits, verify_logits=vb[0].clone(), greedy=toks,
                            greedy_logits=torch.stack(step_logits))
    return res


def executor_traces(spec_dec, fast_spec_dec):
    traces = []
    for seed, noise, max_new in [(1, 0.0, 13), (2, 0.3, 16), (3, 1.5, 12), (4, 0.8, 17)]:
        vocab, hidden = 40, 12
        tgt = ToyLM(vocab, hidden, seed)
        drf = ToyLM(vocab, hidden, seed + 50, like=tgt, noise=noise)
        prompt = torch.randint(0, vocab, (1, 5), generator=torch.Generator().manual_seed(seed + 99))
        log = []
        strict = spec_dec.spec_decode_greedy(tgt, drf, prompt, max_new, k=4, log=log.append)
        fast = fast_spec_dec.spec_decode_greedy_optimized(tgt, drf, prompt, max_new, k=4)
        traces.append(dict(seed=seed, noise=noise, max_new=max_new, vocab=vocab, hidden=hidden,
                           prompt=prompt.clone(), gen=list(strict["gen"]), fast_gen=list(fast["gen"]),
                           stats=dict(strict["stats"]),
                           control=[{k: v for k, v in row.items()} for row in log]))
    return traces


def main():
    kref, model_self, spec_cache, spec_dec, fast_spec_dec = _import_reference()
    torch.manual_seed(0)
    data = dict(
        version=1,
        torch=torch.__version__,
        attention=attention_cases(kref),
        fp8=fp8_cases(model_self),
        spec_cache=spec_cache_cases(spec_cache),
        accept=accept_cases(),
        traces=executor_traces(spec_dec, fast_spec_dec),
        elementwise=elementwise_cases(kref),
        model=model_cases(model_self),
    )
    path = HERE / "golden_v1.pt"
    torch.save(data, path)
    print(f"wrote {path} ({path.stat().st_size / 1024:.1f} KiB)")


if __name__ == "__main__":
    main()
