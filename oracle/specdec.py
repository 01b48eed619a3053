"""Greedy speculative-decoding oracle (test infrastructure only): a restatement of the
reference's strict executor, spec_decode_greedy (specdec/engine/spec_dec.py:189-275),
over any model with the reference engine's interface (``embed_tokens``, ``_run(x, cache,
need_logits)`` with per-layer dict caches, ``set_kv_format``), such as oracle.engine.QwenLM.

One round (spec_dec.py:204-265):
  * the draft proposes k_eff = min(k, max_new - emitted) candidates greedily, one
    single-token step each (_propose, :150-161);
  * the target runs the candidate block on its cache and keeps the block's logits rows
    (_verify, :164-181);
  * g = argmax of [saved_next] + rows[:kp - 1]; m = length of the common prefix of g and
    the candidates (:233-236);
  * m < kp: emit cands[:m] + [g[m]], trim both caches to pre + m, then one repair step of
    g[m] on each model (:238-246); m == kp: emit the candidates, keep the block cache,
    trim the draft to pre + kp and carry the last block row as saved_next (:247-253).
The caches are trimmed with oracle.spec_cache.trim_cache (spec_cache.py:10-28).

Used by tests/ (pinned against the reference executor's control traces in
tests/golden) and by bench.py's CPU baseline of SpecDec decode tokens/s.
"""

from __future__ import annotations

import torch

from . import spec_cache as osc

FMT = {"base_bf16": "fp16", "v_fp8": "v_fp8"}


def _run_tokens(model, tokens, cache):
    dev = model.embed_tokens.weight.device if hasattr(model.embed_tokens, "weight") else "cpu"
    ids = torch.tensor([tokens], device=dev)
    return model._run(model.embed_tokens(ids), cache, need_logits=True)


@torch.inference_mode()
def spec_decode_greedy(target, draft, prompt_ids, max_new_tokens: int, *, k: int = 4, eos_id=None,
                       target_kv: str = "base_bf16", draft_kv: str = "base_bf16", log=None):
    target.set_kv_format(FMT[target_kv])
    draft.set_kv_format(FMT[draft_kv])
    tgt_lg, tgt_cache = target._run(target.embed_tokens(prompt_ids), None, need_logits=True)
    drf_lg, drf_cache = draft._run(draft.embed_tokens(prompt_ids), None, need_logits=True)
    saved_next = tgt_lg[:, -1:]
    drf_lg = drf_lg[:, -1:]
    gen = []
    st = dict(rounds=0, proposed=0, accepted=0)
    while len(gen) < max_new_tokens:
        k_eff = min(k, max_new_tokens - len(gen))
        pre = osc.cache_length(tgt_cache)
        # propose
        cands, lg = [], drf_lg
        for _ in range(k_eff):
            t = int(lg.reshape(-1, lg.shape[-1])[-1].argmax())
            cands.append(t)
            lg, drf_cache = _run_tokens(draft, [t], drf_cache)
            if t == eos_id:
                break
        prop_lg = lg
        kp = len(cands)
        if kp == 0:
            break
        # verify the block
        blk_lg, tgt_blk = _run_tokens(target, cands, tgt_cache)
        rows = blk_lg[0, -kp:]
        g = [int(x.argmax()) for x in [saved_next] + [rows[j] for j in range(kp - 1)]]
        m = 0
        while m < kp and g[m] == cands[m]:
            m += 1
        if m < kp:
            r = g[m]
            emitted = cands[:m] + [r]
            tgt_cache = osc.trim_cache(tgt_blk, pre + m)
            lg, tgt_cache = _run_tokens(target, [r], tgt_cache)
            saved_next = lg[:, -1:]
            drf_cache = osc.trim_cache(drf_cache, pre + m)
            lg, drf_cache = _run_tokens(draft, [r], drf_cache)
            drf_lg = lg[:, -1:]
        else:
            emitted = list(cands)
            tgt_cache = tgt_blk
            drf_cache = osc.trim_cache(drf_cache, pre + kp)
            saved_next = rows[kp - 1]
            drf_lg = prop_lg
        gen += emitted
        st["rounds"] += 1
        st["proposed"] += kp
        st["accepted"] += m
        if log is not None:
            log(dict(round=st["rounds"] - 1, Kp=kp, m=m, pre=pre, tgt_len=osc.cache_length(tgt_cache),
                     drf_len=osc.cache_length(drf_cache), cands=cands, g=g, emitted=emitted))
        if emitted and emitted[-1] == eos_id:
            break
    return {"gen": gen, "stats": st}
