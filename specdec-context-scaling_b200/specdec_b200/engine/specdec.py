"""Batched greedy speculative decoding with device-resident state.

Algorithm (greedy SpecDec, spec_dec.py:206-250, in its block-verify form with the
pending token leading the verify block, bonus_accept_oracle.py:119-160): every
sequence carries a *pending* token -- the last emitted token, not yet in either
cache.  One round:

  1. the draft reads the pending token (and, after a round that accepted all k
     candidates, first the k-th candidate it never read) and proposes
     c1 .. ck greedily, one q_len-1 step per candidate;
  2. the target verifies [pending, c1 .. ck] in one q_len = k+1 step;
  3. greedy accept on the device: g_j = argmax(row j), m = length of the common
     prefix of (g_0 .. g_{k-1}) and (c1 .. ck); emitted tokens c1 .. cm, g_m;
     g_m becomes the new pending token;
The draft's proposals and the target's g_j come straight from the hidden states through
the fused LM-head argmax (the logits are never written).
  4. rollback on the device: the target keeps pending + c1 .. cm
     (len + 1 + m), the draft the same minus ck when m == k.

A sequence that has emitted max_new tokens is frozen on the device at the start of
the next round: its query lengths are 0 in every step of the round (no append, no
attention rows), accept treats it as inactive (m = 0, lengths kept), and nothing is
emitted for it, so its caches stop growing while slower sequences finish.

Every step of a round is a fixed-shape device computation (the ragged q_len of
step 1 lives in device arrays), so a round is captured once in a CUDA graph and
replayed with no host synchronisation; the host only checks the emitted-token
counts every few rounds.  Emitted tokens equal target-only greedy decoding,
except where bf16 rounding flips a near-tie of the target's logits.
"""

from __future__ import annotations

import torch

from ..kernels import ops
from .model import PagedModel, StepLayout


class SpecDecEngine:
    def __init__(self, target: PagedModel, draft: PagedModel, num_seqs: int, prompt_len: int, max_new: int, *,
                 k: int = 4, target_v: str = "bf16", draft_v: str = "bf16", check_every: int = 4):
        if k < 1:
            raise ValueError("k must be >= 1")
        if target.cfg.vocab != draft.cfg.vocab:
            raise ValueError("target and draft must share the vocabulary")
        self.target, self.draft = target, draft
        self.B, self.k, self.P, self.max_new = num_seqs, k, prompt_len, max_new
        self.check_every = check_every
        dev = target.device
        self.device = dev
        # a sequence is frozen once it has max_new tokens, so its caches hold at most the
        # prompt, max_new + k emitted tokens and one verify block
        cap = prompt_len + max_new + 2 * (k + 1) + 2
        self.tc = target.new_cache(num_seqs, cap, target_v)
        self.dc = draft.new_cache(num_seqs, cap, draft_v)
        self.L0 = StepLayout(num_seqs, 2, dev)
        self.L1 = StepLayout(num_seqs, 1, dev)
        self.LV = StepLayout(num_seqs, k + 1, dev)
        self.ws0 = ops.attn_workspace(self.L0.batch, draft.cfg.heads, self.dc)
        self.ws1 = ops.attn_workspace(self.L1.batch, draft.cfg.heads, self.dc)
        self.wsv = ops.attn_workspace(self.LV.batch, target.cfg.heads, self.tc)
        i32 = dict(dtype=torch.int32, device=dev)
        self.pending = torch.zeros(num_seqs, **i32)
        self.catch = torch.zeros(num_seqs, **i32)     # 1: the draft has not read the last round's ck
        self.c_last = torch.zeros(num_seqs, **i32)
        self.cands = torch.zeros(num_seqs, k, **i32)
        self.kp = torch.full((num_seqs,), k, **i32)
        self.width = max_new + k + 1
        self.out = torch.zeros(num_seqs, self.width, **i32)
        self.n_out = torch.zeros(num_seqs, **i32)
        self.g = torch.zeros(num_seqs, k + 1, **i32)
        self.m = torch.zeros(num_seqs, **i32)
        self.next_token = torch.zeros(num_seqs, **i32)
        self.new_tlen = torch.zeros(num_seqs, **i32)
        self.new_dlen = torch.zeros(num_seqs, **i32)
        self.accepted = torch.zeros(num_seqs, dtype=torch.int64, device=dev)
        self.active_rounds = torch.zeros(num_seqs, dtype=torch.int64, device=dev)
        self.rounds = 0
        self.status = torch.zeros(1, **i32)
        self.acc_ws = ops.accept_workspace(num_seqs, k + 1, target.cfg.vocab, dev)
        self.dtok = torch.zeros(num_seqs, **i32)  # the draft's greedy tokens of one step
        self.lm_ws_d = ops.lmhead_workspace(num_seqs, dev)
        self.lm_ws_t = ops.lmhead_workspace(num_seqs * (k + 1), dev)
        self.graph = None
        self.idx = torch.arange(k + 1, device=dev, dtype=torch.int32)
        self.active = torch.ones(num_seqs, **i32)   # 0: the sequence has its max_new tokens

    # ------------------------------------------------------------------ prompt
    @torch.inference_mode()
    def prefill(self, prompts: torch.Tensor, chunk: int = 4) -> None:
        """Prompt pass of both models; the target's first prediction is emitted and pending.
        Every per-sequence length, counter and status starts over."""
        if tuple(prompts.shape) != (self.B, self.P):
            raise ValueError(f"prompts must be ({self.B}, {self.P})")
        self.status.zero_()
        for s0 in range(0, self.B, chunk):
            ids = prompts[s0:s0 + chunk]
            lg = self.target.prefill(ids, self.tc, s0, status=self.status)
            self.pending[s0:s0 + ids.shape[0]] = lg.argmax(-1).int()
            self.draft.prefill(ids, self.dc, s0, need_logits=False, status=self.status)
        self.out.zero_()
        self.out[:, 0] = self.pending
        self.n_out.fill_(1)
        self.active.fill_(1)
        self.catch.zero_()
        self.accepted.zero_()
        self.active_rounds.zero_()
        self.rounds = 0

    # ------------------------------------------------------------------ one round
    def _round(self) -> None:
        k = self.k
        draft, target = self.draft, self.target
        act = self.active
        act.copy_(self.n_out < self.max_new)  # frozen sequences: every q_len 0 below
        # 1. draft: [ck_prev, pending] after a full accept, else [pending]
        q0 = (1 + self.catch) * act
        first = torch.where(self.catch > 0, self.c_last, self.pending)
        tok0 = torch.stack([first, self.pending], dim=1).reshape(-1)
        self.L0.set(self.dc.lengths, q0)
        h = draft.step(tok0, self.L0, self.dc, self.ws0, status=self.status)
        self.cands[:, 0] = draft.greedy(h[self.L0.last_rows()], self.dtok, self.lm_ws_d)
        self.dc.lengths.add_(q0)
        for i in range(1, k):
            self.L1.set(self.dc.lengths, act)
            h = draft.step(self.cands[:, i - 1], self.L1, self.dc, self.ws1, status=self.status)
            self.cands[:, i] = draft.greedy(h, self.dtok, self.lm_ws_d)
            self.dc.lengths.add_(act)
        # 2. target verify of [pending, c1 .. ck]; g_j of every verify row (rows b (k+1) + j)
        vt = torch.cat([self.pending.unsqueeze(1), self.cands], dim=1).reshape(-1)
        self.LV.set(self.tc.lengths, act * (k + 1))
        h = target.step(vt, self.LV, self.tc, self.wsv, status=self.status)
        target.greedy(h, self.g.view(-1), self.lm_ws_t)
        # 3. greedy accept from g (+ the target's rolled-back length len + 1 + m)
        ops.greedy_accept(None, row0=self.LV.q_row0, n_rows=self.LV.q_len, cands=self.cands, kp=self.kp,
                          max_rows=k + 1, g=self.g, m=self.m, next_token=self.next_token,
                          len_before=self.tc.lengths, len_after=self.new_tlen, keep_offset=1,
                          status=self.status)
        # emitted: c1 .. cm then g_m, at out[b, n_out[b] ..]
        m = self.m.unsqueeze(1)
        vals = torch.where(self.idx[:k].unsqueeze(0) < m, self.cands, self.next_token.unsqueeze(1))
        vals = torch.cat([vals, self.next_token.unsqueeze(1)], dim=1)
        pos = (self.n_out.unsqueeze(1) + self.idx.unsqueeze(0)).clamp(max=self.width - 1).long()
        keep = (self.idx.unsqueeze(0) <= m) & (act.unsqueeze(1) > 0)
        self.out.scatter_(1, pos, torch.where(keep, vals, self.out.gather(1, pos)))
        self.n_out.add_((self.m + 1) * act)
        self.accepted.add_(self.m)  # 0 for frozen sequences
        self.active_rounds.add_(act)
        # 4. rollback on the device (accept keeps a frozen sequence's target length)
        self.tc.lengths.copy_(self.new_tlen)
        full = (self.m == k).int() * act
        torch.where(act > 0, self.new_tlen - full, self.dc.lengths, out=self.new_dlen)
        ops.trim_lengths(self.dc.lengths, self.new_dlen, out=self.dc.lengths, status=self.status)
        torch.where(act > 0, full, self.catch, out=self.catch)
        torch.where(act > 0, self.cands[:, k - 1], self.c_last, out=self.c_last)
        torch.where(act > 0, self.next_token, self.pending, out=self.pending)

    @torch.inference_mode()
    def capture(self) -> None:
        """Record one round as a CUDA graph (after one eager warm-up round).  Capturing
        before ``prefill`` keeps it out of the decode: prefill resets every length and
        counter the warm-up touched."""
        self._round()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._round()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = g

    @torch.inference_mode()
    def decode(self, use_graph: bool = True) -> int:
        """Rounds until every sequence has emitted max_new tokens; returns the rounds run."""
        if use_graph and self.graph is None:
            raise RuntimeError("call capture() before prefill() to decode with the round graph")
        while True:
            for _ in range(self.check_every):
                if use_graph:
                    self.graph.replay()
                else:
                    self._round()
                self.rounds += 1
            if int(self.n_out.min()) >= self.max_new:
                break
            if self.rounds > self.max_new + self.check_every:
                raise RuntimeError("decode made no progress")
        st = int(self.status.item())
        if st:
            from .. import _lib

            raise RuntimeError(f"device status {st:#x}: {_lib.status_message(st)}")
        return self.rounds

    def tokens(self) -> torch.Tensor:
        """(num_seqs, max_new) emitted tokens (the first is the prompt pass's prediction)."""
        return self.out[:, :self.max_new]

    def acceptance(self) -> float:
        """Mean accepted candidates per round and sequence, over the rounds each sequence
        was active in (not frozen)."""
        return float(self.accepted.sum()) / max(1, int(self.active_rounds.sum()))
