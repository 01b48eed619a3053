"""Attention oracle (test infrastructure): CPU restatement of the reference formulas.

``eager_attention`` follows reference.attention (specdec/kernels/reference.py:47-56),
which is the eager decode/verify branch of SelfAttention.forward
(specdec/engine/model_self.py:740-775):
    scores = dtype(q @ k_rep^T) / sqrt(D)       (rounded in the input dtype)
    scores[j > i + (T - S)] = -inf              (reference.py:40-44)
    attn = dtype(softmax_fp32(scores))
    out = dtype(attn @ v_rep)
``attention_fp32`` follows reference.attention_fp32 (reference.py:59-70): the same
mask with fp32 products, the algorithm reference of the CUDA kernels.
"""

from __future__ import annotations

import torch


def kv_repeat(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """GQA expansion (model_self.py:294-298): KV head k serves query heads k*n_rep .. k*n_rep+n_rep-1."""
    if n_rep == 1:
        return x
    return torch.repeat_interleave(x, n_rep, dim=1)


def offset_causal_mask(s: int, t: int) -> torch.Tensor:
    """True where key j is hidden from query row i: j > i + (t - s)."""
    i = torch.arange(s).view(s, 1)
    j = torch.arange(t).view(1, t)
    return j > i + (t - s)


def eager_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    q, k, v = q.cpu(), k.cpu(), v.cpu()
    n_rep = q.shape[1] // k.shape[1]
    kr, vr = kv_repeat(k, n_rep), kv_repeat(v, n_rep)
    scores = torch.matmul(q, kr.transpose(-2, -1)) / (q.shape[-1] ** 0.5)
    s, t = q.shape[-2], k.shape[-2]
    scores = scores.masked_fill(offset_causal_mask(s, t), float("-inf"))
    attn = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(attn, vr)


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    q, k, v = q.cpu(), k.cpu(), v.cpu()
    n_rep = q.shape[1] // k.shape[1]
    kr, vr = kv_repeat(k, n_rep).float(), kv_repeat(v, n_rep).float()
    scores = torch.matmul(q.float(), kr.transpose(-2, -1)) * (q.shape[-1] ** -0.5)
    s, t = q.shape[-2], k.shape[-2]
    scores = scores.masked_fill(offset_causal_mask(s, t), float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), vr).to(q.dtype)


def ragged_attention(q_rows, k_seqs, v_seqs, q_lens, fp32: bool = True):
    """Packed-row attention of a ragged batch: q_rows (sum q_len, H, D); k/v_seqs lists of (KV, T_b, D).

    Returns (sum q_len, H, D) in q's dtype; sequence b's rows are q_rows[off_b : off_b + q_len[b]]."""
    fn = attention_fp32 if fp32 else eager_attention
    outs, off = [], 0
    for b, n in enumerate(q_lens):
        if n == 0:
            continue
        q = q_rows[off:off + n].permute(1, 0, 2).unsqueeze(0)  # (1, H, n, D)
        o = fn(q, k_seqs[b].unsqueeze(0), v_seqs[b].unsqueeze(0))
        outs.append(o[0].permute(1, 0, 2))
        off += n
    return torch.cat(outs, dim=0)


def within_tolerance(got: torch.Tensor, ref: torch.Tensor, rtol: float = 2e-2, atol: float = 1e-2):
    """The north-star bar for bf16 attention: |got - ref| <= atol + rtol * |ref| elementwise.

    Returns (ok, max_abs_err, worst_excess)."""
    g, r = got.float().cpu(), ref.float().cpu()
    err = (g - r).abs()
    bound = atol + rtol * r.abs()
    excess = (err - bound).max().item()
    return bool(excess <= 0.0 and torch.isfinite(g).all()), err.max().item(), excess
