"""Model-level oracle (test infrastructure only): a torch restatement of the reference
engine's decoder (specdec/engine/model_self.py), used

* as the module ``specdec_b200.kernels.patch`` patches in tests (same class surface:
  RMSNORM, MLP, SelfAttention, DecoderLayer, QwenLM, module-level apply_rope /
  quantize_kv_fp8 / dequantize_kv_fp8), and
* as the greedy-decoding reference of the end-to-end SpecDec tests: plain target-only
  greedy decoding with the engine's eager attention (bf16 scores, fp32 softmax, bf16
  probabilities) and per-layer dict caches grown with torch.cat.

Cited behaviour:
  RMSNORM                  model_self.py:225-235 (fp32 mean of squares, cast back, weight multiply)
  MLP                      model_self.py:246-270 (down(silu(gate(x)) * up(x)))
  Build_Rope_cache         model_self.py:272-284 (fp32 angles, cat(cos, cos), cast to x dtype)
  rotate_half / apply_rope model_self.py:286-292
  kv_repeat                model_self.py:294-298
  quantize / dequantize    model_self.py:300-320 (E4M3_MAX 448, GROUP_SIZE 32, GROUP_V 128)
  SelfAttention.forward    model_self.py:668-800 (fp16 / fp8 / v_fp8 dict caches; eager branch)
  QwenLM._run              model_self.py:845-860 (start_pos from layer 0's cache; tied logits)

It is never imported by the product path (specdec_b200/), only by tests/,
__graft_entry__.smoke() and bench.py's CPU baseline.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

E4M3_MAX = 448.0
GROUP_SIZE = 32
GROUP_V = 128


def quantize_kv_fp8(x: torch.Tensor, group_size: int = GROUP_SIZE):
    d = x.shape[-1]
    g = d // group_size
    xg = x.float().view(*x.shape[:-1], g, group_size)
    s = xg.abs().amax(dim=-1, keepdim=True) / E4M3_MAX
    s = torch.where(s == 0, torch.ones_like(s), s)
    q = (xg / s).to(torch.float8_e4m3fn).reshape_as(x)
    return q, s.squeeze(-1)


def dequantize_kv_fp8(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.float16):
    g = scale.shape[-1]
    qg = q.float().view(*q.shape[:-1], g, q.shape[-1] // g)
    return (qg * scale.unsqueeze(-1)).reshape_as(q).to(dtype)


def rope_cache(head_dim: int, seq_len: int, theta: float, device, dtype, start_pos: int = 0):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    pos = torch.arange(start_pos, start_pos + seq_len, device=device, dtype=torch.float32)
    ang = torch.outer(pos, inv)
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)[None, None]
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)[None, None]
    return cos.to(dtype), sin.to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x, cos, sin):
    return x * cos + rotate_half(x) * sin


def kv_repeat(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    b, kv, s, d = x.shape
    return x.unsqueeze(2).expand(b, kv, n_rep, s, d).reshape(b, kv * n_rep, s, d)


class RMSNORM(nn.Module):
    def __init__(self, hidden: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden))
        self.eps = eps

    def forward(self, x):
        x32 = x.float()
        normed = x32 * torch.rsqrt((x32 * x32).mean(dim=-1, keepdim=True) + self.eps)
        return self.weight * normed.to(x.dtype)


class MLP(nn.Module):
    def __init__(self, hidden: int, intermediate: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden, intermediate, bias=False)
        self.up_proj = nn.Linear(hidden, intermediate, bias=False)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class SelfAttention(nn.Module):
    def __init__(self, hidden: int, heads: int, kv_heads: int, head_dim: int, attn_bias: bool = False):
        super().__init__()
        self.q_proj = nn.Linear(hidden, heads * head_dim, bias=attn_bias)
        self.k_proj = nn.Linear(hidden, kv_heads * head_dim, bias=attn_bias)
        self.v_proj = nn.Linear(hidden, kv_heads * head_dim, bias=attn_bias)
        self.o_proj = nn.Linear(heads * head_dim, hidden, bias=False)
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.kv_format = "fp16"
        self.fp8_g_k = self.fp8_g_v = GROUP_SIZE
        self.fp8_k = self.fp8_v = True

    def forward(self, x, cos, sin, cache=None):
        b, s, _ = x.shape
        q = self.q_proj(x).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(b, s, self.kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, s, self.kv_heads, self.head_dim).transpose(1, 2)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        fmt = cache.get("fmt", self.kv_format) if cache is not None else self.kv_format
        if fmt == "v_fp8":
            k_on, v_on, gk, gv = False, True, GROUP_SIZE, GROUP_V
        elif fmt == "fp8":
            k_on, v_on, gk, gv = self.fp8_k, self.fp8_v, self.fp8_g_k, self.fp8_g_v
        else:
            k_on = v_on = False
            gk = gv = GROUP_SIZE
        kq = vq = None
        k_cur, v_cur = k, v
        if k_on:
            kq = quantize_kv_fp8(k, gk)
            k_cur = dequantize_kv_fp8(kq[0], kq[1], x.dtype)
        if v_on:
            vq = quantize_kv_fp8(v, gv)
            v_cur = dequantize_kv_fp8(vq[0], vq[1], x.dtype)
        if cache is None:
            k_all, v_all = k_cur, v_cur
        elif fmt == "fp16":
            k_all = cache["k"] = torch.cat([cache["k"], k], dim=2)
            v_all = cache["v"] = torch.cat([cache["v"], v], dim=2)
        else:
            if "k_scale" in cache:
                k_all = torch.cat([dequantize_kv_fp8(cache["k"], cache["k_scale"], x.dtype), k_cur], dim=2)
            else:
                k_all = cache["k"] = torch.cat([cache["k"], k_cur], dim=2)
            if "v_scale" in cache:
                v_all = torch.cat([dequantize_kv_fp8(cache["v"], cache["v_scale"], x.dtype), v_cur], dim=2)
            else:
                v_all = cache["v"] = torch.cat([cache["v"], v_cur], dim=2)
        T = k_all.shape[2] if cache is not None else s
        n_rep = self.heads // self.kv_heads
        scores = torch.matmul(q, kv_repeat(k_all, n_rep).transpose(-2, -1)) / (self.head_dim ** 0.5)
        if cache is None:
            scores = scores.masked_fill(torch.ones(s, T, dtype=torch.bool, device=x.device).triu(1), float("-inf"))
        elif s > 1:
            mask = torch.ones(s, T, dtype=torch.bool, device=x.device).triu(T - s + 1)
            scores = scores.masked_fill(mask, float("-inf"))
        attn = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
        out = torch.matmul(attn, kv_repeat(v_all, n_rep)).to(q.dtype)
        out = out.transpose(1, 2).contiguous().view(b, s, self.heads * self.head_dim)
        if cache is None:
            if fmt in ("fp8", "v_fp8"):
                new_cache = {"fmt": fmt}
                new_cache.update({"k": kq[0], "k_scale": kq[1]} if k_on else {"k": k_all})
                new_cache.update({"v": vq[0], "v_scale": vq[1]} if v_on else {"v": v_all})
            else:
                new_cache = {"k": k_all, "v": v_all}
        else:
            if fmt in ("fp8", "v_fp8"):
                if k_on:
                    cache["k"] = torch.cat([cache["k"], kq[0]], dim=2)
                    cache["k_scale"] = torch.cat([cache["k_scale"], kq[1]], dim=2)
                if v_on:
                    cache["v"] = torch.cat([cache["v"], vq[0]], dim=2)
                    cache["v_scale"] = torch.cat([cache["v_scale"], vq[1]], dim=2)
            new_cache = cache
        return self.o_proj(out), new_cache


class DecoderLayer(nn.Module):
    def __init__(self, hidden, heads, kv_heads, head_dim, intermediate, attn_bias=False):
        super().__init__()
        self.self_attn = SelfAttention(hidden, heads, kv_heads, head_dim, attn_bias)
        self.mlp = MLP(hidden, intermediate)
        self.input_layernorm = RMSNORM(hidden)
        self.post_attention_layernorm = RMSNORM(hidden)

    def forward(self, x, cos, sin, cache=None):
        a, new_cache = self.self_attn(self.input_layernorm(x), cos, sin, cache)
        x = x + a
        return x + self.mlp(self.post_attention_layernorm(x)), new_cache


class Embedding(nn.Module):
    def __init__(self, vocab: int, hidden: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(vocab, hidden))

    def forward(self, ids):
        return self.weight[ids]


class QwenLM(nn.Module):
    def __init__(self, vocab, hidden, heads, kv_heads, head_dim, intermediate, num_layers, rope_theta=1e6,
                 attn_bias=True):
        super().__init__()
        self.embed_tokens = Embedding(vocab, hidden)
        self.layers = nn.ModuleList(
            [DecoderLayer(hidden, heads, kv_heads, head_dim, intermediate, attn_bias) for _ in range(num_layers)])
        self.norm = RMSNORM(hidden)
        self.head_dim = head_dim
        self.rope_theta = rope_theta
        self.kv_format = "fp16"

    def set_kv_format(self, fmt: str) -> None:
        self.kv_format = fmt
        for layer in self.layers:
            layer.self_attn.kv_format = fmt

    def _run(self, x, cache_list=None, need_logits=True):
        start = 0 if cache_list is None or cache_list[0] is None else cache_list[0]["k"].shape[2]
        cos, sin = rope_cache(self.head_dim, x.size(1), self.rope_theta, x.device, x.dtype, start)
        new = []
        for i, layer in enumerate(self.layers):
            x, c = layer(x, cos, sin, None if cache_list is None else cache_list[i])
            new.append(c)
        x = self.norm(x)
        return (x @ self.embed_tokens.weight.T if need_logits else None), new


@torch.inference_mode()
def greedy_decode(model: QwenLM, prompt: torch.Tensor, max_new: int):
    """Target-only greedy decoding of one sequence (1, P): the tokens SpecDec must emit, and
    the top-2 logit gap of every step (to explain divergences at near-ties)."""
    lg, cache = model._run(model.embed_tokens(prompt), None)
    out, gaps = [], []
    for _ in range(max_new):
        last = lg[0, -1].float()
        top = torch.topk(last, 2).values
        gaps.append(float(top[0] - top[1]))
        t = int(last.argmax())
        out.append(t)
        lg, cache = model._run(model.embed_tokens(torch.tensor([[t]], device=prompt.device)), cache)
    return out, gaps
