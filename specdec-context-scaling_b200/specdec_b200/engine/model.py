"""Qwen2-style decoder over the paged KV cache, running this build's kernels.

The forward math is the reference engine's (specdec/engine/model_self.py: RMSNORM
:225-235, SelfAttention :668-800, MLP :246-270, DecoderLayer, QwenLM._run :845-860
with tied embeddings) on a different data layout: the query rows of a batch are
packed token-major, every sequence owns pages of a static-capacity pool, and the
new K/V rows are appended in place instead of re-concatenating the history.

Per layer of a decode / verify step (rows = packed query rows of all sequences):
  h   = rmsnorm(x)                                 specdec_rmsnorm
  qkv = h W_qkv^T + b_qkv                          cuBLAS (one fused GEMM)
  q = rope(q) out; rope(k) and v appended to the layer's pages (V quantised to E4M3
      for an e4m3 cache), one launch                specdec_rope_append
  o   = paged attention of q over the layer's pages        specdec_paged_attention
  x  += o W_o^T                                    cuBLAS (residual added in place)
  x  += W_down swiglu(W_gate|up rmsnorm(x))        specdec_rmsnorm, cuBLAS, specdec_swiglu_packed
Prefill (the whole prompt at once) uses torch's fused causal attention for the
prompt block and appends the prompt's K/V into the pages; decode never does.

Weights come from a state dict with the reference's parameter names
(``embed_tokens.weight``, ``layers.{i}.self_attn.q_proj.weight`` ...), so a
reference QwenLM's weights load directly, or from a seeded random init.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..kernels import ops
from .paged_cache import PagedKVCache


@dataclass(frozen=True)
class ModelConfig:
    vocab: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    layers: int
    rope_theta: float = 1_000_000.0
    eps: float = 1e-6
    attn_bias: bool = True


# BASELINE geometries: target Qwen2.5-1.5B, draft Qwen2.5-0.5B (random-init weights)
QWEN25_1P5B = ModelConfig(vocab=151936, hidden=1536, heads=12, kv_heads=2, head_dim=128, intermediate=8960, layers=28)
QWEN25_0P5B = ModelConfig(vocab=151936, hidden=896, heads=14, kv_heads=2, head_dim=64, intermediate=4864, layers=24)


def random_state(cfg: ModelConfig, seed: int, device="cuda", std: float = 0.02, dtype=torch.bfloat16) -> dict:
    """Seeded random weights with the reference's parameter names (same seed -> same weights
    on every rank, so data-parallel ranks need no weight broadcast)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    H, KV, D, Hd, I = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.intermediate
    sd = {"embed_tokens.weight": rnd(cfg.vocab, Hd), "norm.weight": torch.ones(Hd, dtype=dtype, device=device)}
    for i in range(cfg.layers):
        p = f"layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = rnd(H * D, Hd)
        sd[p + "self_attn.k_proj.weight"] = rnd(KV * D, Hd)
        sd[p + "self_attn.v_proj.weight"] = rnd(KV * D, Hd)
        if cfg.attn_bias:
            sd[p + "self_attn.q_proj.bias"] = rnd(H * D)
            sd[p + "self_attn.k_proj.bias"] = rnd(KV * D)
            sd[p + "self_attn.v_proj.bias"] = rnd(KV * D)
        sd[p + "self_attn.o_proj.weight"] = rnd(Hd, H * D)
        sd[p + "mlp.gate_proj.weight"] = rnd(I, Hd)
        sd[p + "mlp.up_proj.weight"] = rnd(I, Hd)
        sd[p + "mlp.down_proj.weight"] = rnd(Hd, I)
        sd[p + "input_layernorm.weight"] = torch.ones(Hd, dtype=dtype, device=device)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(Hd, dtype=dtype, device=device)
    return sd


def _e4m3_round_trip(v: torch.Tensor) -> torch.Tensor:
    """bf16(e4m3(v / s) * s) with s = max|v| / 448 per token row (1 for an all-zero row): the
    values specdec_append_kv's codes and scales stand for (quantize_kv_fp8 with one group per
    head, model_self.py:304-320).  Used by the prompt pass only."""
    x = v.float()
    s = x.abs().amax(dim=-1, keepdim=True) / 448.0
    s = torch.where(s == 0, torch.ones_like(s), s)
    return ((x / s).to(torch.float8_e4m3fn).float() * s).to(v.dtype)


@dataclass
class _Layer:
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor | None
    w_o: torch.Tensor
    w_gu: torch.Tensor  # gate_proj and up_proj stacked: (2 inter, hidden)
    w_down: torch.Tensor
    ln1: torch.Tensor
    ln2: torch.Tensor


class StepLayout:
    """Static row layout of one batched step: sequence b owns packed rows
    b * q_max .. b * q_max + q_max - 1 and uses the first ``q_len[b]`` of them.

    The device tensors are updated in place (no host sync) before each step, so a
    step captured in a CUDA graph replays with new lengths."""

    def __init__(self, num_seqs: int, q_max: int, device):
        self.num_seqs, self.q_max, self.rows = num_seqs, q_max, num_seqs * q_max
        i32 = dict(dtype=torch.int32, device=device)
        self.q_row0 = torch.arange(num_seqs, **i32) * q_max
        self.q_len = torch.full((num_seqs,), q_max, **i32)
        self.pos0 = torch.zeros(num_seqs, **i32)      # cache length before the step
        self.ctx_len = torch.full((num_seqs,), q_max, **i32)
        self.offs = torch.arange(q_max, device=device, dtype=torch.int32)
        self.batch = ops.RaggedBatch(self.q_row0, self.q_len, self.ctx_len, num_seqs, q_max, self.rows)

    def set(self, pos0: torch.Tensor, q_len: torch.Tensor | None = None) -> None:
        """Device-side update: new query lengths (optional) and cache lengths."""
        if q_len is not None:
            self.q_len.copy_(q_len)
        self.pos0.copy_(pos0)
        torch.add(self.pos0, self.q_len, out=self.ctx_len)

    def positions(self) -> torch.Tensor:
        """(rows,) sequence position of every packed row (padding rows repeat the last one)."""
        last = (self.q_len - 1).clamp(min=0).unsqueeze(1)
        return (self.pos0.unsqueeze(1) + torch.minimum(self.offs.unsqueeze(0), last)).reshape(-1)

    def last_rows(self) -> torch.Tensor:
        """(num_seqs,) packed row of every sequence's last query row."""
        return (self.q_row0 + self.q_len - 1).long()


class PagedModel:
    """Decoder weights in fused, layout-ready form plus the batched paged forward."""

    def __init__(self, cfg: ModelConfig, state: dict, device="cuda", dtype=torch.bfloat16):
        self.cfg = cfg
        self.device = torch.device(device)

        def get(k):
            return state[k].to(device=self.device, dtype=dtype).contiguous()

        self.embed = get("embed_tokens.weight")
        self.norm = get("norm.weight")
        self.layers = []
        for i in range(cfg.layers):
            p = f"layers.{i}."
            a = p + "self_attn."
            w_qkv = torch.cat([get(a + "q_proj.weight"), get(a + "k_proj.weight"), get(a + "v_proj.weight")])
            b_qkv = None
            if (a + "q_proj.bias") in state:
                b_qkv = torch.cat([get(a + "q_proj.bias"), get(a + "k_proj.bias"), get(a + "v_proj.bias")])
            self.layers.append(_Layer(w_qkv.contiguous(), None if b_qkv is None else b_qkv.contiguous(),
                                      get(a + "o_proj.weight"),
                                      torch.cat([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")]),
                                      get(p + "mlp.down_proj.weight"),
                                      get(p + "input_layernorm.weight"), get(p + "post_attention_layernorm.weight")))
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=self.device,
                                                               dtype=torch.float32) / cfg.head_dim))

    @classmethod
    def random(cls, cfg: ModelConfig, seed: int, device="cuda") -> "PagedModel":
        return cls(cfg, random_state(cfg, seed, device), device)

    def new_cache(self, num_seqs: int, capacity: int, v_dtype: str = "bf16") -> PagedKVCache:
        c = self.cfg
        return PagedKVCache.allocate(c.layers, num_seqs, c.kv_heads, c.head_dim, capacity, v_dtype=v_dtype,
                                     device=self.device)

    # ------------------------------------------------------------------ pieces
    def _cos_sin(self, pos: torch.Tensor):
        """(rows, D) cos / sin in the model dtype at integer positions ``pos`` (model_self.py:272-284)."""
        ang = pos.float().unsqueeze(1) * self.inv_freq.unsqueeze(0)
        cos = torch.cat([ang.cos(), ang.cos()], dim=1).to(self.embed.dtype)
        sin = torch.cat([ang.sin(), ang.sin()], dim=1).to(self.embed.dtype)
        return cos, sin

    def _qkv(self, L: _Layer, h: torch.Tensor, cos, sin):
        """Packed rows -> q (1, H, rows, D) and k (1, KV, rows, D) after RoPE, v (KV, rows, D)."""
        c = self.cfg
        rows = h.shape[0]
        qkv = torch.addmm(L.b_qkv, h, L.w_qkv.t()) if L.b_qkv is not None else h @ L.w_qkv.t()
        qkv = qkv.view(rows, c.heads + 2 * c.kv_heads, c.head_dim)
        q = ops.apply_rope(qkv[:, :c.heads].transpose(0, 1).unsqueeze(0), cos, sin)
        k = ops.apply_rope(qkv[:, c.heads:c.heads + c.kv_heads].transpose(0, 1).unsqueeze(0), cos, sin)
        v = qkv[:, c.heads + c.kv_heads:].transpose(0, 1).contiguous()
        return q, k, v

    def _mlp(self, L: _Layer, x: torch.Tensor) -> torch.Tensor:
        """x + down(silu(gate(h)) * up(h)), h = rmsnorm(x): one gate|up GEMM, the residual
        added by the down GEMM (in place on x)."""
        h = ops.rmsnorm(x, L.ln2, self.cfg.eps)
        return x.addmm_(ops.swiglu_packed(h @ L.w_gu.t()), L.w_down.t())

    def logits(self, hidden_rows: torch.Tensor) -> torch.Tensor:
        """Tied LM head (model_self.py:857): (n, hidden) -> (n, vocab)."""
        return hidden_rows @ self.embed.t()

    def greedy(self, hidden_rows: torch.Tensor, out: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
        """Greedy tokens (n,) int32 of the tied LM head without writing the logits
        (specdec_lmhead_argmax: the LM-head GEMM fused with torch.argmax's order)."""
        return ops.lmhead_argmax(hidden_rows, self.embed, out=out, workspace=workspace)

    # ------------------------------------------------------------------ forward passes
    def step(self, tokens: torch.Tensor, layout: StepLayout, cache: PagedKVCache, workspace: torch.Tensor,
             *, status: torch.Tensor | None = None) -> torch.Tensor:
        """One decode / verify step of ``layout.rows`` packed query rows (token ids ``tokens``).

        Appends every sequence's ``q_len`` new K/V rows at positions ``pos0 ..`` of all
        layers and returns the final-norm hidden states (rows, hidden).  Rows past a
        sequence's q_len are padding: their outputs are meaningless and never stored."""
        c = self.cfg
        rows = layout.rows
        x = self.embed[tokens.long()]
        cos, sin = self._cos_sin(layout.positions())
        q = torch.empty(rows, c.heads, c.head_dim, dtype=x.dtype, device=x.device)
        # attention writes every row of each sequence's q_len; padding rows stay unset
        # (meaningless, never stored, never mixed into other rows)
        o = torch.empty(rows, c.heads, c.head_dim, dtype=x.dtype, device=x.device)
        for li, L in enumerate(self.layers):
            h = ops.rmsnorm(x, L.ln1, c.eps)
            qkv = torch.addmm(L.b_qkv, h, L.w_qkv.t()) if L.b_qkv is not None else h @ L.w_qkv.t()
            # rotated q, and rotated k + v appended to the cache, in one launch
            ops.rope_append(qkv.view(rows, c.heads + 2 * c.kv_heads, c.head_dim), cos, sin, cache, li,
                            num_q_heads=c.heads, row0=layout.q_row0, n_new=layout.q_len, pos0=layout.pos0,
                            max_new=layout.q_max, q_out=q, status=status)
            # layers after the first reuse layer 0's plan; the only KV the steps before write
            # is this step's new tokens, so the history may be loaded early
            ops.paged_attention(q, cache, li, layout.batch, out=o, workspace=workspace, reuse_plan=li > 0,
                                status=status, history_ready=li > 0)
            x.addmm_(o.view(rows, c.heads * c.head_dim), L.w_o.t())
            x = self._mlp(L, x)
        return ops.rmsnorm(x, self.norm, c.eps)

    def prefill(self, ids: torch.Tensor, cache: PagedKVCache, seq0: int, *, need_logits: bool = True,
                status: torch.Tensor | None = None) -> torch.Tensor | None:
        """Prompt pass of sequences seq0 .. seq0 + n - 1 (ids (n, P)): writes their K/V at
        positions 0 .. P-1 of every layer, sets their lengths to P and returns the logits
        of each prompt's last position (n, vocab).  The causal attention inside the
        prompt block uses torch's fused attention (prefill is not the decode path)."""
        c = self.cfg
        n, P = ids.shape
        rows = n * P
        dev = ids.device
        i32 = dict(dtype=torch.int32, device=dev)
        seqs = torch.arange(cache.num_seqs, **i32)
        inside = (seqs >= seq0) & (seqs < seq0 + n)
        row0 = torch.where(inside, (seqs - seq0) * P, torch.zeros_like(seqs))
        n_new = torch.where(inside, torch.full_like(seqs, P), torch.zeros_like(seqs))
        pos0 = torch.zeros(cache.num_seqs, **i32)
        x = self.embed[ids.reshape(-1).long()]
        cos, sin = self._cos_sin(torch.arange(P, device=dev).repeat(n))
        n_rep = c.heads // c.kv_heads
        for li, L in enumerate(self.layers):
            h = ops.rmsnorm(x, L.ln1, c.eps)
            q, k, v = self._qkv(L, h, cos, sin)
            ops.append_kv(k[0].transpose(0, 1), v.transpose(0, 1), cache, li, row0=row0, n_new=n_new, pos0=pos0,
                          max_new=P, status=status)
            if cache.v_dtype == "e4m3":
                # the prompt attends over the V the pool now holds (E4M3 codes times their
                # scales), as the reference's V-only FP8 prompt pass attends over
                # dequantize(quantize(v)) (model_self.py:702-704)
                v = _e4m3_round_trip(v)
            q4 = q[0].view(c.heads, n, P, c.head_dim).transpose(0, 1)
            k4 = k[0].view(c.kv_heads, n, P, c.head_dim).transpose(0, 1).repeat_interleave(n_rep, dim=1)
            v4 = v.view(c.kv_heads, n, P, c.head_dim).transpose(0, 1).repeat_interleave(n_rep, dim=1)
            o = F.scaled_dot_product_attention(q4, k4, v4, is_causal=True, scale=1.0 / math.sqrt(c.head_dim))
            x = x + o.transpose(1, 2).reshape(rows, c.heads * c.head_dim) @ L.w_o.t()
            x = self._mlp(L, x)
        cache.lengths.copy_(torch.where(inside, torch.full_like(seqs, P), cache.lengths))
        cache.host_lengths = None
        if not need_logits:
            return None
        last = x.view(n, P, -1)[:, -1]
        return self.logits(ops.rmsnorm(last.contiguous(), self.norm, c.eps))
