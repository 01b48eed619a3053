"""Kernel packs for the engine's model classes (the patch.install / restore /
current_pack contract of specdec/kernels/patch.py:139-173).

A pack replaces some of four engine entry points with this build's CUDA ops:

  rms     RMSNORM.forward        -> ops.rmsnorm
  rope    the module's apply_rope -> ops.apply_rope
  swiglu  MLP.forward            -> down_proj(ops.swiglu(gate_proj(x), up_proj(x)))
  attn    SelfAttention.forward  -> the engine's own cache handling (per-layer dict
                                    caches, FP8 formats, attention-phase accounting)
                                    with the score computation replaced by
                                    ops.attention (tensor-core split-KV kernel)

Packs (specdec/kernels/patch.py:13-18): "torch" (nothing), "elementwise" (rms,
rope, swiglu), "attention" (attn), "all".  An unknown pack raises ValueError.
``install`` always starts from the original entry points, so packs do not stack.

The patched module is ``specdec.engine.model_self`` unless ``set_target`` names
another module with the same surface (RMSNORM, MLP, SelfAttention classes and the
module-level apply_rope / quantize_kv_fp8 / dequantize_kv_fp8 functions).
"""

from __future__ import annotations

import importlib
import types

_PACKS = {
    "torch": frozenset(),
    "elementwise": frozenset({"rms", "rope", "swiglu"}),
    "attention": frozenset({"attn"}),
    "all": frozenset({"rms", "rope", "swiglu", "attn"}),
}

_target: types.ModuleType | None = None
_saved: dict | None = None  # original entry points of _target
_pack = "torch"


def set_target(module: types.ModuleType | None) -> None:
    """Patch ``module`` instead of specdec.engine.model_self (restores the current target first)."""
    global _target, _saved
    restore()
    _target = module
    _saved = None


def _module() -> types.ModuleType:
    global _target
    if _target is None:
        _target = importlib.import_module("specdec.engine.model_self")
    return _target


def _originals() -> dict:
    global _saved
    if _saved is None:
        m = _module()
        _saved = {
            "rope": m.apply_rope,
            "rms": m.RMSNORM.forward,
            "swiglu": m.MLP.forward,
            "attn": m.SelfAttention.forward,
        }
    return _saved


# ------------------------------------------------------------------ replacements
def _rms_forward(self, x):
    from . import ops

    return ops.rmsnorm(x, self.weight, self.eps, backend="cuda")


def _rope(x, cos, sin):
    from . import ops

    return ops.apply_rope(x, cos, sin, backend="cuda")


def _mlp_forward(self, x):
    from . import ops

    return self.down_proj(ops.swiglu(self.gate_proj(x), self.up_proj(x), backend="cuda"))


def _quant_plan(self, m, fmt: str):
    """(k_on, v_on, k_group, v_group) of the cache format (model_self.py:686-697)."""
    if fmt == "v_fp8":
        return False, True, m.GROUP_SIZE, m.GROUP_V
    if fmt == "fp8":
        return self.fp8_k, self.fp8_v, self.fp8_g_k, self.fp8_g_v
    return False, False, m.GROUP_SIZE, m.GROUP_SIZE


def _history(m, cache, key: str, cur16, dtype):
    """Full-length bf16 K or V of a dict cache plus the current tokens.  FP8 payloads
    (a ``<key>_scale`` entry) are dequantised; a bf16 history is written back at full
    length, as the engine does (model_self.py:717-729)."""
    import torch

    if key + "_scale" in cache:
        return torch.cat([m.dequantize_kv_fp8(cache[key], cache[key + "_scale"], dtype), cur16], dim=2)
    full = torch.cat([cache[key], cur16], dim=2)
    cache[key] = full
    return full


def _attn_forward(self, x, cos, sin, cache=None):
    """SelfAttention.forward (model_self.py:668-800) with the eager score tensor replaced
    by ops.attention (ops.attention_fp8v over a V-only FP8 history, which is then never
    dequantised); cache formats, FP8 quantisation and phase accounting unchanged."""
    import torch

    from . import ops

    m = _module()
    b, s, _ = x.shape

    def heads(proj, n):
        return proj(x).view(b, s, n, self.head_dim).transpose(1, 2)

    q = m.apply_rope(heads(self.q_proj, self.heads), cos, sin)
    k = m.apply_rope(heads(self.k_proj, self.kv_heads), cos, sin)
    v = heads(self.v_proj, self.kv_heads)
    fmt = cache.get("fmt", self.kv_format) if cache is not None else self.kv_format
    k_on, v_on, gk, gv = _quant_plan(self, m, fmt)
    codes = {}
    if k_on:
        codes["k"] = m.quantize_kv_fp8(k, gk)
        k_cur = m.dequantize_kv_fp8(codes["k"][0], codes["k"][1], x.dtype)
    else:
        k_cur = k
    if v_on:
        codes["v"] = m.quantize_kv_fp8(v, gv)
        v_cur = m.dequantize_kv_fp8(codes["v"][0], codes["v"][1], x.dtype)
    else:
        v_cur = v

    # V-only FP8 history (bf16 K, E4M3 V of one group per head): the kernel reads the codes
    # and scales as the cache stores them -- the new tokens' codes are appended first, as the
    # cache update below would -- and widens them inside its PV product, so the history is
    # never dequantised (the reference dequantises all of it every call, patch.py:94-103)
    fused_v = (cache is not None and fmt != "fp16" and v_on and not k_on and "v_scale" in cache
               and "k_scale" not in cache and self.head_dim == 128 and q.dtype == torch.bfloat16
               and codes["v"][1].shape[-1] == 1)
    v_codes_all = v_scale_all = None
    if cache is None:
        k_all, v_all = k_cur, v_cur
    elif fmt == "fp16":
        k_all = torch.cat([cache["k"], k], dim=2)
        v_all = torch.cat([cache["v"], v], dim=2)
        cache["k"], cache["v"] = k_all, v_all
    elif fused_v:
        k_all = _history(m, cache, "k", k_cur, x.dtype)
        v_codes_all = torch.cat([cache["v"], codes["v"][0]], dim=2)
        v_scale_all = torch.cat([cache["v_scale"], codes["v"][1]], dim=2)
        v_all = None
    else:
        k_all = _history(m, cache, "k", k_cur, x.dtype)
        v_all = _history(m, cache, "v", v_cur, x.dtype)

    T = k_all.shape[2] if cache is not None else s
    path = "eager"
    decide = getattr(m, "decide_attention_path", None)
    if decide is not None:
        path, reason = decide(m._ATTENTION_PHASE, s)
        m._record_attention_call(path, m._ATTENTION_PHASE, s, T, reason, self.heads, self.kv_heads, self.head_dim)
    if path == "fused":
        if v_all is None:
            v_all = m.dequantize_kv_fp8(v_codes_all, v_scale_all, x.dtype)
        out = m._fused_prefill_attention(q, k_all, v_all, self.head_dim)
    elif v_all is None:
        out = ops.attention_fp8v(q, k_all, v_codes_all, v_scale_all)
    else:
        out = ops.attention(q, k_all, v_all, backend="cuda")
    out = out.transpose(1, 2).contiguous().view(b, s, self.heads * self.head_dim)

    if cache is None:
        if fmt in ("fp8", "v_fp8"):
            new_cache = {"fmt": fmt}
            for key, on, full in (("k", k_on, k_all), ("v", v_on, v_all)):
                if on:
                    new_cache[key], new_cache[key + "_scale"] = codes[key]
                else:
                    new_cache[key] = full
        else:
            new_cache = {"k": k_all, "v": v_all}
    else:
        if fmt in ("fp8", "v_fp8"):
            for key in ("k", "v"):
                if key == "v" and v_codes_all is not None:
                    cache["v"], cache["v_scale"] = v_codes_all, v_scale_all  # appended above
                elif key in codes:
                    cache[key] = torch.cat([cache[key], codes[key][0]], dim=2)
                    cache[key + "_scale"] = torch.cat([cache[key + "_scale"], codes[key][1]], dim=2)
        new_cache = cache
    return self.o_proj(out), new_cache


_REPLACEMENTS = {"rms": _rms_forward, "rope": _rope, "swiglu": _mlp_forward, "attn": _attn_forward}


def _apply(entries: dict) -> None:
    m = _module()
    m.apply_rope = entries["rope"]
    m.RMSNORM.forward = entries["rms"]
    m.MLP.forward = entries["swiglu"]
    m.SelfAttention.forward = entries["attn"]


# ------------------------------------------------------------------ public API
def install(pack: str) -> str:
    """Activate a kernel pack on the engine's classes; returns the pack name."""
    global _pack
    if pack not in _PACKS:
        raise ValueError(f"unknown pack {pack!r}; choose from {sorted(_PACKS)}")
    orig = _originals()
    chosen = _PACKS[pack]
    _apply({part: (_REPLACEMENTS[part] if part in chosen else orig[part]) for part in orig})
    _pack = pack
    return pack


def restore() -> None:
    """Put the original entry points back (pack "torch")."""
    global _pack
    if _saved is not None:
        _apply(_saved)
    _pack = "torch"


def current_pack() -> str:
    return _pack
