"""Operator surface of the B200 build (mirrors specdec/kernels/ops.py:1-76).

The reference dispatches ``backend in {"torch", "cuda", "triton"}``.  This build
has exactly one implementation per op -- hand-written sm_100a CUDA behind the
C ABI -- so ``backend`` must be ``"cuda"``; any other value raises
``ValueError(backend)`` as the reference does for an unknown backend
(ops.py:39,52,64,76).  There is no CPU or eager fallback.

Beyond the reference's four ops this module exposes the paged decode path:
``paged_attention``, ``ragged_plan``, ``append_kv``, ``greedy_accept`` and
``trim_lengths``.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from .. import _lib
from ..engine.paged_cache import PagedKVCache


def triton_available() -> bool:
    """Always False: this build ships no Triton kernels (the reference checks the import, ops.py:8-13)."""
    return False


def _backend(backend: str) -> None:
    if backend != "cuda":
        raise ValueError(backend)


def _lib_handle():
    from .build import load

    return load().lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return _lib.F32
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    return -1


def _cos_sin(x, cos, sin):
    """Flatten cos/sin to (seq, dim) the way the reference op does (ops.py:15-27)."""
    seq, dim = x.shape[-2], x.shape[-1]

    def flat(t):
        t = t.to(dtype=x.dtype)
        while t.ndim > 2 and t.shape[0] == 1:
            t = t.squeeze(0)
        if tuple(t.shape) != (seq, dim):
            t = t.reshape(-1, seq, dim)[-1]
        return t.contiguous()

    return flat(cos), flat(sin)


# ---------------------------------------------------------------------------- reference ops
def rmsnorm(x, weight, eps: float = 1e-6, backend: str = "cuda"):
    _backend(backend)
    from .build import load

    return load().rmsnorm(x.contiguous(), weight.contiguous(), float(eps))


def apply_rope(x, cos, sin, backend: str = "cuda"):
    _backend(backend)
    cos, sin = _cos_sin(x, cos, sin)
    from .build import load

    return load().apply_rope(x, cos, sin)


def swiglu(gate, up, backend: str = "cuda"):
    _backend(backend)
    from .build import load

    return load().swiglu(gate.contiguous(), up.contiguous())


def attention(q, k, v, backend: str = "cuda"):
    """Offset-causal GQA attention, q (B,H,S,D), k/v (B,KV,T,D); row i sees keys j <= i + (T-S)."""
    _backend(backend)
    from .build import load

    return load().attention(q.contiguous(), k.contiguous(), v.contiguous())


def _attention_cuda(q, k, v):
    # argument checks of attention_cuda (attention.cu:245-260)
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("tensors must be CUDA")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise RuntimeError("tensors must be contiguous")
    if not (q.dim() == 4 and k.dim() == 4 and v.dim() == 4):
        raise RuntimeError("q, k, v are rank-4")
    if not (q.dtype == k.dtype == v.dtype):
        raise RuntimeError("dtype mismatch")
    B, H, S, D = q.shape
    KV, T = k.shape[1], k.shape[2]
    if k.shape[0] != B or v.shape[0] != B:
        raise RuntimeError("batch mismatch")
    if tuple(v.shape[1:3]) != (KV, T):
        raise RuntimeError("T mismatch")
    if k.shape[3] != D or v.shape[3] != D:
        raise RuntimeError("head_dim mismatch")
    code = _dtype_code(q)
    if code < 0:
        raise RuntimeError("attention supports float32 and bfloat16")
    lib = _lib_handle()
    out = torch.empty_like(q)
    ws_bytes = lib.specdec_attention_workspace_bytes(B, H, KV, S, D, 0) if code == _lib.BF16 else 0
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    rc = lib.specdec_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), code, B, H, KV, S, T, D,
        ws.data_ptr(), ws.numel(), _stream(),
    )
    _lib.check(rc, "attention")
    return out


def attention_fp8v(q, k, v_codes, v_scale):
    """The contiguous op over a V-only FP8 dict cache: q (B,H,S,128) and k (B,KV,T,128) bf16,
    v_codes (B,KV,T,128) float8_e4m3fn and v_scale (B,KV,T,1) float32 -- the cache's "v" and
    "v_scale" as stored.  Equals attention(q, k, dequantize_kv_fp8(v_codes, v_scale)) without
    forming the dequantised V: the codes are widened inside the kernel's PV product."""
    for t in (q, k, v_codes, v_scale):
        if not t.is_cuda:
            raise RuntimeError("tensors must be CUDA")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise RuntimeError("q and k must be bfloat16")
    if v_codes.dtype != torch.float8_e4m3fn or v_scale.dtype != torch.float32:
        raise RuntimeError("v_codes must be float8_e4m3fn and v_scale float32")
    q, k, v_codes, v_scale = (t.contiguous() for t in (q, k, v_codes, v_scale))
    B, H, S, D = q.shape
    KV, T = k.shape[1], k.shape[2]
    if tuple(v_codes.shape) != (B, KV, T, D) or v_scale.numel() != B * KV * T or k.shape[0] != B:
        raise RuntimeError("k, v_codes and v_scale must be (B, KV, T, D), (B, KV, T, D) and (B, KV, T, 1)")
    lib = _lib_handle()
    out = torch.empty_like(q)
    ws_bytes = lib.specdec_attention_workspace_bytes(B, H, KV, S, D, 0)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    rc = lib.specdec_attention_fp8v(q.data_ptr(), k.data_ptr(), v_codes.data_ptr(), v_scale.data_ptr(), out.data_ptr(),
                                    B, H, KV, S, T, D, ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "attention_fp8v")
    return out


def _rmsnorm_cuda(x, weight, eps):
    if not (x.is_cuda and weight.is_cuda):
        raise RuntimeError("x must be CUDA")
    if x.dtype != weight.dtype:
        raise RuntimeError("x and weight dtype differ")
    hidden = x.shape[-1]
    if hidden != weight.numel():
        raise RuntimeError("weight must match the last dimension")
    code = _dtype_code(x)
    if code < 0:
        raise RuntimeError("rmsnorm supports float32 and bfloat16")
    out = torch.empty_like(x)
    rows = x.numel() // hidden if hidden else 0
    rc = _lib_handle().specdec_rmsnorm(x.data_ptr(), weight.data_ptr(), out.data_ptr(), code, rows, hidden,
                                       float(eps), _stream())
    _lib.check(rc, "rmsnorm")
    return out


def _rope_cuda(x, cos, sin):
    if not (x.is_cuda and cos.is_cuda and sin.is_cuda):
        raise RuntimeError("tensors must be CUDA")
    if x.dim() != 4:
        raise RuntimeError("x is (batch, heads, seq, head_dim)")
    if not (x.dtype == cos.dtype == sin.dtype):
        raise RuntimeError("dtype mismatch")
    B, H, S, D = x.shape
    if cos.numel() != S * D:
        raise RuntimeError("cos must be (seq, head_dim)")
    if sin.numel() != cos.numel():
        raise RuntimeError("sin shape differs from cos")
    if x.stride(3) != 1:
        x = x.contiguous()
    code = _dtype_code(x)
    if code < 0:
        raise RuntimeError("rope supports float32 and bfloat16")
    out = torch.empty((B, H, S, D), dtype=x.dtype, device=x.device)
    rc = _lib_handle().specdec_apply_rope(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), cos.data_ptr(),
                                          sin.data_ptr(), out.data_ptr(), code, B, H, S, D, _stream())
    _lib.check(rc, "apply_rope")
    return out


def _swiglu_cuda(gate, up):
    if not (gate.is_cuda and up.is_cuda):
        raise RuntimeError("tensors must be CUDA")
    if gate.shape != up.shape:
        raise RuntimeError("gate and up shapes differ")
    if gate.dtype != up.dtype:
        raise RuntimeError("dtype mismatch")
    code = _dtype_code(gate)
    if code < 0:
        raise RuntimeError("swiglu supports float32 and bfloat16")
    out = torch.empty_like(gate)
    rc = _lib_handle().specdec_swiglu(gate.data_ptr(), up.data_ptr(), out.data_ptr(), code, gate.numel(), _stream())
    _lib.check(rc, "swiglu")
    return out


# ---------------------------------------------------------------------------- paged path
@dataclass
class RaggedBatch:
    """Device description of a ragged batch: query rows, query lengths and KV lengths.

    Query rows of all sequences are packed token-major: row ``i`` of sequence ``b``
    is packed row ``q_row0[b] + i``.  ``ctx_len[b]`` counts the KV tokens visible
    to the last query row (the new tokens included)."""

    q_row0: torch.Tensor
    q_len: torch.Tensor
    ctx_len: torch.Tensor
    num_seqs: int
    max_q_len: int
    total_rows: int
    max_ctx_len: int = 0  # host-known upper bound of ctx_len (0: unknown)

    @classmethod
    def from_lengths(cls, q_lens, ctx_lens, device="cuda") -> "RaggedBatch":
        q_lens = [int(x) for x in q_lens]
        ctx_lens = [int(x) for x in ctx_lens]
        if len(q_lens) != len(ctx_lens) or not q_lens:
            raise ValueError("one q_len and one ctx_len per sequence")
        row0, acc = [], 0
        for n in q_lens:
            row0.append(acc)
            acc += n
        t = torch.tensor([row0, q_lens, ctx_lens], dtype=torch.int32).to(device)
        return cls(t[0].contiguous(), t[1].contiguous(), t[2].contiguous(), len(q_lens), max(max(q_lens), 1), acc,
                   max(ctx_lens))


def attn_workspace(batch: RaggedBatch, num_q_heads: int, cache: PagedKVCache) -> torch.Tensor:
    nbytes = _lib_handle().specdec_attn_workspace_bytes(batch.num_seqs, num_q_heads, cache.num_kv_heads,
                                                        cache.head_dim, batch.max_q_len, 0)
    if nbytes == 0:
        raise ValueError("invalid batch geometry")
    return torch.empty(nbytes, dtype=torch.uint8, device=cache.device)


def _paged_kv(cache: PagedKVCache, layer: int) -> _lib.PagedKV:
    pool = cache.pools[layer]
    return _lib.PagedKV(
        k_pool=pool.k.data_ptr(),
        v_pool=pool.v.data_ptr(),
        v_scale=_ptr(pool.v_scale),
        page_table=cache.page_table.data_ptr(),
        num_pages=cache.num_pages,
        num_kv_heads=cache.num_kv_heads,
        head_dim=cache.head_dim,
        v_dtype=_lib.E4M3 if cache.v_dtype == "e4m3" else _lib.BF16,
        max_pages_per_seq=cache.max_pages,
    )


def attn_args(q: torch.Tensor, out: torch.Tensor, cache: PagedKVCache, layer: int, batch: RaggedBatch,
              workspace: torch.Tensor, *, sm_scale: float | None = None, status: torch.Tensor | None = None,
              reuse_plan: bool = False, split_events=None, history_ready: bool = False,
              cluster_size: int = 0) -> _lib.AttnArgs:
    """Pack the C argument struct of one paged attention call (reusable across calls).

    ``history_ready``: the caller promises that the KV history (positions below
    ctx_len - q_len), the page table and the reused plan are not written by the work
    right before this call on the stream, so the kernel may load them early.
    ``cluster_size``: 0 the library's choice of thread-block clusters for small batches,
    1 none, 8 or 16 clusters of that size (a plan and the calls reusing it agree)."""
    if q.dim() != 3 or q.dtype != torch.bfloat16:
        raise ValueError("q must be bf16 (total_rows, num_q_heads, head_dim)")
    if q.shape[2] != cache.head_dim:
        raise ValueError("q head_dim differs from the cache")
    if q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("q/out head_dim must be contiguous")
    H = q.shape[1]
    scale = (1.0 / math.sqrt(cache.head_dim)) if sm_scale is None else float(sm_scale)
    return _lib.AttnArgs(
        q=q.data_ptr(),
        out=out.data_ptr(),
        q_stride_tok=q.stride(0),
        q_stride_head=q.stride(1),
        o_stride_tok=out.stride(0),
        o_stride_head=out.stride(1),
        batch=_lib.Batch(
            q_row0=batch.q_row0.data_ptr(),
            q_len=batch.q_len.data_ptr(),
            ctx_len=batch.ctx_len.data_ptr(),
            num_seqs=batch.num_seqs,
            num_q_heads=H,
            max_q_len=batch.max_q_len,
            max_ctx_len=batch.max_ctx_len,
        ),
        kv=_paged_kv(cache, layer),
        sm_scale=scale,
        workspace=workspace.data_ptr(),
        workspace_bytes=workspace.numel(),
        status=_ptr(status),
        reuse_plan=1 if reuse_plan else 0,
        num_sms=0,
        split_event_begin=None if split_events is None else _event_handle(split_events[0]),
        split_event_end=None if split_events is None else _event_handle(split_events[1]),
        history_ready=1 if history_ready else 0,
        cluster_size=int(cluster_size),
    )


def _event_handle(ev: torch.cuda.Event) -> int:
    """Raw cudaEvent_t of a torch event (created on first use)."""
    if ev.cuda_event == 0:
        ev.record()
    return ev.cuda_event


def launch_shape(q, cache: PagedKVCache, batch: RaggedBatch, workspace: torch.Tensor, *,
                 cluster_size: int = 0) -> tuple[int, int]:
    """(grid, cluster size) of the verify kernel for this call; cluster size 0 = the persistent grid."""
    args = attn_args(q, q, cache, 0, batch, workspace, cluster_size=cluster_size)
    grid, cs = ctypes.c_int32(0), ctypes.c_int32(0)
    _lib.check(_lib_handle().specdec_attn_launch_shape(ctypes.byref(args), ctypes.byref(grid), ctypes.byref(cs)),
               "attn_launch_shape")
    return int(grid.value), int(cs.value)


def ragged_plan(q, cache: PagedKVCache, batch: RaggedBatch, workspace: torch.Tensor, *, status=None,
                cluster_size: int = 0) -> None:
    """Build the split-KV work list for ``batch`` in ``workspace`` on the device (no host sync)."""
    args = attn_args(q, q, cache, 0, batch, workspace, status=status, cluster_size=cluster_size)
    _lib.check(_lib_handle().specdec_ragged_plan(ctypes.byref(args), _stream()), "ragged_plan")


def paged_attention(q, cache: PagedKVCache, layer: int, batch: RaggedBatch, *, out=None, workspace=None,
                    sm_scale=None, status=None, reuse_plan: bool = False, split_events=None,
                    history_ready: bool = False, cluster_size: int = 0):
    """Decode / verify / ragged attention of packed query rows ``q`` (rows, H, D) over layer ``layer``.

    ``split_events`` (optional pair of torch.cuda.Event with timing) brackets the split-KV kernel."""
    if not q.is_cuda:
        raise RuntimeError("tensors must be CUDA")
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        workspace = attn_workspace(batch, q.shape[1], cache)
        reuse_plan = False
    args = attn_args(q, out, cache, layer, batch, workspace, sm_scale=sm_scale, status=status,
                     reuse_plan=reuse_plan, split_events=split_events, history_ready=history_ready,
                     cluster_size=cluster_size)
    _lib.check(_lib_handle().specdec_paged_attention(ctypes.byref(args), _stream()), "paged_attention")
    return out


def append_kv(k_new, v_new, cache: PagedKVCache, layer: int, *, row0, n_new, pos0, max_new: int,
              len_out=None, status=None) -> None:
    """Write packed new tokens k_new/v_new (rows, KV, D) bf16 into layer ``layer`` (V quantised when E4M3)."""
    for t in (k_new, v_new):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.stride(2) != 1:
            raise ValueError("k_new/v_new must be bf16 (rows, KV, D) with contiguous D")
    if k_new.stride() != v_new.stride():
        raise ValueError("k_new and v_new must share strides")
    args = _append_args(cache, layer, row0, n_new, pos0, max_new, len_out, status, k_new.data_ptr(),
                        v_new.data_ptr(), k_new.stride(0), k_new.stride(1))
    _lib.check(_lib_handle().specdec_append_kv(ctypes.byref(args), _stream()), "append_kv")


def _append_args(cache, layer, row0, n_new, pos0, max_new, len_out, status, k_ptr=0, v_ptr=0, st=0, sh=0):
    pool = cache.pools[layer]
    return _lib.AppendArgs(
        k_new=k_ptr,
        v_new=v_ptr,
        stride_tok=st,
        stride_head=sh,
        row0=row0.data_ptr(),
        n_new=n_new.data_ptr(),
        pos0=pos0.data_ptr(),
        len_out=_ptr(len_out),
        num_seqs=cache.num_seqs,
        max_new=int(max_new),
        k_pool=pool.k.data_ptr(),
        v_pool=pool.v.data_ptr(),
        v_scale=_ptr(pool.v_scale),
        page_table=cache.page_table.data_ptr(),
        num_pages=cache.num_pages,
        num_kv_heads=cache.num_kv_heads,
        head_dim=cache.head_dim,
        v_dtype=_lib.E4M3 if cache.v_dtype == "e4m3" else _lib.BF16,
        max_pages_per_seq=cache.max_pages,
        status=_ptr(status),
    )


def rope_append(qkv, cos, sin, cache: PagedKVCache, layer: int, *, num_q_heads: int, row0, n_new, pos0,
                max_new: int, q_out=None, len_out=None, status=None):
    """Rotate the q and k heads of a fused QKV projection ``qkv`` (rows, H + 2 KV, D) and append k / v.

    Returns q_out (rows, H, D): the rotated queries.  The pool receives what
    ``append_kv(apply_rope(k), v)`` would write, in one launch."""
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 3 or qkv.stride(2) != 1 or qkv.stride(1) != qkv.shape[2]:
        raise ValueError("qkv must be bf16 (rows, heads, D) with contiguous heads")
    rows, D = qkv.shape[0], qkv.shape[2]
    for t in (cos, sin):
        if t.dtype != torch.bfloat16 or t.shape != (rows, D) or not t.is_contiguous():
            raise ValueError("cos/sin must be contiguous bf16 (rows, D)")
    if q_out is None:
        q_out = torch.empty(rows, num_q_heads, D, dtype=qkv.dtype, device=qkv.device)
    args = _lib.RopeAppendArgs(qkv=qkv.data_ptr(), qkv_row_stride=qkv.stride(0), cos=cos.data_ptr(),
                               sin=sin.data_ptr(), q_out=q_out.data_ptr(), rows=rows, num_q_heads=num_q_heads,
                               kv=_append_args(cache, layer, row0, n_new, pos0, max_new, len_out, status))
    _lib.check(_lib_handle().specdec_rope_append(ctypes.byref(args), _stream()), "rope_append")
    return q_out


def swiglu_packed(gate_up, out=None):
    """silu(gate) * up of a fused (rows, 2 inter) bf16 projection -> (rows, inter)."""
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or not gate_up.is_contiguous():
        raise ValueError("gate_up must be contiguous bf16 (rows, 2 inter)")
    rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty(rows, inter, dtype=gate_up.dtype, device=gate_up.device)
    _lib.check(_lib_handle().specdec_swiglu_packed(gate_up.data_ptr(), out.data_ptr(), rows, inter, _stream()),
               "swiglu_packed")
    return out


def accept_workspace(num_seqs: int, max_rows: int, vocab: int, device="cuda") -> torch.Tensor:
    """Zero-filled accept workspace; the kernel leaves its tickets at zero, so it is reusable."""
    n = _lib_handle().specdec_accept_workspace_bytes(num_seqs, max_rows, vocab)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device)


def lmhead_workspace(rows: int, device="cuda") -> torch.Tensor:
    """Zero-filled workspace of lmhead_argmax; every call leaves it zeroed, so it is reusable."""
    n = _lib_handle().specdec_lmhead_workspace_bytes(int(rows))
    if n == 0:
        raise ValueError(f"lmhead_argmax supports 1 .. 65536 rows, got {rows}")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def lmhead_argmax(x, weight, *, out=None, max_value=None, workspace=None, status=None) -> torch.Tensor:
    """Greedy token of every row of ``x`` (rows, hidden) bf16 through the tied LM head
    ``weight`` (vocab, hidden) bf16: argmax over the bf16-rounded logits x @ weight^T, first
    index on ties, NaN largest (torch.argmax), without writing the logits.  Returns (rows,)
    int32; ``max_value`` (rows,) float32 receives the winning logit when given."""
    if x.dim() != 2 or weight.dim() != 2 or x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("x (rows, hidden) and weight (vocab, hidden) must be 2-D bf16")
    if x.shape[1] != weight.shape[1] or x.stride(1) != 1 or not weight.is_contiguous():
        raise ValueError("x rows and weight rows must share a contiguous hidden dimension")
    rows = x.shape[0]
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    if workspace is None:
        workspace = lmhead_workspace(rows, x.device)
    args = _lib.LmHeadArgs(
        x=x.data_ptr(), x_stride=x.stride(0), w=weight.data_ptr(), rows=rows, hidden=x.shape[1],
        vocab=weight.shape[0], argmax=out.data_ptr(), max_value=_ptr(max_value), workspace=workspace.data_ptr(),
        workspace_bytes=workspace.numel(), status=_ptr(status), num_sms=0)
    _lib.check(_lib_handle().specdec_lmhead_argmax(ctypes.byref(args), _stream()), "lmhead_argmax")
    return out


def greedy_accept(logits, *, row0, n_rows, cands, kp, max_rows: int, g=None, m=None, next_token=None,
                  len_before=None, len_after=None, keep_offset: int = 0, workspace=None, status=None):
    """argmax of every verify row, accepted prefix length m, next token and rolled-back lengths.

    ``logits`` is (rows, vocab) bf16/f32 with rows of sequence b at ``row0[b] ..``; or None,
    when ``g`` already holds the rows' argmaxes (lmhead_argmax) and only the accept scan runs.
    Returns (g [B, max_rows], m [B], next_token [B]) int32 device tensors."""
    if logits is None:
        if g is None:
            raise ValueError("without logits, g must hold the argmaxes")
        B = int(kp.numel())
        dev = g.device
        if m is None:
            m = torch.empty(B, dtype=torch.int32, device=dev)
        if next_token is None:
            next_token = torch.empty(B, dtype=torch.int32, device=dev)
        args = _lib.AcceptArgs(
            logits=None, logits_dtype=_lib.BF16, row_stride=0, vocab=0, row0=_ptr(row0), n_rows=n_rows.data_ptr(),
            cands=cands.data_ptr(), kp=kp.data_ptr(), num_seqs=B, max_rows=int(max_rows),
            max_cands=int(cands.shape[1]), g=g.data_ptr(), m=m.data_ptr(), next_token=next_token.data_ptr(),
            len_before=_ptr(len_before), len_after=_ptr(len_after), keep_offset=int(keep_offset), workspace=None,
            workspace_bytes=0, status=_ptr(status))
        _lib.check(_lib_handle().specdec_greedy_accept(ctypes.byref(args), _stream()), "greedy_accept")
        return g, m, next_token
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be (rows, vocab) with contiguous vocab")
    code = _dtype_code(logits)
    if code < 0:
        raise ValueError("logits must be bf16 or f32")
    B = int(kp.numel())
    max_cands = int(cands.shape[1])
    dev = logits.device
    if g is None:
        g = torch.empty(B, max_rows, dtype=torch.int32, device=dev)
    if m is None:
        m = torch.empty(B, dtype=torch.int32, device=dev)
    if next_token is None:
        next_token = torch.empty(B, dtype=torch.int32, device=dev)
    if workspace is None:
        workspace = accept_workspace(B, max_rows, logits.shape[1], dev)
    args = _lib.AcceptArgs(
        logits=logits.data_ptr(),
        logits_dtype=code,
        row_stride=logits.stride(0),
        vocab=logits.shape[1],
        row0=row0.data_ptr(),
        n_rows=n_rows.data_ptr(),
        cands=cands.data_ptr(),
        kp=kp.data_ptr(),
        num_seqs=B,
        max_rows=int(max_rows),
        max_cands=max_cands,
        g=g.data_ptr(),
        m=m.data_ptr(),
        next_token=next_token.data_ptr(),
        len_before=_ptr(len_before),
        len_after=_ptr(len_after),
        keep_offset=int(keep_offset),
        workspace=workspace.data_ptr(),
        workspace_bytes=workspace.numel(),
        status=_ptr(status),
    )
    _lib.check(_lib_handle().specdec_greedy_accept(ctypes.byref(args), _stream()), "greedy_accept")
    return g, m, next_token


def trim_lengths(cur_len, new_len, out=None, status=None):
    """Device rollback: out[b] = new_len[b] if 0 < new_len[b] <= cur_len[b] else cur_len[b] (+ status bit)."""
    if out is None:
        out = torch.empty_like(cur_len)
    rc = _lib_handle().specdec_trim(cur_len.data_ptr(), new_len.data_ptr(), out.data_ptr(), int(cur_len.numel()),
                                    _ptr(status), _stream())
    _lib.check(rc, "trim")
    return out
