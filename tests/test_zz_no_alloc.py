"""GPU: the no-allocation paged attention entry point (specdec_paged_attention_noalloc).

Some callers cannot give this library scratch memory: a plugin host that owns all
device memory and passes only inputs, outputs and a stream, or an FFI binding
without a CUDA allocator.  For them the library keeps a 32 MiB scratch array of its
own.  These tests call that entry point through the C ABI (ctypes) twice in a row,
on two different batches, and compare each result with the regular entry point
(caller workspace) under the attention tolerance of the other GPU tests, and with the
CPU oracle.  The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from gpu_helpers import ATOL, RTOL, assert_close_attention, build_cache, oracle_rows
from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _noalloc_call(q, cache, batch):
    from specdec_b200 import _lib
    from specdec_b200.kernels import ops

    lib = _lib.load_library()
    out = torch.full_like(q, float("nan"))
    dummy = torch.empty(256, dtype=torch.uint8, device=q.device)
    args = ops.attn_args(q, out, cache, 0, batch, dummy)
    args.workspace = None  # the entry point must not need a caller workspace
    args.workspace_bytes = 0
    rc = lib.specdec_paged_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "paged_attention_noalloc")
    return out


def _case(lens, q_lens, fp8, seed, H=12, D=128):
    from specdec_b200.kernels import ops

    cache, ks, vrefs = build_cache(lens, 2, D, fp8=fp8, seed=seed)
    batch = ops.RaggedBatch.from_lengths(q_lens, lens)
    q = torch.randn(batch.total_rows, H, D, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
    return cache, batch, q.cuda(), oracle_rows(q, ks, vrefs, q_lens)


def test_noalloc_matches_workspace_entry_two_calls():
    from specdec_b200.kernels import ops

    cases = [
        _case([8192], [5], fp8=True, seed=41),               # batch-1 verify, many splits
        _case([300, 2048, 77, 1500], [1, 5, 5, 1], fp8=False, seed=42),  # ragged mixed rows
        _case([8192, 640], [1, 1], fp8=False, seed=43, H=14, D=64),     # draft decode (KV-head pairs)
    ]
    for cache, batch, q, ref in cases:
        got = _noalloc_call(q, cache, batch)
        want = ops.paged_attention(q, cache, 0, batch)
        torch.cuda.synchronize()
        ok, err, _ = oatt.within_tolerance(got.cpu(), want.cpu(), RTOL, ATOL)
        assert ok, f"no-alloc output differs from the workspace entry point (max |err| {err:.3e})"
        # and both against the oracle (the fp32 attention formula on the dequantised history)
        assert_close_attention(got.cpu(), ref, "no-alloc vs oracle")


def test_noalloc_rejects_batches_beyond_the_static_scratch():
    from specdec_b200 import _lib
    from specdec_b200.engine.paged_cache import PagedKVCache
    from specdec_b200.kernels import ops

    lib = _lib.load_library()
    B = 512
    cache = PagedKVCache.allocate(1, B, 2, 128, 16, device="cuda")
    batch = ops.RaggedBatch.from_lengths([5] * B, [16] * B)
    q = torch.zeros(batch.total_rows, 12, 128, dtype=torch.bfloat16, device="cuda")
    dummy = torch.empty(256, dtype=torch.uint8, device="cuda")
    args = ops.attn_args(q, q, cache, 0, batch, dummy)
    rc = lib.specdec_paged_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_WORKSPACE
    assert "static scratch" in lib.specdec_last_error().decode()
