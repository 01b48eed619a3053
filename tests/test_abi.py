"""C ABI: the library loads without a GPU, exports every symbol of include/specdec_b200.h,
and rejects bad host arguments before touching the device (the reference's
TORCH_CHECK conditions, attention.cu:245-260, become SPECDEC_ERR_INVALID)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "specdec_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(specdec_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("specdec_paged_attention", "specdec_append_kv", "specdec_greedy_accept", "specdec_trim",
                 "specdec_attention", "specdec_rmsnorm", "specdec_apply_rope", "specdec_swiglu",
                 "specdec_ragged_plan"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    from specdec_b200 import _lib

    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # and the ctypes signature table covers the header exactly
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_abi_version(lib):
    assert lib.specdec_abi_version() == 3


def test_workspace_sizes_are_host_only(lib):
    n1 = lib.specdec_attn_workspace_bytes(1, 12, 2, 128, 5, 148)
    n64 = lib.specdec_attn_workspace_bytes(64, 12, 2, 128, 5, 148)
    assert 0 < n1 < n64
    assert n1 % 256 == 0
    assert lib.specdec_attn_workspace_bytes(1, 12, 5, 128, 5, 148) == 0  # heads do not divide
    assert lib.specdec_accept_workspace_bytes(4, 5, 151936) > 0
    assert lib.specdec_accept_workspace_bytes(0, 5, 151936) == 0


@pytest.mark.parametrize(
    "B,H,KV,S,T,D,dtype,msg",
    [
        (1, 12, 5, 1, 16, 128, 1, "query heads must divide KV heads"),
        (1, 12, 2, 1, 16, 96, 1, "head_dim must be 64 or 128"),
        (1, 12, 2, 0, 16, 128, 1, "empty sequence"),
        (1, 12, 2, 1, 0, 128, 1, "empty sequence"),
        (1, 12, 2, 1, 16, 128, 7, "attention supports float32 and bfloat16"),
    ],
)
def test_attention_rejects_bad_arguments_without_a_device(lib, B, H, KV, S, T, D, dtype, msg):
    fake = ctypes.c_void_p(0x1000)
    rc = lib.specdec_attention(fake, fake, fake, fake, dtype, B, H, KV, S, T, D, fake, 1 << 20, None)
    assert rc == 1
    assert msg in lib.specdec_last_error().decode()


def test_paged_attention_rejects_null_args(lib):
    from specdec_b200 import _lib

    rc = lib.specdec_paged_attention(None, None)
    assert rc == _lib.ERR_INVALID
    args = _lib.AttnArgs()
    rc = lib.specdec_paged_attention(ctypes.byref(args), None)
    assert rc == _lib.ERR_INVALID
    assert "device pointers" in lib.specdec_last_error().decode()


def test_append_rejects_fp8_with_head_dim_64(lib):
    from specdec_b200 import _lib

    a = _lib.AppendArgs(k_new=0x1000, v_new=0x1000, row0=0x1000, n_new=0x1000, pos0=0x1000, num_seqs=1, max_new=1,
                        k_pool=0x1000, v_pool=0x1000, v_scale=0x1000, page_table=0x1000, num_pages=1,
                        num_kv_heads=2, head_dim=64, v_dtype=_lib.E4M3, max_pages_per_seq=1)
    assert lib.specdec_append_kv(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED


def test_struct_layouts_match_c():
    """ctypes layouts: sizes the C compiler gives these structs (x86-64 SysV)."""
    from specdec_b200 import _lib

    assert ctypes.sizeof(_lib.PagedKV) == 56
    assert ctypes.sizeof(_lib.Batch) == 40
    assert ctypes.sizeof(_lib.AttnArgs) == 8 * 2 + 8 * 4 + 40 + 56 + 8 + 8 + 8 + 8 + 8 + 16 + 8


def test_ops_reject_other_backends():
    import torch

    from specdec_b200.kernels import ops

    x = torch.zeros(2, 4)
    for backend in ("torch", "triton", "cpu"):
        with pytest.raises(ValueError):
            ops.attention(x, x, x, backend=backend)
        with pytest.raises(ValueError):
            ops.rmsnorm(x, x[0], backend=backend)
    assert ops.triton_available() is False


def test_wait_selftest_rejects_bad_arguments_without_a_device(lib):
    from specdec_b200 import _lib

    assert lib.specdec_wait_selftest(2, None, 1, 1, 1_000_000, None, None, None) == _lib.ERR_INVALID
    assert lib.specdec_wait_selftest(0, None, 1, 1, 10 ** 10, None, None, None) == _lib.ERR_INVALID
    assert lib.specdec_wait_selftest(1, None, 1, 1, 1_000_000, None, None, None) == _lib.ERR_INVALID
    assert lib.specdec_wait_selftest(0, None, 1, 2, 1_000_000, None, None, None) == _lib.ERR_INVALID
