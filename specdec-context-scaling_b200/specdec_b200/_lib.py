"""ctypes binding of libspecdec_b200.so (the C ABI declared in include/specdec_b200.h).

The shared library is built in-tree by ``specdec_b200.kernels.build.build()``
(``make`` in the package root).  Loading fails loudly when the library is
missing: this package has no CPU or eager-PyTorch fallback for any op.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libspecdec_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

PAGE_TOKENS = 16
ABI_VERSION = 3

F32, BF16, E4M3 = 0, 1, 2

# result codes
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = 0, 1, 2, 3, 4

# device status bits
STATUS_BAD_LENGTH = 0x1
STATUS_PAGE_OVERFLOW = 0x2
STATUS_BAD_PAGE = 0x4
STATUS_TRIM_RANGE = 0x8
STATUS_TIMEOUT = 0x10
STATUS_ACCEPT_RANGE = 0x20
STATUS_PLAN_MISMATCH = 0x40

STATUS_NAMES = {
    STATUS_BAD_LENGTH: "bad length (ctx_len < q_len or q_len > max_q_len)",
    STATUS_PAGE_OVERFLOW: "position beyond the page table",
    STATUS_BAD_PAGE: "page id outside the pool",
    STATUS_TRIM_RANGE: "trim length out of range",
    STATUS_TIMEOUT: "bounded device wait timed out",
    STATUS_ACCEPT_RANGE: "accept row/candidate count out of range",
    STATUS_PLAN_MISMATCH: "reused plan was built for another launch shape (cluster choice or SM budget)",
}

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t


class PagedKV(ctypes.Structure):
    _fields_ = [
        ("k_pool", _vp),
        ("v_pool", _vp),
        ("v_scale", _vp),
        ("page_table", _vp),
        ("num_pages", _i32),
        ("num_kv_heads", _i32),
        ("head_dim", _i32),
        ("v_dtype", _i32),
        ("max_pages_per_seq", _i32),
    ]


class Batch(ctypes.Structure):
    _fields_ = [
        ("q_row0", _vp),
        ("q_len", _vp),
        ("ctx_len", _vp),
        ("num_seqs", _i32),
        ("num_q_heads", _i32),
        ("max_q_len", _i32),
        ("max_ctx_len", _i32),
    ]


class LmHeadArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp),
        ("x_stride", _i64),
        ("w", _vp),
        ("rows", _i32),
        ("hidden", _i32),
        ("vocab", _i32),
        ("argmax", _vp),
        ("max_value", _vp),
        ("workspace", _vp),
        ("workspace_bytes", _sz),
        ("status", _vp),
        ("num_sms", _i32),
    ]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp),
        ("out", _vp),
        ("q_stride_tok", _i64),
        ("q_stride_head", _i64),
        ("o_stride_tok", _i64),
        ("o_stride_head", _i64),
        ("batch", Batch),
        ("kv", PagedKV),
        ("sm_scale", ctypes.c_float),
        ("workspace", _vp),
        ("workspace_bytes", _sz),
        ("status", _vp),
        ("reuse_plan", _i32),
        ("num_sms", _i32),
        ("split_event_begin", _vp),
        ("split_event_end", _vp),
        ("history_ready", _i32),
        ("cluster_size", _i32),
    ]


class AppendArgs(ctypes.Structure):
    _fields_ = [
        ("k_new", _vp),
        ("v_new", _vp),
        ("stride_tok", _i64),
        ("stride_head", _i64),
        ("row0", _vp),
        ("n_new", _vp),
        ("pos0", _vp),
        ("len_out", _vp),
        ("num_seqs", _i32),
        ("max_new", _i32),
        ("k_pool", _vp),
        ("v_pool", _vp),
        ("v_scale", _vp),
        ("page_table", _vp),
        ("num_pages", _i32),
        ("num_kv_heads", _i32),
        ("head_dim", _i32),
        ("v_dtype", _i32),
        ("max_pages_per_seq", _i32),
        ("status", _vp),
    ]


class RopeAppendArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", _vp),
        ("qkv_row_stride", _i64),
        ("cos", _vp),
        ("sin", _vp),
        ("q_out", _vp),
        ("rows", _i32),
        ("num_q_heads", _i32),
        ("kv", AppendArgs),
    ]


class AcceptArgs(ctypes.Structure):
    _fields_ = [
        ("logits", _vp),
        ("logits_dtype", _i32),
        ("row_stride", _i64),
        ("vocab", _i32),
        ("row0", _vp),
        ("n_rows", _vp),
        ("cands", _vp),
        ("kp", _vp),
        ("num_seqs", _i32),
        ("max_rows", _i32),
        ("max_cands", _i32),
        ("g", _vp),
        ("m", _vp),
        ("next_token", _vp),
        ("len_before", _vp),
        ("len_after", _vp),
        ("keep_offset", _i32),
        ("workspace", _vp),
        ("workspace_bytes", _sz),
        ("status", _vp),
    ]


# name -> (restype, argtypes): every symbol include/specdec_b200.h declares
SIGNATURES = {
    "specdec_attn_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "specdec_ragged_plan": (ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    "specdec_paged_attention": (ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    "specdec_paged_attention_noalloc": (ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    "specdec_append_kv": (ctypes.c_int, [ctypes.POINTER(AppendArgs), _vp]),
    "specdec_rope_append": (ctypes.c_int, [ctypes.POINTER(RopeAppendArgs), _vp]),
    "specdec_accept_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "specdec_greedy_accept": (ctypes.c_int, [ctypes.POINTER(AcceptArgs), _vp]),
    "specdec_trim": (ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "specdec_attention_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "specdec_attention": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp],
    ),
    "specdec_rmsnorm": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i64, _i32, ctypes.c_float, _vp]),
    "specdec_apply_rope": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp],
    ),
    "specdec_swiglu": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i64, _vp]),
    "specdec_swiglu_packed": (ctypes.c_int, [_vp, _vp, _i64, _i64, _vp]),
    "specdec_umma_selftest": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "specdec_gather4_selftest": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "specdec_wait_selftest": (ctypes.c_int, [_i32, _vp, _i32, _i32, _i64, _vp, _vp, _vp]),
    "specdec_attn_launch_shape": (ctypes.c_int, [_vp, _vp, _vp]),
    "specdec_lmhead_workspace_bytes": (_sz, [_i32]),
    "specdec_attention_fp8v": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz,
                                              _vp]),
    "specdec_lmhead_argmax": (ctypes.c_int, [_vp, _vp]),
    "specdec_last_error": (ctypes.c_char_p, []),
    "specdec_abi_version": (ctypes.c_int, []),
    "specdec_launch_count": (_i64, []),
}

_LIB = None


class SpecdecError(RuntimeError):
    """A C-ABI entry point refused its arguments or failed to launch."""


def load_library(path: os.PathLike | str | None = None):
    """Load the shared library once and bind every exported symbol."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p.name} is not built; run specdec_b200.kernels.build.build() (make in {p.parent.parent})"
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.specdec_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{p.name} ABI {lib.specdec_abi_version()} != expected {ABI_VERSION}")
    if path is None:
        _LIB = lib
    return lib


def check(rc: int, what: str) -> None:
    """Raise SpecdecError (a RuntimeError, as TORCH_CHECK raised in the reference) on a nonzero code."""
    if rc != OK:
        msg = _LIB.specdec_last_error().decode("utf-8", "replace") if _LIB is not None else ""
        raise SpecdecError(f"{what} failed (code {rc}): {msg}")


def status_message(bits: int) -> str:
    return "; ".join(text for bit, text in STATUS_NAMES.items() if bits & bit) or "ok"
