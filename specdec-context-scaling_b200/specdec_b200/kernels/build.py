"""Build and load the sm_100a extension (replaces specdec/kernels/build.py:17-52).

The reference JIT-compiles a pybind11 module for whatever GPU is visible.  This
build compiles one C-ABI shared library for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with ``make`` in the package
root and binds it with ctypes, so it cross-compiles on a machine without a GPU
and the built ``.so`` travels with the source tree.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

from .. import _lib

PKG_ROOT = Path(__file__).resolve().parents[2]  # .../specdec-context-scaling_b200

_MOD = None


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile csrc/*.cu into specdec_b200/libspecdec_b200.so (incremental)."""
    jobs = jobs or min(8, os.cpu_count() or 1)
    cmd = ["make", "-C", str(PKG_ROOT), f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed:\n{res.stdout}\n{res.stderr}")
    return _lib.LIB_PATH


class _Module:
    """The object ``load()`` returns: the reference extension's four ops plus the paged path."""

    def __init__(self, lib):
        self.lib = lib

    def attention(self, q, k, v):
        from . import ops

        return ops._attention_cuda(q, k, v)

    def rmsnorm(self, x, weight, eps):
        from . import ops

        return ops._rmsnorm_cuda(x, weight, eps)

    def apply_rope(self, x, cos, sin):
        from . import ops

        return ops._rope_cuda(x, cos, sin)

    def swiglu(self, gate, up):
        from . import ops

        return ops._swiglu_cuda(gate, up)


def load():
    """Return the loaded extension module; needs a CUDA device, as the reference's load()."""
    global _MOD
    if _MOD is not None:
        return _MOD
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required to build the custom kernels")
    _MOD = _Module(_lib.load_library())
    return _MOD
