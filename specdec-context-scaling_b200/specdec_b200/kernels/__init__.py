"""B200 (sm_100a) kernels with the call surface of specdec/kernels (__init__.py:1-3)."""

from .ops import apply_rope, attention, rmsnorm, swiglu, triton_available

__all__ = ["apply_rope", "attention", "rmsnorm", "swiglu", "triton_available"]
