"""GPU: the tcgen05 operand layouts (128-byte-swizzled K-major and MN-major shared-memory
descriptors, TMEM accumulators) against a torch fp32 matmul."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_umma_selftest_matches_matmul():
    from specdec_b200 import _lib

    lib = _lib.load_library()
    g = torch.Generator().manual_seed(3)
    k, v = (torch.randn(128, 128, generator=g).to(torch.bfloat16) for _ in range(2))
    q, p = (torch.randn(32, 128, generator=g).to(torch.bfloat16) for _ in range(2))
    dk, dq, dv, dp = (t.cuda() for t in (k, q, v, p))
    o1 = torch.zeros(128, 32, device="cuda")
    o2 = torch.zeros(128, 32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.specdec_umma_selftest(dk.data_ptr(), dq.data_ptr(), dv.data_ptr(), dp.data_ptr(),
                                         o1.data_ptr(), o2.data_ptr(), st.data_ptr(), s), "umma_selftest")
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    torch.testing.assert_close(o1.cpu(), k.float() @ q.float().T, rtol=1e-5, atol=1e-3)
    torch.testing.assert_close(o2.cpu(), v.float().T @ p.float().T, rtol=1e-5, atol=1e-3)
