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


def test_tma_gather4_page_rows():
    """Four-row tensor gathers (one-row boxes) fetch exactly the requested 2048-byte and
    64-byte rows: the page-row loads of the attention kernel."""
    import ctypes

    from specdec_b200 import _lib

    lib = _lib.load_library()
    n = 1000
    g = torch.Generator().manual_seed(3)
    big = torch.randint(0, 256, (n, 2048), generator=g, dtype=torch.uint8).cuda()
    small = torch.randint(0, 256, (n, 64), generator=g, dtype=torch.uint8).cuda()
    for rows in ([7, 0, 999, 7], [500, 501, 2, 3]):
        out = torch.zeros(8192 + 256, dtype=torch.uint8, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        r = (ctypes.c_int32 * 4)(*rows)
        rc = lib.specdec_gather4_selftest(big.data_ptr(), small.data_ptr(), n, ctypes.cast(r, ctypes.c_void_p),
                                          out.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, _lib.status_message(rc) if hasattr(_lib, "status_message") else rc
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(out[:8192].view(4, 2048).cpu(), big[rows].cpu())
        assert torch.equal(out[8192:].view(4, 64).cpu(), small[rows].cpu())


@pytest.mark.parametrize("mode,n_ctas,grid,expect_timeout", [(0, 0, 1, True), (1, 3, 2, True), (1, 2, 2, False)])
def test_bounded_waits_give_up_and_report(mode, n_ctas, grid, expect_timeout):
    """The timeout path every device wait of the library relies on, with a 1 ms limit:
    an mbarrier that nothing arrives on, and the grid barrier expecting more CTAs than the
    grid has, raise SPECDEC_STATUS_TIMEOUT and return (after about the limit, well before
    the default one-second limit); a grid barrier whose CTAs all arrive passes."""
    from specdec_b200 import _lib

    lib = _lib.load_library()
    counter = torch.zeros(1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    limit = 1_000_000
    _lib.check(lib.specdec_wait_selftest(mode, counter.data_ptr(), n_ctas, grid, limit, status.data_ptr(),
                                         waited.data_ptr(), torch.cuda.current_stream().cuda_stream), "wait_selftest")
    torch.cuda.synchronize()
    st, ns = int(status.item()), int(waited.item())
    if expect_timeout:
        assert st == _lib.STATUS_TIMEOUT
        assert limit <= ns < 100 * limit
    else:
        assert st == 0 and ns < limit
    # the context is still usable
    assert float(torch.ones(4, device="cuda").sum()) == 4.0

