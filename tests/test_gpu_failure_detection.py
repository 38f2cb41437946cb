"""GPU: bounded device waits report instead of hanging.

tinym_selftest_wait_timeout launches the kernel with fault injection on the
host side: its producer issues no copies, so nothing ever completes the
full barriers.  Each consumer wait runs out after a short limit, sets a bit
in the device error word, and the CTA releases its tensor memory and exits.
No GPU fault is raised; afterwards a normal GEMM on the same context must
still be correct.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ERR_BITS = 0x3F  # producer / MMA / epilogue / drain / consumer / reduction wait bits


def _operands(oracle, m, k, n, device):
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=11, dist="normal")
    x = torch.from_numpy(xq).to(device).view(torch.float8_e4m3fn)
    w = torch.from_numpy(wq).to(device).view(torch.float8_e4m3fn)
    return xq, wq, alpha, x, w


@pytest.mark.parametrize("kernel,split,m", [(1, 1, 9), (1, 2, 16), (2, 1, 1), (2, 3, 1)])
def test_wait_timeout_reports_and_context_survives(cuda_device, oracle, kernel, split, m):
    import torch

    import tinym_b200 as t

    k, n = 1024, 256
    xq, wq, alpha, x, w = _operands(oracle, m, k, n, cuda_device)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    assert t.device_status(clear=True) == 0
    plan = t.make_plan(kernel, split, 4, 16 if kernel == 1 else 0, 4 if kernel == 2 else 0)
    lib = t.capi()
    st = lib.tinym_selftest_wait_timeout(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k,
                                         plan, 2_000_000, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.tinym_last_error()
    flags = t.device_status(clear=True)
    assert flags != 0 and (flags & ~ERR_BITS) == 0, hex(flags)
    assert t.device_status(clear=True) == 0
    # the context is intact: a normal call is still exact to the oracle
    out = t.gemm(x, w, torch.from_numpy(alpha).to(cuda_device), plan=plan)
    torch.cuda.synchronize()
    ref = oracle.reference(xq, wq, alpha)
    assert oracle.max_rel_err(out.float().cpu().numpy(), ref) <= 4e-3
    assert t.device_status() == 0


def test_selftest_rejects_bad_timeout(cuda_device):
    import tinym_b200 as t

    lib = t.capi()
    assert lib.tinym_selftest_wait_timeout(16, 16, 16, 1, 128, 128, None, 0, None) == 1
    assert lib.tinym_selftest_wait_timeout(16, 16, 16, 1, 128, 128, None, 10**11, None) == 1


def test_timeout_raises_at_next_drop_in_call(cuda_device, oracle):
    """A GEMM whose bounded wait ran out left its output unspecified.  The
    kernel also posts its error bits to the device's pinned pending-error
    word, so the next call through the drop-in API (candidate_kernel.fp8_gemm)
    raises RuntimeError without any synchronisation by the caller; the call
    after that runs normally and is exact to the oracle again."""
    import torch

    import candidate_kernel
    import tinym_b200 as t

    m, k, n = 9, 1024, 256
    xq, wq, alpha, x, w = _operands(oracle, m, k, n, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    candidate_kernel.build()
    candidate_kernel.fp8_gemm(x, w, a)  # the device's first GEMM creates its pending-error word
    torch.cuda.synchronize()
    assert t.device_status(clear=True) == 0
    assert t.pending_errors() == 0
    y = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    lib = t.capi()
    st = lib.tinym_selftest_wait_timeout(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, None,
                                         2_000_000, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.tinym_last_error()
    torch.cuda.synchronize()  # the timed-out kernel has finished; the caller does not read Y
    with pytest.raises(RuntimeError, match="TINYM_ERR_DEVICE_TIMEOUT"):
        candidate_kernel.fp8_gemm(x, w, a)
    out = candidate_kernel.fp8_gemm(x, w, a)
    torch.cuda.synchronize()
    ref = oracle.reference(xq, wq, alpha)
    assert oracle.max_rel_err(out.float().cpu().numpy(), ref) <= 4e-3
    assert oracle.mismatches(out.float().cpu().numpy(), ref) == 0
    # the synchronising status still holds the self-test's bits in the device word
    assert t.device_status(clear=True) & ERR_BITS
    assert t.device_status() == 0 and t.pending_errors() == 0
