"""Bounded device waits (failure handling without a GPU fault).

The reference's one failure mechanism is its OOM chunk retry (utils/dispatcher.py:244-293); this
library sizes its workspace up front instead, and every mbarrier wait of its GEMM pipelines is
bounded: a wait that runs out flags ORDA_ERR_TIMEOUT in the caller's status word and the kernel
returns. The testing hook below makes such a wait run out on purpose (an mbarrier that nothing
arrives at, with a limit of microseconds) and checks the status word, the time waited, and that the
context still runs the fused loss afterwards.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

ok = pytest.importorskip("orda_ce_kernel")
from orda_ce_kernel import TiedTeacher, _native, distillation_loss  # noqa: E402


@pytest.mark.parametrize("limit_ns", [20_000, 2_000_000])
def test_wait_that_nobody_completes_times_out_and_returns(limit_ns):
    lib = _native.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(lib.orda_debug_wait_timeout(status.data_ptr(), limit_ns, waited.data_ptr(), stream),
                  "orda_debug_wait_timeout")
    torch.cuda.synchronize()
    assert int(status.item()) == _native.ERR_TIMEOUT
    w = int(waited.item())
    assert limit_ns <= w < limit_ns + 50_000_000, w  # gave up after the limit, not much later


def test_wait_gives_up_at_once_when_the_status_is_already_flagged():
    """A role of the same launch that already flagged an error makes the other waits give up
    without waiting for their own limit (the pipelines unwind together)."""
    lib = _native.load()
    status = torch.full((1,), _native.ERR_TIMEOUT, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    _native.check(lib.orda_debug_wait_timeout(status.data_ptr(), 1_000_000_000, waited.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream), "orda_debug_wait_timeout")
    torch.cuda.synchronize()
    assert int(status.item()) == _native.ERR_TIMEOUT
    assert int(waited.item()) < 100_000_000


def test_invalid_limits_are_rejected_without_launching():
    lib = _native.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.orda_debug_wait_timeout(status.data_ptr(), 0, waited.data_ptr(), s) == _native.ERR_INVALID_ARGUMENT
    assert lib.orda_debug_wait_timeout(status.data_ptr(), 3_000_000_000, waited.data_ptr(), s) == \
        _native.ERR_INVALID_ARGUMENT
    assert lib.orda_debug_wait_timeout(None, 1000, waited.data_ptr(), s) == _native.ERR_INVALID_ARGUMENT


def test_context_is_usable_after_a_timeout():
    from oracle.distill_oracle import distill_reference

    lib = _native.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    _native.check(lib.orda_debug_wait_timeout(status.data_ptr(), 50_000, waited.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream), "orda_debug_wait_timeout")
    g = torch.Generator().manual_seed(7)
    hs = torch.randn(130, 64, generator=g).to(torch.bfloat16)
    ht = torch.randn(130, 64, generator=g).to(torch.bfloat16)
    w = (torch.randn(700, 64, generator=g) * 0.1).to(torch.bfloat16)
    labels = torch.randint(0, 700, (130,), generator=g)
    hs_d = hs.cuda().requires_grad_(True)
    out = distillation_loss(hs_d, w.cuda(), labels.cuda(), TiedTeacher(ht.cuda()), kl_weight=0.5)
    out.loss.backward()
    torch.cuda.synchronize()
    assert int(status.item()) == _native.ERR_TIMEOUT
    ref = distill_reference(hs.double().numpy(), w.double().numpy(), labels.numpy(), mode="tied",
                            teacher_hidden=ht.double().numpy(), kl_weight=0.5)
    assert float(out.loss) == pytest.approx(ref.loss, rel=1e-3)
