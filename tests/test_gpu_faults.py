"""Failure detection without a GPU fault: a readiness flag that nothing sets makes the
kernel's bounded wait run out; the kernel reports the error in its status words, returns,
and the context stays usable (a reset and the next run are correct).  The two-phase kernel
waits on hidden row-block readiness (status 2); the hidden-slice decode kernel (cfg3) on the
other clusters' partials of its Y rows (status 3)."""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import prepare_ffn
from ffn_optim_b200 import cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case_id", ["cfg1_fp16", "cfg3_bf16"])
def test_dependency_wait_times_out_and_recovers(case_id):
    case = C.get_case(case_id)
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared = prepare_ffn(x, w1, w2, down_impl="basic")
    good = prepared.run().clone()
    prepared.check()
    prepared.set_wait_limit(0.2)
    prepared.set_fault_injection(1)
    prepared.run()
    status = prepared.status()
    hslice = prepared.plan.kernel["variant"] == 12
    # FFN_B200_KERNEL_DEP_TIMEOUT, or FFN_B200_KERNEL_SK_TIMEOUT for the hidden-slice reduction
    assert status[0] == (3 if hslice else 2), status
    with pytest.raises(RuntimeError, match="partial wait timed out" if hslice else "readiness wait timed out"):
        prepared.check()  # also resets counters, flags and status
    prepared.set_fault_injection(0)
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    assert torch.equal(y, good)
    torch.cuda.synchronize()
    assert np.isfinite(y.float().cpu().numpy()).all()


def test_dynamic_claims_without_reset_report_and_recover():
    """A launch that aborted leaves the tile-claim counter short of its epoch base; a next
    launch without the reset rejects its out-of-range claims (status 5, or a timeout in the
    CTAs that wait behind them) instead of using them as tile coordinates, and a reset
    restores correct results."""
    m, k, h, n = 8192, 512, 2048, 1024
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).bfloat16().cuda()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).bfloat16().cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).bfloat16().cuda()
    prepared = prepare_ffn(x, w1, w2, schedule="dynamic")
    good = prepared.run().clone()
    prepared.check()
    prepared.set_wait_limit(0.2)
    prepared.set_fault_injection(1)
    prepared.run()
    torch.cuda.synchronize()
    assert prepared.status()[0] == 2
    prepared.set_fault_injection(0)
    prepared.run()  # no reset in between
    torch.cuda.synchronize()
    assert prepared.status()[0] != 0
    prepared.reset()
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    assert torch.equal(y, good)
