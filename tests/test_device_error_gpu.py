"""Device-side failure reporting on the B200, without faulting the GPU.

Every wait in the kernels is bounded; a wait that gives up sets the library's
device error word, stops and returns.  These tests make a bounded wait run
out on purpose through ``cast_selftest_bounded_wait`` (one CTA waiting on an
mbarrier arrival that nothing makes, with a 20 ms limit), check that the
status reaches Python as ``CastError`` through the wrappers' check, and that
the context is still usable afterwards."""

import numpy as np
import pytest
import torch

from cast_b200 import _lib, rcsa
from oracle import rcsa as orc

pytestmark = pytest.mark.gpu
TIMEOUT = 6  # CAST_ERR_DEVICE_TIMEOUT


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_bounded_wait_completes_when_the_arrival_comes(cuda):
    lib = _lib.load()
    assert lib.cast_device_error(_stream()) == 0
    _lib.call("cast_selftest_bounded_wait", 1, 20000, _stream())
    _lib.check_device(_stream(), "selftest")


def test_bounded_wait_gives_up_and_reports(cuda):
    lib = _lib.load()
    assert lib.cast_device_error(_stream()) == 0
    _lib.call("cast_selftest_bounded_wait", 0, 20000, _stream())
    with pytest.raises(_lib.CastError) as exc:
        _lib.check_device(_stream(), "selftest")
    assert exc.value.status == TIMEOUT and "DEVICE_TIMEOUT" in str(exc.value)
    # the word was read and cleared: the next check passes
    _lib.check_device(_stream(), "selftest")


def test_plan_check_raises_then_context_is_usable(cuda):
    """A plan's check reports a device error set before it, and the next
    call runs normally and matches the oracle."""
    g = torch.Generator().manual_seed(5)
    block, nq, nh, budget = 128, 2, 3, 2
    q = torch.randn(1, 2, nq * block, 128, generator=g).bfloat16()
    k = torch.randn(1, 2, (nq + nh) * block, 128, generator=g).bfloat16()
    v = torch.randn(1, 2, (nq + nh) * block, 128, generator=g).bfloat16()
    plan = rcsa.RCSAPlan(1, 2, q.shape[2], k.shape[2], 128, block_size=block, budget=budget,
                         policy="bf16", device=cuda)
    _lib.call("cast_selftest_bounded_wait", 0, 20000, _stream())
    with pytest.raises(_lib.CastError) as exc:
        plan.check()
    assert exc.value.status == TIMEOUT
    out = plan(q.to(cuda), k.to(cuda), v.to(cuda))
    plan.check()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    sel, cnt, _, _, _ = orc.rcsa_select(qn, kn, block, budget)
    np.testing.assert_array_equal(plan.indices.cpu().numpy(), sel)
    ref = orc.block_sparse_attention(qn, kn, vn, sel, cnt, block, block)
    assert float(np.abs(out.float().cpu().numpy() - ref).max()) < 2e-2


def test_selftest_rejects_bad_limits(cuda):
    lib = _lib.load()
    assert lib.cast_selftest_bounded_wait(0, 0, None) == 1
    assert lib.cast_selftest_bounded_wait(0, 2000000, None) == 1
