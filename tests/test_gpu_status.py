"""GPU check of the failure-detection path: the bounded mbarrier wait that
every kernel uses gives up after its limit, reports GDN_STATUS_WAIT_TIMEOUT
through the device status word, and leaves the context usable.

The wait that runs out is on an mbarrier phase that nothing completes (no
fault, no trap): gdn_b200_selftest_wait through the C ABI."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 0x1  # GDN_STATUS_WAIT_TIMEOUT


def _selftest(timeout_us: int):
    from gdn_b200 import _capi, ops
    res = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    rc = _capi.lib.gdn_b200_selftest_wait(timeout_us, ctypes.c_void_p(res.data_ptr()),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _capi.lib.gdn_b200_error_string(rc)
    status = ops.device_status(clear=True)
    return [int(x) for x in res.cpu()], status


@pytest.mark.parametrize("timeout_us", [1000, 20000])
def test_bounded_wait_gives_up_and_reports(cuda, timeout_us):
    from gdn_b200 import ops
    assert ops.device_status(clear=True) == 0
    (done, stuck, waited_us), status = _selftest(timeout_us)
    assert done == 1            # the completed phase is seen at once
    assert stuck == 0           # the phase nothing completes times out
    assert status & WAIT_TIMEOUT
    assert timeout_us <= waited_us <= timeout_us + 50000, waited_us
    assert ops.device_status(clear=True) == 0  # cleared by the read above


def test_context_usable_after_timeout(cuda):
    from gdn_b200 import NVFP4StatePool, ops, workloads
    _selftest(1000)
    HK, HV, D, B = 16, 32, 128, 2
    pool = NVFP4StatePool.zeros(2, HV, D, "cuda")
    pool.load_fp32(workloads.initial_states(2, HV, D, seed=1).cuda())
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=0, device="cuda")
    slot = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    o = ops.decode(x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, pool)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    assert ops.device_status(clear=True) == 0


def test_selftest_argument_errors(cuda):
    from gdn_b200 import _capi
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert _capi.lib.gdn_b200_selftest_wait(0, ctypes.c_void_p(res.data_ptr()), s) != 0
    assert _capi.lib.gdn_b200_selftest_wait(3000000, ctypes.c_void_p(res.data_ptr()), s) != 0
    assert _capi.lib.gdn_b200_selftest_wait(1000, None, s) != 0
