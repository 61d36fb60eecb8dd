"""The bounded waits of the tensor-core kernels give up instead of hanging.

tau_dxb_selftest_wait_timeout runs one CTA whose threads wait on an mbarrier
phase that nothing completes, with a short host-chosen limit instead of the
kernels' 2 s. The wait must give up, set its bit in the device error word and
raise the CTA's abort flag, and the CTA must free its tensor memory and
return; the context then still runs work. Nothing faults or traps: the wait
is on a flag that nothing sets.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_context_stays_usable():
    from tau_dxb_b200 import _capi as C
    from tau_dxb_b200 import wta as W
    lib = C.lib()
    torch.cuda.init()
    assert lib.tau_dxb_device_error(1) in (0, C.DEVERR_SELFTEST)     # start clean
    for limit_ms in (1, 20):
        status = ctypes.c_int32(-1)
        t0 = time.perf_counter()
        rc = lib.tau_dxb_selftest_wait_timeout(limit_ms * 10 ** 6, ctypes.byref(status), C.stream_ptr())
        elapsed = time.perf_counter() - t0
        C.check("tau_dxb_selftest_wait_timeout", rc)
        assert status.value == 2, status.value          # gave up (bit 1), never "completed" (bit 0)
        assert lib.tau_dxb_device_error(1) == C.DEVERR_SELFTEST
        assert lib.tau_dxb_device_error(0) == 0           # the reset cleared it
        assert elapsed >= limit_ms * 1e-3 and elapsed < 2.0, elapsed
    # the context still runs kernels correctly
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(64, 3072, device="cuda", generator=g).to(torch.bfloat16)
    y, bits = W.wta_select(x, 306, W.THRESHOLD)
    thr = x.float().kthvalue(3072 - 306 + 1, dim=-1, keepdim=True).values
    assert torch.equal(W.unpack_mask(bits, 3072), x.float() >= thr)
