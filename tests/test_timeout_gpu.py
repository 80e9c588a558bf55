"""The timeout path of the device-side bounded waits: every wait of the library's kernels on
an mbarrier or a flag gives up after a wall-clock limit, raises G4_DEVERR_TIMEOUT with the
waiting site, and the kernel winds down.  g4_selftest_wait_timeout makes one such wait run
out (an mbarrier that nothing completes): nothing faults or hangs, the host reads the status,
and the context keeps working."""
import ctypes as C
import importlib
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

L = importlib.import_module("gemma4-js_b200._lib")


def test_bounded_wait_times_out_and_context_recovers(rt, ctx, g4):
    ctx.check_device()  # clean before
    t0 = time.monotonic()
    L.call("g4_selftest_wait_timeout", ctx.handle, 0x1234)
    with pytest.raises(g4.G4Error) as ei:
        ctx.check_device()
    elapsed = time.monotonic() - t0
    assert ei.value.status == -4  # G4_ERR_TIMEOUT
    assert "wait site 4660" in str(ei.value)  # 0x1234
    assert 1.0 < elapsed < 30.0
    ctx.check_device()  # the word was cleared; the context is usable
    x = torch.arange(16, dtype=torch.float32, device="cuda")
    y = torch.empty_like(x)
    L.call("g4_scale", ctx.handle, C.c_void_p(x.data_ptr()), 16, C.c_float(2.0), C.c_void_p(y.data_ptr()))
    ctx.check_device()
    assert torch.equal(y, x * 2)
