"""The failure path of the bounded waits, exercised without a fault.

Every spin wait in the kernels gives up after a wall-clock limit, records a code
in the device status word and returns, so the context stays usable. Here the
normalisation is launched by its self-test entry point, which waits for one
arrival more than it launches: nothing ever supplies it, so the wait runs out
after a shortened limit (50 ms). The test checks that the kernel returned, that
the status reads the normalisation's code, that the output is NaN (the failure
is visible downstream), that the next call succeeds, and that the opt-in status
check of the public API raises.
"""

from __future__ import annotations

import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, _native, ops

pytestmark = pytest.mark.gpu

NORMALIZE_TIMEOUT = 4  # status code of the normalisation's arrival wait


def _selftest(device, batch=2, rows=64, cols=48):
    lib = _native.load()
    x = torch.randn((batch, rows, cols), device=device)
    out = torch.zeros((batch, rows, cols), dtype=torch.float16, device=device)
    ws = torch.empty(lib.gns_normalize_workspace_size(batch, rows, cols), dtype=torch.uint8, device=device)
    rc = lib.gns_selftest_normalize_timeout(batch, rows, cols, x.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                            ws.numel(), _native.stream_handle(device))
    _native.check(rc, "gns_selftest_normalize_timeout")
    return out


@pytest.fixture
def short_wait_limit(cuda_device):
    previous = _native.set_wait_limit_ns(50_000_000)
    yield
    _native.set_wait_limit_ns(previous)
    _native.device_status(clear=True)


def test_expired_wait_reports_status_and_poisons_output(cuda_device, short_wait_limit):
    assert _native.device_status(clear=True) == 0
    out = _selftest(cuda_device)
    torch.cuda.synchronize(cuda_device)
    assert _native.device_status(clear=True) == NORMALIZE_TIMEOUT
    assert torch.isnan(out).all()
    # the context is still usable: the next call computes a valid result
    x = torch.randn((2, 64, 192), device=cuda_device).bfloat16()
    y = GramNewtonSchulz()(x)
    torch.cuda.synchronize(cuda_device)
    assert _native.device_status(clear=True) == 0
    assert torch.isfinite(y).all()


def test_opt_in_status_check_raises(cuda_device, short_wait_limit):
    x = torch.randn((2, 64, 192), device=cuda_device).bfloat16()
    previous = ops.set_status_checks(True)
    try:
        GramNewtonSchulz()(x)  # nothing pending: passes
        _selftest(cuda_device)
        with pytest.raises(ops.DeviceWaitError, match="status 4"):
            GramNewtonSchulz()(x)
        # the check cleared the word: the next call passes
        GramNewtonSchulz()(x)
    finally:
        ops.set_status_checks(previous)


def test_wait_limit_bounds():
    with pytest.raises(_native.NativeError, match="between"):
        _native.set_wait_limit_ns(10)
