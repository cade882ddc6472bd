"""The device error channel, exercised without a GPU fault: a kernel whose
bounded wait can never complete (an mbarrier nothing arrives on) gives up after
its time limit, records a code and returns; the host reads it through
vla_sync_check() and the context stays usable afterwards."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_device_timeout(cuda):
    from vla_b200 import _lib
    lib = _lib.load()
    _lib.check(lib.vla_sync_check())  # start from a clear error word
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.vla_test_expired_wait(1000, stream))  # 1 ms limit
    code = ctypes.c_uint(0)
    torch.cuda.synchronize()
    _lib.check(lib.vla_peek_device_error(ctypes.byref(code)))
    assert code.value == 0x1FF
    assert lib.vla_sync_check() == _lib.VLA_E_DEVICE_TIMEOUT
    assert "0x1ff" in _lib.last_error()
    # the word was cleared and the context still runs kernels correctly
    _lib.check(lib.vla_sync_check())
    x = torch.randn(64, 960, device="cuda").to(torch.bfloat16)
    g = torch.ones(960, dtype=torch.bfloat16, device="cuda")
    from vla_b200 import device as dev
    y = dev.rms_norm(x, g, 1e-5)
    ref = torch.nn.functional.rms_norm(x.float(), (960,), g.float(), 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=2e-2, rtol=2e-2)
    _lib.check(lib.vla_sync_check())
