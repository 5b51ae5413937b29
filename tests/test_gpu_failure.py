"""Failure detection on the GPU without a fault: a kernel whose wait can never
complete gives up after a short limit and reports through the status word;
the context stays usable afterwards."""

import ctypes as C

import pytest
import torch

from tiktok_techjam_2026_track3_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.ttj_selftest_wait_timeout(status.data_ptr(), 20000, stream) == 0  # 20 ms
    code = C.c_int(0)
    rc = lib.ttj_read_status(status.data_ptr(), C.byref(code), stream)
    assert rc == -5 and code.value == 6  # TTJ_ERR_DEVICE_TIMEOUT, kDevTimeoutInjected
    assert b"bounded wait" in lib.ttj_last_error()
    # the context is still healthy: a real op runs and the shared status word is clean
    x = torch.randn(128, 256, device=dev, dtype=torch.float16)
    w = torch.randn(256, 256, device=dev, dtype=torch.float16) * 0.05
    b = torch.zeros(256, device=dev, dtype=torch.float16)
    y = ops.linear(x, w, b)
    torch.testing.assert_close(y.float(), x.float() @ w.float().T, rtol=2e-2, atol=2e-2)
    ops.check_device_status(dev)
