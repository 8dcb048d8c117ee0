"""Failure path of the bounded device waits, made to happen without faulting
the GPU: silcu_check_bounded_wait runs the tensor-core kernels' wait on a
barrier that nothing arrives at, with a short limit; the wait gives up,
records its code, and the kernel returns.  silcu_device_status then reports
SILCU_TIMEOUT once (reading clears it), and the context keeps working."""
import ctypes as C

import numpy as np
import pytest
import torch

from silarray_b200 import _lib, gpu

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_device_recovers(cuda):
    lib = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.silcu_device_status(stream) == 0  # nothing pending
    assert lib.silcu_check_bounded_wait(2000, stream) == 0  # 2 ms limit
    assert lib.silcu_synchronize(stream) == 0
    assert lib.silcu_device_status(stream) == 3  # SILCU_TIMEOUT
    assert b"code 77" in lib.silcu_last_error()
    assert lib.silcu_device_status(stream) == 0  # read once, cleared
    x = torch.randn(64, 512, device="cuda")
    got = gpu.softmax(x).cpu().numpy()
    x64 = x.cpu().numpy().astype(np.float64)
    e = np.exp(x64 - x64.max(1, keepdims=True))
    np.testing.assert_allclose(got, e / e.sum(1, keepdims=True), rtol=1e-5, atol=1e-7)
    gpu.device_status()
    assert lib.silcu_check_bounded_wait(0, stream) == 1  # limit outside 1..1e6 us: rejected, nothing launched
