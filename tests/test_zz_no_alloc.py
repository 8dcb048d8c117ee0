"""silcu_sum_f32_noalloc: the whole-array sum for callers that cannot
allocate device memory (allocator callbacks, plugins whose host forbids
cudaMalloc).  Called through the C ABI and compared with silcu_sum_f32 and
with an fp64 sum (|g - s64| <= 1e-5 * sum|x|), on two calls in a row so that
the shared built-in scratch is reused.  Collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

from silarray_b200 import _lib
from tests._tol import assert_sum_close

pytestmark = pytest.mark.gpu


def test_noalloc_sum_matches_workspace_sum(cuda):
    lib = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws_bytes = lib.silcu_reduce_workspace_bytes(1 << 24)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    for n, seed in ((1 << 24, 0), (100003, 1)):
        x = np.random.default_rng(seed).uniform(-1, 1, n).astype(np.float32)
        t = torch.from_numpy(x).cuda()
        a = torch.empty((), dtype=torch.float32, device="cuda")
        b = torch.empty((), dtype=torch.float32, device="cuda")
        _lib.check(lib.silcu_sum_f32_noalloc(C.c_void_p(t.data_ptr()), n, C.c_void_p(a.data_ptr()), stream))
        _lib.check(lib.silcu_sum_f32(C.c_void_p(t.data_ptr()), n, C.c_void_p(b.data_ptr()),
                                     C.c_void_p(ws.data_ptr()), ws_bytes, stream))
        torch.cuda.synchronize()
        assert_sum_close(a.item(), x, what="noalloc sum")
        assert_sum_close(b.item(), x, what="workspace sum")
        assert abs(a.item() - b.item()) <= 1e-5 * float(np.abs(x).sum())
