"""Split-output producers (softmax / layer_norm / weight split) write the exact
tf32 split of the plain result: hi = tf32_rna(y), hi + lo == y bit for bit."""
import numpy as np
import pytest
import torch

from silarray_b200 import gpu

pytestmark = pytest.mark.gpu


def _split(x):
    u = x.view(np.uint32).astype(np.uint64)
    hi = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)
    return hi, (x - hi).astype(np.float32)


@pytest.mark.parametrize("rows,cols", [(64, 512), (7, 1000), (3, 8192), (2, 40001)])
def test_row_split_outputs(cuda, rows, cols):
    rng = np.random.default_rng(cols)
    x = torch.from_numpy(rng.normal(0, 2, (rows, cols)).astype(np.float32)).cuda()
    g = torch.from_numpy(rng.normal(1, .1, cols).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.normal(0, .1, cols).astype(np.float32)).cuda()
    for plain, (hi, lo) in ((gpu.softmax(x), gpu.softmax_split(x, rows, cols)),
                            (gpu.layer_norm(x, gamma=g, beta=b), gpu.layer_norm_split(x, g, b, rows, cols))):
        torch.cuda.synchronize()
        y = plain.cpu().numpy().ravel()
        eh, el = _split(y)
        np.testing.assert_array_equal(hi.cpu().numpy().ravel(), eh)
        np.testing.assert_array_equal(lo.cpu().numpy().ravel(), el)


def test_weight_split_transposed(cuda):
    w = np.random.default_rng(1).normal(0, .02, (96, 200)).astype(np.float32)
    hi, lo = gpu.split(torch.from_numpy(w).cuda(), 96, 200, transpose=True)
    torch.cuda.synchronize()
    eh, el = _split(np.ascontiguousarray(w.T))
    np.testing.assert_array_equal(hi.cpu().numpy().reshape(200, 96), eh)
    np.testing.assert_array_equal(lo.cpu().numpy().reshape(200, 96), el)
