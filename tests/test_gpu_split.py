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


@pytest.mark.parametrize("B,H,S,D,pair", [(2, 3, 512, 64, True), (1, 2, 100, 64, True), (2, 2, 64, 48, True),
                                          (1, 2, 96, 64, False)])
def test_transpose_split_heads(cuda, B, H, S, D, pair):
    """V [B, S, H*D] (a row of all heads per token) -> per-head V^T [D, S]
    split hi/lo, from a split pair (value = hi + lo) or a plain array: bit
    equal to the split of the transposed value."""
    rng = np.random.default_rng(S + D)
    ld = H * D + 8  # padded row, as a column slice of a wider matrix
    v = rng.normal(0, 1, (B, S, ld)).astype(np.float32)
    vh, vl = _split(v)
    src, src_lo = (torch.from_numpy(vh).cuda(), torch.from_numpy(vl).cuda()) if pair else \
        (torch.from_numpy(v).cuda(), None)
    hi = torch.empty(B * H * D * S, device="cuda")
    lo = torch.empty(B * H * D * S, device="cuda")
    gpu.transpose_split(src.reshape(-1), S, D, ld, batch=B, heads=H, s_b=S * ld, s_h=D,
                        src_lo=None if src_lo is None else src_lo.reshape(-1), out=(hi, lo))
    torch.cuda.synchronize()
    want = np.stack([v[b, :, h * D:(h + 1) * D].T for b in range(B) for h in range(H)])
    wh, wl = _split(np.ascontiguousarray(want))
    np.testing.assert_array_equal(hi.cpu().numpy().reshape(want.shape), wh)
    np.testing.assert_array_equal(lo.cpu().numpy().reshape(want.shape), wl)
