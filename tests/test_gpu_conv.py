"""conv2d (silcu_conv2d_f32: GEMM on the 3xTF32 tensor-core path, its A tiles
im2col TMA boxes of the split input when C_in % 16 == 0, else a split patch matrix)
against the oracle restatement of the reference's conv2d arithmetic
(oracle.c: orc_conv2d_f32; the reference has no CPU conv2d) and, for odd
kernels, an fp64 torch convolution as an independent check.  NHWC input,
OHWI weight, stride 1, padding K/2.  Tolerance: |g - r| <= sqrt(K_dim) *
(1e-6 + 1e-5 |r|) with K_dim = K*K*C_in, the dot-product bound."""
import numpy as np
import pytest
import torch

import oracle as O
from silarray_b200 import gpu
from tests._tol import assert_dot_close

pytestmark = pytest.mark.gpu


def _torch_ref(x, w):
    K = w.shape[1]
    t = torch.nn.functional.conv2d(torch.from_numpy(x).double().permute(0, 3, 1, 2),
                                   torch.from_numpy(w).double().permute(0, 3, 1, 2), padding=K // 2)
    return t.permute(0, 2, 3, 1).reshape(-1, w.shape[0]).numpy()


@pytest.mark.parametrize("N,C_in,C_out,H,W,K", [
    (2, 5, 7, 9, 9, 3),      # odd channels: scalar patch loads, plain patch matrix, CUDA-core GEMM
    (1, 3, 32, 224, 224, 3),  # the reference benchmark's ImageNet first layer (C_in = 3)
    (2, 8, 12, 7, 7, 5),     # K = 5
    (2, 16, 32, 10, 12, 1),  # K = 1 (a per-pixel GEMM)
    (2, 16, 32, 10, 12, 2),  # even K: padding 1 before, 0 after
    (16, 64, 128, 56, 56, 3),  # the reference benchmark's ResNet mid layer
    # C_in % 16 == 0: the im2col TMA path (no patch matrix)
    (3, 16, 64, 7, 9, 3),    # M = 189: a partial row tile, tiles that span images
    (2, 32, 256, 12, 10, 5),  # K = 5 (padding 2), 256-column tiles
    (1, 128, 64, 16, 16, 3),  # M = 256, K_dim = 1152: split K
    (2, 48, 36, 11, 13, 4),  # even K = 4 (padding 2 before, 1 after), C_out % 32 != 0
])
def test_conv2d_matches_oracle(cuda, N, C_in, C_out, H, W, K):
    rng = np.random.default_rng(N * 1000 + C_in * 10 + K)
    x = rng.normal(0, 1, (N, H, W, C_in)).astype(np.float32)
    w = rng.normal(0, 1.0 / np.sqrt(K * K * C_in), (C_out, K, K, C_in)).astype(np.float32)
    got = gpu.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    got = got.cpu().numpy().reshape(-1, C_out)
    M = N * H * W
    bands = [(0, min(M, 300))] if M > 4000 else [(0, M)]
    if M > 4000:
        bands += [(M // 2, M // 2 + 200), (M - 300, M)]
    Kd = K * K * C_in
    for m0, m1 in bands:
        ref = O.conv2d(x, w, rows=(m0, m1))
        assert_dot_close(got[m0:m1], ref, Kd, what=f"conv2d rows {m0}:{m1}")
    if K % 2 == 1 and M <= 60000:
        assert_dot_close(got, _torch_ref(x, w), Kd, what="conv2d vs fp64 torch")
    again = gpu.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()).cpu().numpy().reshape(-1, C_out)
    np.testing.assert_array_equal(got, again)
    gpu.device_status()
