"""Reductions and row ops on the GPU vs the oracle.

Bit-exact: argmax indices (first index of the maximum, FLT_MIN floor of the
CPU branch), int sums, min/max.  fp32 sums: |g - s64| <= 1e-5 * sum|x|
against an fp64 sum (the oracle's own sequential fp32 sum drifts by more
than that at these lengths).  softmax / layer_norm: rel 1e-5 / abs 1e-6
against the oracle, and against an fp64 recomputation."""
import numpy as np
import pytest
import torch

import oracle as O
from silarray_b200 import gpu
from tests._tol import assert_close, assert_sum_close

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("n", [1, 3, 1000, 4097, 1 << 22, (1 << 24) + 5])
def test_whole_array_reductions(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    t = dev(x)
    assert_sum_close(host(gpu.sum_f32(t)), x, what="sum")
    assert host(gpu.min_f32(t)) == x.min()
    assert host(gpu.max_f32(t)) == x.max()
    idx, val = gpu.argmax_all_f32(t)
    i = int(host(idx))
    ref = O.argmax(x.reshape(1, -1))[0]
    assert i == ref and host(val) == x[ref]


def test_argmax_all_ties_and_floor(cuda):
    x = np.zeros(1 << 20, np.float32)
    x[777] = 5.0
    x[555] = 5.0
    x[999999] = 5.0
    idx, _ = gpu.argmax_all_f32(dev(x))
    assert int(host(idx)) == 555
    neg = -np.ones(1 << 16, np.float32)
    idx, _ = gpu.argmax_all_f32(dev(neg))
    assert int(host(idx)) == 0  # nothing above FLT_MIN: the CPU branch returns 0


def test_sum_i32_wraps(cuda):
    rng = np.random.default_rng(1)
    x = rng.integers(-2 ** 31, 2 ** 31 - 1, 1 << 20, dtype=np.int64).astype(np.int32)
    assert int(host(gpu.sum_i32(dev(x)))) == O.sum_all(x)


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 3), (64, 300), (33, 128), (4, 1000), (17, 1024),
                                       (8, 2048), (8, 4096), (8, 8192), (4, 16384), (3, 32768),
                                       (2, 40000), (2, 40001), (1000, 8192), (700, 16384), (600, 32768),
                                       (301, 8256)])
def test_row_ops(cuda, rows, cols):
    """Row ops against the oracle.  Rows up to 4096 columns run from
    registers (a warp or a CTA per row); softmax / layer_norm / argmax on
    rows of 4K-32K columns (multiples of 64) run one CTA per row (up to 8192)
    or one 2-CTA cluster per row from shared memory; the row sum keeps the row
    in registers across a 4-CTA cluster; other widths take the generic loop."""
    _check_row_ops(rows, cols)


def _check_row_ops(rows, cols):
    rng = np.random.default_rng(rows * 100003 + cols)
    x = rng.normal(0, 2, (rows, cols)).astype(np.float32)
    X = dev(x)
    sm = host(gpu.softmax(X))
    # the oracle divides by a sequential fp32 sum, whose own error grows
    # ~sqrt(cols) * 2^-24; beyond 4096 columns allow for it
    assert_close(sm, O.softmax(x), rel=1e-5 if cols <= 4096 else 3e-5, abs_=1e-6, what="softmax vs oracle")
    x64 = x.astype(np.float64)
    e = np.exp(x64 - x64.max(1, keepdims=True))
    assert_close(sm, e / e.sum(1, keepdims=True), rel=1e-5, abs_=1e-7, what="softmax vs fp64")
    g = rng.normal(1, 0.1, cols).astype(np.float32)
    b = rng.normal(0, 0.1, cols).astype(np.float32)
    ln = host(gpu.layer_norm(X, gamma=dev(g), beta=dev(b)))
    assert_close(ln, O.layer_norm(x, g, b), rel=1e-5, abs_=2e-6 if cols > 1 else 1e-6, what="layer_norm")
    np.testing.assert_array_equal(host(gpu.argmax_f32(X)), O.argmax(x))
    s1 = host(gpu.sum_axis_f32(X, rows, cols, 1))
    for r in range(rows):
        assert_sum_close(s1[r], x[r], what=f"sum(axis=1) row {r}")
    s0 = host(gpu.sum_axis0_f32(X))
    for c in range(0, cols, max(1, cols // 50)):
        assert_sum_close(s0[c], x[:, c], what=f"sum(axis=0) col {c}")


_VARIANT_SHAPES = [(3, 8256), (5, 16384), (3, 32768), (600, 32768)]


def run_row_variant(env):
    """Runs the long-row cases in a fresh process (the implementation
    switches are read once per process) with `env` set; used by the test
    below and as a script: python -m tests.test_gpu_reduce VAR=VALUE."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path.insert(0, %r); from tests import test_gpu_reduce as T; "
            "[T._check_row_ops(r, c) for r, c in T._VARIANT_SHAPES]; print('variant ok')" % root)
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env}, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "variant ok" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


@pytest.mark.parametrize("env", [{"SILCU_ROW_SMEM_CL": "4"}, {"SILCU_ROW_IMPL": "0"}, {"SILCU_ROW_IMPL": "1"}],
                         ids=["smem-cluster4", "register-rows", "smem-rowsum"])
def test_row_ops_other_implementations(cuda, env):
    """The row-op variants the defaults do not select: the 4-CTA shared-memory
    cluster above 8K columns, the register-resident long-row kernels
    (clusters of 4) for every op, and the shared-memory row sum."""
    run_row_variant(env)


def test_argmax_ties_and_floor_rows(cuda):
    S = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "seeded.npz"))
    np.testing.assert_array_equal(host(gpu.argmax_f32(dev(S["argmax_ties_x"]))), S["argmax_ties"])
    np.testing.assert_array_equal(host(gpu.argmax_f32(dev(S["argmax_neg_x"]))), S["argmax_neg"])


def test_argmax_split_rows(cuda):
    """Few very long rows take the split path (workspace + finish kernel)."""
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (2, 1 << 22)).astype(np.float32)
    x[1, 12345] = 100.0
    x[1, 4000000] = 100.0
    got = host(gpu.argmax_f32(dev(x)))
    np.testing.assert_array_equal(got, O.argmax(x))


def test_golden_rows(cuda):
    S = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "seeded.npz"))
    X = dev(S["rows_x"])
    assert_close(host(gpu.softmax(X)), S["softmax"], what="softmax golden")
    assert_close(host(gpu.layer_norm(X, gamma=dev(S["ln_g"]), beta=dev(S["ln_b"]))), S["layer_norm"],
                 rel=1e-5, abs_=2e-6, what="layer_norm golden")
    assert_close(host(gpu.sum_axis_f32(X, 64, 300, 1)), S["sum_axis1"], rel=1e-4, abs_=1e-4, what="sum1")
    assert_close(host(gpu.sum_axis0_f32(X)), S["sum_axis0"], rel=1e-4, abs_=1e-4, what="sum0")


@pytest.mark.parametrize("shape,axis", [((3, 2, 3), 0), ((3, 2, 3), 1), ((3, 2, 3), 2),
                                        ((7, 500, 33), 1), ((4096, 1024), 0), ((2, 9000, 5), 1)])
def test_sum_axis_nd(cuda, shape, axis):
    rng = np.random.default_rng(len(shape) + axis)
    x = rng.normal(0, 1, shape).astype(np.float32)
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    got = host(gpu.sum_axis_f32(dev(x.ravel()), outer, shape[axis], inner)).reshape(
        shape[:axis] + shape[axis + 1:])
    ref = x.astype(np.float64).sum(axis)
    lim = 1e-5 * np.abs(x.astype(np.float64)).sum(axis) + 1e-6
    assert (np.abs(got - ref) <= lim).all()


def test_layer_norm_known_answer(cuda):
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    out = host(gpu.layer_norm(dev(x), gamma=dev(np.ones(3, np.float32)), beta=dev(np.zeros(3, np.float32))))
    np.testing.assert_allclose(out, [[-1.2247, 0, 1.2247]] * 2, atol=1e-3)


def test_softmax_known_answer(cuda):
    x = np.array([[1, 2, 3]], np.float32)
    np.testing.assert_allclose(host(gpu.softmax(dev(x))), [[0.0900, 0.2447, 0.6652]], atol=1e-3)


@pytest.mark.parametrize("n", [1, 6, 1000, 4096])
def test_small_sum_is_sequential_fp32(cuda, n):
    """Up to 4096 elements the sum is the reference's sequential fp32 sum, bit for bit."""
    x = np.random.default_rng(n).uniform(-1, 1, n).astype(np.float32)
    assert host(gpu.sum_f32(dev(x))) == O.sum_all(x)


@pytest.mark.parametrize("shape,axis", [((7, 300, 33), 0), ((7, 300, 33), 1), ((7, 300, 33), 2),
                                        ((4096, 1024), 1), ((3, 5), 1), ((2, 1001), 1),
                                        # rows through the warp-per-32-rows kernel: a partial
                                        # warp of rows, a partial last tile, one short tile
                                        ((33, 36), 1), ((100, 8192), 1), ((5, 4), 1), ((70, 1000), 1)])
def test_sum_axis_sequential_bit_exact(cuda, shape, axis):
    """silcu_sum_axis_seq_f32 adds in the reference CPU loop's order
    (include/array.h:2303-2317): bit-identical to the oracle's restatement."""
    rng = np.random.default_rng(sum(shape) + axis)
    x = rng.normal(0, 1, shape).astype(np.float32)
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    got = host(gpu.sum_axis_seq_f32(dev(x.ravel()), outer, shape[axis], inner))
    np.testing.assert_array_equal(got, O.sum_axis(x, axis).ravel())
