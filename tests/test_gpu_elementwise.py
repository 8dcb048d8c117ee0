"""Elementwise parity on the GPU through the C ABI (silarray_b200.gpu is a thin
ctypes mirror of it) against the oracle: bit-exact for add/sub/mul/div/relu,
affine and int ops; rel 1e-5 / abs 1e-6 for pow/sigmoid (CUDA powf/expf
round differently from glibc)."""
import numpy as np
import pytest
import torch

import oracle as O
from silarray_b200 import gpu
from tests._tol import assert_close

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("n,lb", [(1, 1), (7, 7), (1000, 1000), (1001, 1001), (4096 * 33, 33),
                                  (4096 * 64, 64), (1 << 20, 1), (123457, 5)])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "pow"])
def test_binary_f32(cuda, op, n, lb):
    rng = np.random.default_rng(n + lb)
    a = rng.normal(0, 1, n).astype(np.float32)
    b = rng.normal(0, 1, lb).astype(np.float32)
    if op == "pow":
        a = np.abs(a) + 0.1
    got = host(getattr(gpu, op)(dev(a), dev(b)))
    ref = O.binary(op, a, b, n)
    if op == "pow":
        assert_close(got, ref, rel=2e-6, abs_=1e-30, what="pow")
    else:
        np.testing.assert_array_equal(got, ref)


def test_binary_broadcast_left_operand(cuda):
    rng = np.random.default_rng(3)
    a = rng.normal(0, 1, 96).astype(np.float32)
    b = rng.normal(0, 1, 96 * 50).astype(np.float32)
    for op in ("add", "sub", "mul", "div"):
        np.testing.assert_array_equal(host(getattr(gpu, op)(dev(a), dev(b))), O.binary(op, a, b))


def test_binary_unaligned_views(cuda):
    rng = np.random.default_rng(4)
    a = dev(rng.normal(0, 1, 1003).astype(np.float32))
    b = dev(rng.normal(0, 1, 1003).astype(np.float32))
    got = host(gpu.add(a[1:], b[2:1002]))
    np.testing.assert_array_equal(got, O.binary("add", a.cpu().numpy()[1:], b.cpu().numpy()[2:1002]))


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "pow"])
def test_binary_i32(cuda, op):
    rng = np.random.default_rng(11)
    n = 5000
    a = rng.integers(-2 ** 31, 2 ** 31 - 1, n, dtype=np.int64).astype(np.int32)
    b = rng.integers(-2 ** 31, 2 ** 31 - 1, n, dtype=np.int64).astype(np.int32)
    if op == "pow":
        a = rng.integers(-9, 10, n).astype(np.int32)
        b = rng.integers(0, 9, n).astype(np.int32)
    if op == "div":
        b[b == 0] = 3
    got = host(getattr(gpu, op)(dev(a), dev(b)))
    np.testing.assert_array_equal(got, O.binary(op, a, b))
    got = host(getattr(gpu, op)(dev(a), dev(b[:7])))
    np.testing.assert_array_equal(got, O.binary(op, a, b[:7]))


@pytest.mark.parametrize("n", [1, 5, 4096, 100003])
def test_unary(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 3, n).astype(np.float32)
    assert_close(host(gpu.sigmoid(dev(x))), O.sigmoid(x), what="sigmoid")
    np.testing.assert_array_equal(host(gpu.relu(dev(x))), O.relu(x))
    d = rng.normal(0, 1, n).astype(np.float32)
    assert_close(host(gpu.sigmoid_backward(dev(d), dev(x))), O.sigmoid_backward(d, x), rel=1e-5, abs_=1e-7,
                 what="sigmoid_backward")


def test_bias_sigmoid(cuda):
    rng = np.random.default_rng(9)
    x = rng.normal(0, 2, (37, 129)).astype(np.float32)
    b = rng.normal(0, 1, 129).astype(np.float32)
    t = dev(x.ravel())
    gpu.bias_sigmoid(t, dev(b))
    assert_close(host(t), O.bias_sigmoid(x, b).ravel(), what="bias_sigmoid")


@pytest.mark.parametrize("op,left", [("add", False), ("sub", False), ("mul", False), ("div", False),
                                     ("add", True), ("sub", True), ("mul", True)])
def test_affine_matches_scalar_fold(cuda, op, left):
    """The reference folds `x op s` into x*scale+offset (include/array.h:1888-1940);
    the host computes scale/offset the same way, the kernel applies them with
    the reference's rounding (two roundings below 5e6 elements, fmaf above)."""
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, 10007).astype(np.float32)
    s = np.float32(2.7)
    if not left:
        scale, offset = {"add": (1, s), "sub": (1, -s), "mul": (s, 0), "div": (np.float32(1) / s, 0)}[op]
    else:
        scale, offset = {"add": (1, s), "sub": (-1, s), "mul": (s, 0)}[op]
    got = host(gpu.affine(dev(x), scale=float(scale), offset=float(offset)))
    np.testing.assert_array_equal(got, O.scalar_op(op, s, x, left=left))
    # n >= 5e6: the reference applies the fold with fmaf (NEON, include/cpu.h:329-350)
    xl = rng.normal(0, 1, 5_000_000).astype(np.float32)
    got = host(gpu.affine(dev(xl), scale=float(scale), offset=float(offset), fused=True))
    np.testing.assert_array_equal(got, O.scalar_op(op, s, xl, left=left))


def test_fused_chain_equals_node_by_node(cuda):
    """((x + b_row) * 2 - y) / z, relu, as one fused kernel == per-node oracle."""
    rng = np.random.default_rng(21)
    rows, cols = 300, 257
    x = rng.normal(0, 1, rows * cols).astype(np.float32)
    y = rng.normal(0, 1, rows * cols).astype(np.float32)
    z = rng.normal(0, 1, rows * cols).astype(np.float32) + 3
    b = rng.normal(0, 1, cols).astype(np.float32)
    prog = [("load", 0, 0), ("load", 1, 1), ("add", 2, 0, 1), ("affine", 2, 2, 0, 2.0, 0.0),
            ("load", 3, 2), ("sub", 2, 2, 3), ("load", 4, 3), ("div", 2, 2, 4), ("relu", 5, 2)]
    got = host(gpu.fused(prog, [dev(x), dev(b), dev(y), dev(z)], rows * cols))
    r = O.binary("add", x, b)
    r = O.scalar_op("mul", 2.0, r)
    r = O.binary("sub", r, y)
    r = O.binary("div", r, z)
    r = O.relu(r)
    np.testing.assert_array_equal(got, r)


def test_known_answer_vectors(cuda):
    """test/test_array.cpp:95-126 and 643-706 through the GPU."""
    import json, os
    cases = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))["cases"]
    n = 0
    for c in cases:
        if c["op"] in ("add", "sub", "mul", "div") and c["name"] != "broadcast_both":
            a = np.array(c["inputs"]["a"]["data"], c["inputs"]["a"]["dtype"])
            b = np.array(c["inputs"]["b"]["data"], c["inputs"]["b"]["dtype"])
            got = host(getattr(gpu, c["op"])(dev(a), dev(b)))
            np.testing.assert_array_equal(got, np.array(c["ref"], c["ref_dtype"]))
            n += 1
    assert n >= 7
