"""Pins the parity oracle (CPU only, no GPU).

1. The C restatement (oracle/oracle.c) reproduces every known-answer case of
   the reference test suite (tests/golden/known_answers.json) bit for bit
   against the reference CPU build's outputs recorded there, and within the
   reference test's own abs 1e-3 of the values the reference asserts.
2. Where the reference build is present (oracle/_ref/libsilref.so), the
   restatement equals it bit for bit on seeded inputs (dot within fp32
   rounding: cblas' summation order is not the restatement's fp64 one).
3. Where the reference sources are present, the reference's own doctest suite
   passes on the oracle build.
"""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))["cases"]
SEED = np.load(os.path.join(HERE, "golden", "seeded.npz"))


def _arr(spec):
    return np.array(spec["data"], dtype=spec["dtype"]).reshape(spec["shape"])


def _restate(c):
    ins = {k: _arr(v) for k, v in c["inputs"].items()}
    op = c["op"]
    if op in ("add", "sub", "mul", "div", "pow"):
        a, b = ins["a"], ins["b"]
        if a.shape != b.shape and a.ndim == b.ndim and a.ndim == 2 and a.size > 1 and b.size > 1:
            # both-sided broadcast: the reference materialises both operands
            # (include/array.h:2500-2517) before the storage-length loop
            shape = np.broadcast_shapes(a.shape, b.shape)
            a, b = np.broadcast_to(a, shape).copy(), np.broadcast_to(b, shape).copy()
        return O.binary(op, a, b)
    if op == "scalar":
        return O.scalar_op(c["scalar_op"], c["scalar"], ins["x"], left=c["left"])
    if op == "dot_i32":
        return O.dot_i32(ins["a"], ins["b"])
    if op == "dot":
        return O.sgemm(ins["a"], ins["b"])
    if op == "dot_t":
        a, b = ins["a"], ins["b"]
        if c["ta"]:
            return O.sgemm(a, b, ta=True)
        return O.sgemm(a, b, tb=True)
    if op == "dot_nd":
        a, b = ins["a"], ins["b"]
        a2 = a.reshape(1, -1) if a.ndim == 1 else a
        b2 = b.reshape(-1, 1) if b.ndim == 1 else b
        return O.sgemm(a2, b2)
    if op == "linear":
        d = O.sgemm(ins["x"], ins["W"])
        return O.binary("add", d, ins["b"])
    if op == "sigmoid":
        return O.sigmoid(ins["x"])
    if op == "relu":
        return O.relu(ins["x"])
    if op == "sum_axis":
        return O.sum_axis(ins["x"], c["axis"])
    if op == "sum":
        return np.array([O.sum_all(ins["x"])])
    if op == "min":
        x = ins["x"]
        return np.array([x.min()])
    if op == "max":
        x = ins["x"]
        return np.array([x.max()])
    if op == "layer_norm":
        return O.layer_norm(ins["x"], ins["g"], ins["b"])
    if op == "softmax":
        return O.softmax(ins["x"])
    if op == "argmax":
        return O.argmax(ins["x"])
    raise KeyError(op)


@pytest.mark.parametrize("c", GOLD, ids=[c["name"] for c in GOLD])
def test_restatement_matches_reference_known_answers(c):
    got = np.asarray(_restate(c)).ravel()
    ref = np.array(c["ref"], dtype=c["ref_dtype"])
    if c["op"] in ("dot", "dot_t", "dot_nd", "linear"):
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(got.astype(ref.dtype), ref)
    if c.get("expect") is not None:
        np.testing.assert_allclose(ref.astype(np.float64), np.array(c["expect"], np.float64), atol=1e-3)
    for k, v in (c.get("expect_points") or {}).items():
        assert abs(float(ref[int(k)]) - v) <= 1e-3


def test_restatement_matches_seeded_fixtures():
    S = SEED
    X = S["rows_x"]
    np.testing.assert_array_equal(O.softmax(X), S["softmax"])
    np.testing.assert_array_equal(O.layer_norm(X, S["ln_g"], S["ln_b"]), S["layer_norm"])
    np.testing.assert_array_equal(O.argmax(S["argmax_ties_x"]), S["argmax_ties"])
    np.testing.assert_array_equal(O.argmax(S["argmax_neg_x"]), S["argmax_neg"])
    assert (S["argmax_neg"] == 0).all()
    np.testing.assert_array_equal(O.sum_axis(X, 1), S["sum_axis1"])
    np.testing.assert_array_equal(O.sum_axis(X, 0), S["sum_axis0"])
    np.testing.assert_allclose(O.sgemm(S["dot_a"], S["dot_b"]), S["dot"], rtol=1e-6, atol=1e-6)
    for op in ("add", "sub", "mul", "div"):
        np.testing.assert_array_equal(O.binary(op, S["ew_a"], S["ew_b"]), S[f"ew_{op}"])
    np.testing.assert_array_equal(O.binary("pow", np.abs(S["ew_a"]), S["ew_b"]), S["ew_pow"])
    np.testing.assert_array_equal(O.sigmoid(S["ew_a"]), S["sigmoid"])
    np.testing.assert_array_equal(O.relu(S["ew_a"]), S["relu"])
    np.testing.assert_array_equal(O.sigmoid_backward(S["ew_b"], S["ew_a"]), S["sigmoid_backward"])
    lin = O.binary("add", O.sgemm(S["dot_a"], S["dot_b"]), S["lin_b"]).reshape(70, 40)
    np.testing.assert_allclose(lin, S["linear"], rtol=1e-6, atol=1e-6)
    ls = O.bias_sigmoid(O.sgemm(S["dot_a"], S["dot_b"]), S["lin_b"])
    np.testing.assert_allclose(ls, S["linear_sigmoid"], rtol=1e-6, atol=1e-6)


@pytest.mark.skipif(O.ref is None, reason="reference CPU build not present")
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_restatement_equals_reference_build(seed):
    R = O.ref
    rng = np.random.default_rng(seed)
    rows, cols = int(rng.integers(1, 40)), int(rng.integers(1, 700))
    X = rng.normal(0, 2, (rows, cols)).astype(np.float32)
    np.testing.assert_array_equal(O.softmax(X), R.softmax(X))
    g = rng.normal(1, .1, cols).astype(np.float32)
    b = rng.normal(0, .1, cols).astype(np.float32)
    np.testing.assert_array_equal(O.layer_norm(X, g, b), R.layer_norm(X, g, b))
    np.testing.assert_array_equal(O.argmax(X), R.argmax(X))
    np.testing.assert_array_equal(O.sum_axis(X, 1), R.sum_axis(X, 1))
    np.testing.assert_array_equal(O.sum_axis(X, 0), R.sum_axis(X, 0))
    assert O.sum_all(X) == R.reduce("sum", X)
    assert O.min_all(X) == R.reduce("min", X)
    assert O.max_all(X) == R.reduce("max", X)
    # storage-length broadcasting (row vector); a length-1 operand is folded
    # into the affine pass by the lazy evaluator (x / s becomes x * (1/s))
    for op in ("add", "sub", "mul", "div"):
        np.testing.assert_array_equal(O.binary(op, X, X[0]), R.binary(op, X, X[0]))
        s1 = X[:1, :1].ravel()
        np.testing.assert_array_equal(O.scalar_op(op, s1[0], X).reshape(-1), R.binary(op, X, s1))
    # scalar chains on either side, including the 5e6 NEON threshold path
    for op in ("add", "sub", "mul", "div"):
        for left in (False, True):
            s = float(rng.normal()) + 3.0
            np.testing.assert_array_equal(O.scalar_op(op, s, X, left=left), R.scalar_chain(X, [(op, s, left)]))
    I = rng.integers(-1000, 1000, (rows, cols)).astype(np.int32)
    np.testing.assert_array_equal(O.sum_axis(I, 1), R.sum_axis(I, 1))
    assert O.sum_all(I) == R.reduce("sum", I)
    A = rng.uniform(-1, 1, (rows, 33)).astype(np.float32)
    B = rng.uniform(-1, 1, (33, 21)).astype(np.float32)
    np.testing.assert_allclose(O.sgemm(A, B), R.dot(A, B), rtol=2e-6, atol=2e-6)


@pytest.mark.skipif(O.ref is None, reason="reference CPU build not present")
def test_affine_fold_large_path_uses_fma():
    """n >= 5e6 takes cpu::affine (NEON fmaf); smaller n the vDSP branches."""
    R = O.ref
    x = np.random.default_rng(7).normal(0, 1, 5_000_000).astype(np.float32)
    np.testing.assert_array_equal(O.scalar_op("sub", 1.5, x, left=True), R.scalar_chain(x, [("sub", 1.5, True)]))


REF = os.environ.get("SILARRAY_REF", "/root/reference")


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "test", "test_array.cpp")),
                    reason="reference sources not present (set SILARRAY_REF)")
def test_reference_doctest_suite_passes_on_oracle_build():
    root = os.path.dirname(HERE)
    r = subprocess.run(["make", "-s", "-C", os.path.join(root, "oracle"), f"REF={REF}", "check-ref"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "Status: SUCCESS" in r.stdout
