"""Generates tests/golden/*.json / *.npz from the reference's own CPU build.

Run here (where the reference sources exist and oracle/_ref/libsilref.so was
built by `make -C oracle`):  python tests/golden/make_golden.py

known_answers.json  the reference test suite's known-answer cases
                    (test/test_array.cpp, cited per case): inputs, the values
                    the reference test asserts (checked there at abs 1e-3),
                    and the exact output of the reference CPU build.
seeded.npz          seeded synthetic inputs at parity-test sizes with the
                    reference CPU build's outputs.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

R = oracle.ref
assert R is not None, "oracle/_ref/libsilref.so is missing: run `make -C oracle` first"


def f32(x):
    return np.asarray(x, np.float32)


def tolist(x):
    return np.asarray(x).ravel().tolist()


cases = []


def case(name, cite, op, inputs, expect, got, **kw):
    cases.append({"name": name, "cite": cite, "op": op,
                  "inputs": {k: {"shape": list(np.shape(v)), "dtype": str(np.asarray(v).dtype),
                                 "data": tolist(v)} for k, v in inputs.items()},
                  "expect": tolist(expect) if expect is not None else None,
                  "ref": tolist(got), "ref_dtype": str(np.asarray(got).dtype), **kw})


# test/test_array.cpp:95-126 vector arithmetic
a = f32([7.82637e-06, 0.131538, 0.755605, 0.45865, 0.532767, 0.218959, 0.0470446, 0.678865,
         0.679296, 0.934693, 0.383502, 0.519416, 0.830965, 0.0345721, 0.0534616, 0.5297])
b = f32([0.671149, 0.00769819, 0.383416, 0.0668422, 0.417486, 0.686773, 0.588977, 0.930436,
         0.846167, 0.526929, 0.0919649, 0.653919, 0.415999, 0.701191, 0.910321, 0.762198])
exp = {
    "add": [0.671157, 0.139236, 1.13902, 0.525492, 0.950253, 0.905732, 0.636021, 1.6093, 1.52546,
            1.46162, 0.475467, 1.17334, 1.24696, 0.735763, 0.963782, 1.2919],
    "sub": [-0.671141, 0.12384, 0.372189, 0.391808, 0.115281, -0.467814, -0.541932, -0.251571,
            -0.166871, 0.407764, 0.291537, -0.134503, 0.414966, -0.666619, -0.856859, -0.232498],
    "mul": [5.25266e-06, 0.0010126, 0.289711, 0.0306572, 0.222423, 0.150375, 0.0277082, 0.63164,
            0.574798, 0.492517, 0.0352687, 0.339656, 0.345681, 0.0242416, 0.0486672, 0.403736],
    "div": [1.16612e-05, 17.0869, 1.97072, 6.86168, 1.27613, 0.318823, 0.0798751, 0.72962,
            0.802792, 1.77385, 4.17009, 0.794312, 1.99752, 0.0493048, 0.0587283, 0.694964],
}
for op, e in exp.items():
    case(f"vector_{op}", "test/test_array.cpp:95-126", op, {"a": a, "b": b}, e, R.binary(op, a, b))

# test/test_array.cpp:135-148 pow
ia, ib = np.array([1, 2, 3], np.int32), np.array([2, 2, 2], np.int32)
case("pow_int_ab", "test/test_array.cpp:137-139", "pow", {"a": ia, "b": ib}, [1, 4, 9], R.binary("pow", ia, ib))
case("pow_int_ba", "test/test_array.cpp:140", "pow", {"a": ib, "b": ia}, [2, 4, 8], R.binary("pow", ib, ia))
fa, fb = f32([1, 2, 3]), f32([2, 2, 2])
case("pow_float_ab", "test/test_array.cpp:143-145", "pow", {"a": fa, "b": fb}, [1, 4, 9], R.binary("pow", fa, fb))
case("pow_float_ba", "test/test_array.cpp:146", "pow", {"a": fb, "b": fa}, [2, 4, 8], R.binary("pow", fb, fa))

# test/test_array.cpp:210-220 scalar operations (affine folding)
m = f32([[1, 2], [3, 4]])
for op, s, left, e in [("add", 1, False, [2, 3, 4, 5]), ("sub", 1, False, [0, 1, 2, 3]),
                       ("mul", 2, False, [2, 4, 6, 8]), ("div", 2, False, [0.5, 1, 1.5, 2]),
                       ("add", 1, True, [2, 3, 4, 5]), ("sub", 1, True, [0, -1, -2, -3]),
                       ("mul", 2, True, [2, 4, 6, 8]), ("div", 2, True, [2, 1, 2.0 / 3.0, 0.5])]:
    case(f"scalar_{'l' if left else 'r'}{op}", "test/test_array.cpp:210-220", "scalar",
         {"x": m}, e, R.scalar_chain(m, [(op, float(s), left)]), scalar=float(s), left=left, scalar_op=op)

# test/test_array.cpp:222-260 dot (int and float)
ai = np.arange(1, 13, dtype=np.int32).reshape(3, 4)
bi = np.arange(1, 9, dtype=np.int32).reshape(4, 2)
case("dot_mm_int", "test/test_array.cpp:230-236", "dot_i32", {"a": ai, "b": bi},
     [50, 60, 114, 140, 178, 220], R.dot_i32(ai, bi))
af, bf = ai.astype(np.float32), bi.astype(np.float32)
case("dot_mm_float", "test/test_array.cpp:254-260", "dot", {"a": af, "b": bf},
     [50, 60, 114, 140, 178, 220], R.dot(af, bf))
v4 = np.arange(1, 5, dtype=np.float32)
case("dot_vv", "test/test_array.cpp:222-228", "dot_nd", {"a": v4, "b": v4}, [30], R.dot_nd(v4, v4))
case("dot_vm", "test/test_array.cpp:238-244", "dot_nd", {"a": v4, "b": bf}, [50, 60], R.dot_nd(v4, bf))
m24 = np.arange(1, 9, dtype=np.float32).reshape(2, 4)
case("dot_mv", "test/test_array.cpp:246-252", "dot_nd", {"a": m24, "b": v4}, [30, 70], R.dot_nd(m24, v4))

# test/test_array.cpp:262-277 linear
x = f32([[1, 2, 3], [4, 5, 6]])
W = f32([[1, 2], [3, 4], [5, 6]])
bb = f32([10, 20])
case("linear", "test/test_array.cpp:262-268", "linear", {"x": x, "W": W, "b": bb},
     [32, 48, 59, 84], R.linear(x, W, bb))

# test/test_array.cpp:279-317 sigmoid / relu
sv = f32([0, 1, -1, 5, -5])
case("sigmoid", "test/test_array.cpp:280-287", "sigmoid", {"x": sv}, None, R.unary("sigmoid", sv),
     expect_points={"0": 0.5, "1": 0.7310, "2": 0.2689})
rv = f32([-2, -1, 0, 1, 2])
case("relu", "test/test_array.cpp:305-311", "relu", {"x": rv}, [0, 0, 0, 1, 2], R.unary("relu", rv))

# test/test_array.cpp:319-334 dot with transpose (ones * 0.5)
ones43, ones42, w32 = np.ones((4, 3), np.float32), np.ones((4, 2), np.float32), np.full((3, 2), 0.5, np.float32)
case("dot_nt", "test/test_array.cpp:324-327", "dot_t", {"a": ones42, "b": w32}, [1.0] * 12,
     R.dot(ones42, w32, tb=True), ta=False, tb=True)
case("dot_tn", "test/test_array.cpp:329-332", "dot_t", {"a": ones43, "b": ones42}, [4.0] * 6,
     R.dot(ones43, ones42, ta=True), ta=True, tb=False)

# test/test_array.cpp:474-514 aggregates
t = np.arange(1, 19, dtype=np.int32).reshape(3, 2, 3)
for ax, e in [(0, [21, 24, 27, 30, 33, 36]), (1, [5, 7, 9, 17, 19, 21, 29, 31, 33]), (2, [6, 15, 24, 33, 42, 51])]:
    case(f"sum_axis{ax}_int", "test/test_array.cpp:493-495", "sum_axis", {"x": t}, e, R.sum_axis(t, ax), axis=ax)
    tf = t.astype(np.float32)
    case(f"sum_axis{ax}_float", "test/test_array.cpp:493-495", "sum_axis", {"x": tf}, e, R.sum_axis(tf, ax), axis=ax)
case("sum_int", "test/test_array.cpp:491-492", "sum", {"x": t}, [171], [R.reduce("sum", t)])
case("sum_float", "test/test_array.cpp:496", "sum", {"x": f32([1.1, 2.2])}, [3.3], [R.reduce("sum", f32([1.1, 2.2]))])
ones = np.ones(10000, np.float32)
case("sum_ones_10000", "test/test_array.cpp:500-501", "sum", {"x": ones}, [10000.0], [R.reduce("sum", ones)])
case("min_int", "test/test_array.cpp:486-489", "min", {"x": t}, [1], [R.reduce("min", t)])
case("max_int", "test/test_array.cpp:486-489", "max", {"x": t}, [18], [R.reduce("max", t)])

# test/test_array.cpp:516-547 layer_norm
xl = f32([[1, 2, 3], [4, 5, 6]])
case("layer_norm", "test/test_array.cpp:518-530", "layer_norm",
     {"x": xl, "g": f32([1, 1, 1]), "b": f32([0, 0, 0])}, [-1.2247, 0, 1.2247, -1.2247, 0, 1.2247],
     R.layer_norm(xl, f32([1, 1, 1]), f32([0, 0, 0])))
case("layer_norm_g2b1", "test/test_array.cpp:532-536", "layer_norm",
     {"x": xl, "g": f32([2, 2, 2]), "b": f32([1, 1, 1])}, None,
     R.layer_norm(xl, f32([2, 2, 2]), f32([1, 1, 1])), expect_points={"1": 1.0})

# test/test_array.cpp:549-576 softmax
sm = f32([1, 2, 3])
case("softmax_1d", "test/test_array.cpp:563-567", "softmax", {"x": sm}, [0.0900, 0.2447, 0.6652], R.softmax(sm))
ms = np.array([[7, 8, 9], [10, 11, 12]], np.float32)
case("softmax_2d", "test/test_array.cpp:550-558", "softmax", {"x": ms}, None, R.softmax(ms))

# test/test_array.cpp:626-630 argmax
am = np.array([[3, 1, 2], [6, 8, 7]], np.int32)
case("argmax_int", "test/test_array.cpp:626-630", "argmax", {"x": am}, [0, 1], R.argmax(am))
case("argmax_float", "test/test_array.cpp:626-630 (float input)", "argmax", {"x": am.astype(np.float32)},
     [0, 1], R.argmax(am.astype(np.float32)))

# test/test_array.cpp:643-706 raw backend add (storage-level)
case("msl_add_float", "test/test_array.cpp:643-662", "add", {"a": f32([1, 2, 3, 4]), "b": f32([10, 20, 30, 40])},
     [11, 22, 33, 44], R.binary("add", f32([1, 2, 3, 4]), f32([10, 20, 30, 40])))
case("msl_add_int", "test/test_array.cpp:664-684", "add",
     {"a": np.array([1, 2, 3, 4], np.int32), "b": np.array([10, 20, 30, 40], np.int32)}, [11, 22, 33, 44],
     R.binary("add", np.array([1, 2, 3, 4], np.int32), np.array([10, 20, 30, 40], np.int32)))
case("msl_add_float_broadcast", "test/test_array.cpp:686-706", "add", {"a": f32([1, 2, 3, 4]), "b": f32([10])},
     [11, 12, 13, 14], R.binary("add", f32([1, 2, 3, 4]), f32([10])))

# test/test_array.cpp:614-624 broadcast {3,1} + {1,3}
ba = np.array([[1], [2], [3]], np.int32)
bb2 = np.array([[10, 20, 30]], np.int32)
case("broadcast_both", "test/test_array.cpp:614-619", "add", {"a": ba, "b": bb2},
     [11, 21, 31, 12, 22, 32, 13, 23, 33], R.binary("add", ba, bb2))

with open(os.path.join(HERE, "known_answers.json"), "w") as f:
    json.dump({"generator": "tests/golden/make_golden.py", "cases": cases}, f, indent=1)

# ------------------------------------------------------------- seeded cases
rng = np.random.default_rng(20261201)
S = {}
X = rng.normal(0, 2, (64, 300)).astype(np.float32)
S["rows_x"] = X
S["softmax"] = R.softmax(X)
g = rng.normal(1, 0.1, 300).astype(np.float32)
be = rng.normal(0, 0.1, 300).astype(np.float32)
S["ln_g"], S["ln_b"] = g, be
S["layer_norm"] = R.layer_norm(X, g, be)
Xt = np.round(X).astype(np.float32)  # many ties
S["argmax_ties_x"] = Xt
S["argmax_ties"] = R.argmax(Xt)
S["argmax_neg_x"] = -np.abs(X) - 1.0  # no value above FLT_MIN: reference returns 0
S["argmax_neg"] = R.argmax(S["argmax_neg_x"])
S["sum_axis1"] = R.sum_axis(X, 1)
S["sum_axis0"] = R.sum_axis(X, 0)
A = rng.uniform(-1, 1, (70, 50)).astype(np.float32)
B = rng.uniform(-1, 1, (50, 40)).astype(np.float32)
S["dot_a"], S["dot_b"] = A, B
S["dot"] = R.dot(A, B)
bl = rng.normal(0, 0.01, 40).astype(np.float32)
S["lin_b"] = bl
S["linear"] = R.linear(A, B, bl)
S["linear_sigmoid"] = R.linear(A, B, bl, sigmoid=True)
Ab = rng.normal(0, 1, (3, 33, 20)).astype(np.float32)
Bb = rng.normal(0, 1, (3, 20, 17)).astype(np.float32)
S["bmm_a"], S["bmm_b"] = Ab, Bb
S["batched_dot"] = R.batched_dot(Ab, Bb)
E = rng.normal(0, 1, 1000).astype(np.float32)
F = rng.normal(0, 1, 1000).astype(np.float32)
S["ew_a"], S["ew_b"] = E, F
for op in ("add", "sub", "mul", "div"):
    S[f"ew_{op}"] = R.binary(op, E, F)
S["ew_pow"] = R.binary("pow", np.abs(E), F)
S["sigmoid"] = R.unary("sigmoid", E)
S["relu"] = R.unary("relu", E)
S["sigmoid_backward"] = R.sigmoid_backward(E, F)
np.savez_compressed(os.path.join(HERE, "seeded.npz"), **S)
print("wrote", len(cases), "known-answer cases and", len(S), "seeded arrays")
