"""Test infrastructure only: numpy front-end of the parity oracle.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, and only as the checker.  The product (silarray_b200) never
imports it and has no CPU fallback.

Two libraries sit behind it:
  * ``liboracle.so``      -- oracle.c, the plain-C restatement of the reference
                             CPU backend (always built by oracle/Makefile);
  * ``_ref/libsilref.so`` -- the reference's own CPU path compiled from its
                             sources (ref_capi.cpp); present where the reference
                             was available at build time.  ``ref`` is None
                             when it is missing.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_szp = np.ctypeslib.ndpointer(np.uintp, flags="C_CONTIGUOUS")
_sz = C.c_size_t

OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4}


def build():
    """Compile the oracle (and the reference build where sources exist)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load(path):
    if not os.path.exists(path):
        return None
    return C.CDLL(path)


def _lib():
    lib = _load(os.path.join(_HERE, "liboracle.so"))
    if lib is None:
        build()
        lib = _load(os.path.join(_HERE, "liboracle.so"))
    sig = {
        "orc_binary_f32": [C.c_int, _f32p, _sz, _f32p, _sz, _f32p, _sz],
        "orc_binary_i32": [C.c_int, _i32p, _sz, _i32p, _sz, _i32p, _sz],
        "orc_scalar_op_f32": [C.c_int, C.c_float, C.c_int, _f32p, _f32p, _sz],
        "orc_sigmoid_f32": [_f32p, _f32p, _sz],
        "orc_relu_f32": [_f32p, _f32p, _sz],
        "orc_sigmoid_backward_f32": [_f32p, _f32p, _f32p, _sz],
        "orc_bias_sigmoid_f32": [_f32p, _f32p, _sz, _sz],
        "orc_layer_norm_f32": [_f32p, _f32p, _f32p, _f32p, _sz, _sz, C.c_float],
        "orc_softmax_f32": [_f32p, _f32p, _sz, _sz],
        "orc_argmax_f32": [_f32p, _i32p, _sz, _sz],
        "orc_argmax_i32": [_i32p, _i32p, _sz, _sz],
        "orc_sum_f32": [_f32p, _sz],
        "orc_sum_i32": [_i32p, _sz],
        "orc_min_f32": [_f32p, _sz],
        "orc_max_f32": [_f32p, _sz],
        "orc_sum_axis_f32": [_f32p, _f32p, _sz, _sz, _sz],
        "orc_sum_axis_i32": [_i32p, _i32p, _sz, _sz, _sz],
        "orc_sgemm_rows": [C.c_void_p, C.c_void_p, _f32p, _sz, _sz, _sz, _sz,
                           _sz, C.c_int, C.c_int, _sz, _sz],
        "orc_dot_i32": [_i32p, _i32p, _i32p, _sz, _sz, _sz],
        "orc_conv2d_f32": [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz],
    }
    for name, args in sig.items():
        getattr(lib, name).argtypes = args
    lib.orc_sum_f32.restype = C.c_float
    lib.orc_min_f32.restype = C.c_float
    lib.orc_max_f32.restype = C.c_float
    lib.orc_sum_i32.restype = C.c_int32
    return lib


lib = _lib()


def _f(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _i(x):
    return np.ascontiguousarray(x, dtype=np.int32)


# ---------------------------------------------------------------- restatement
def binary(op, a, b, n=None):
    """out[i] = a[i % len(a)] op b[i % len(b)] (storage-length broadcasting)."""
    if a.dtype == np.int32:
        a, b = _i(a).ravel(), _i(b).ravel()
        n = n or max(a.size, b.size)
        out = np.empty(n, np.int32)
        lib.orc_binary_i32(OPS[op], a, a.size, b, b.size, out, n)
        return out
    a, b = _f(a).ravel(), _f(b).ravel()
    n = n or max(a.size, b.size)
    out = np.empty(n, np.float32)
    lib.orc_binary_f32(OPS[op], a, a.size, b, b.size, out, n)
    return out


def scalar_op(op, s, x, left=False):
    x = _f(x).ravel()
    out = np.empty_like(x)
    lib.orc_scalar_op_f32(OPS[op], float(s), int(left), x, out, x.size)
    return out


def sigmoid(x):
    x = _f(x)
    y = np.empty_like(x)
    lib.orc_sigmoid_f32(x.ravel(), y.ravel(), x.size)
    return y


def relu(x):
    x = _f(x)
    y = np.empty_like(x)
    lib.orc_relu_f32(x.ravel(), y.ravel(), x.size)
    return y


def sigmoid_backward(dout, x):
    dout, x = _f(dout), _f(x)
    y = np.empty_like(x)
    lib.orc_sigmoid_backward_f32(dout.ravel(), x.ravel(), y.ravel(), x.size)
    return y


def bias_sigmoid(x, bias):
    y = _f(x).copy()
    bias = _f(bias)
    lib.orc_bias_sigmoid_f32(y.ravel(), bias, y.size, bias.size)
    return y


def layer_norm(x, g, b, eps=1e-5):
    x = _f(x)
    y = np.empty_like(x)
    lib.orc_layer_norm_f32(x, y, _f(g), _f(b), x.shape[0], x.shape[1], eps)
    return y


def softmax(x):
    x = _f(x)
    y = np.empty_like(x)
    rows, cols = (1, x.size) if x.ndim == 1 else x.shape
    lib.orc_softmax_f32(x.ravel(), y.ravel(), rows, cols)
    return y


def argmax(x):
    rows, cols = x.shape
    idx = np.empty(rows, np.int32)
    if x.dtype == np.int32:
        lib.orc_argmax_i32(_i(x), idx, rows, cols)
    else:
        lib.orc_argmax_f32(_f(x), idx, rows, cols)
    return idx


def sum_all(x):
    if x.dtype == np.int32:
        return int(lib.orc_sum_i32(_i(x).ravel(), x.size))
    return np.float32(lib.orc_sum_f32(_f(x).ravel(), x.size))


def min_all(x):
    return np.float32(lib.orc_min_f32(_f(x).ravel(), x.size))


def max_all(x):
    return np.float32(lib.orc_max_f32(_f(x).ravel(), x.size))


def sum_axis(x, axis):
    shape = list(x.shape)
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    out_shape = shape[:axis] + shape[axis + 1:]
    if x.dtype == np.int32:
        y = np.empty(out_shape, np.int32)
        lib.orc_sum_axis_i32(_i(x).ravel(), y.ravel(), outer, shape[axis], inner)
    else:
        y = np.empty(out_shape, np.float32)
        lib.orc_sum_axis_f32(_f(x).ravel(), y.ravel(), outer, shape[axis], inner)
    return y


def sgemm(a, b, ta=False, tb=False, rows=None):
    """C = op(a) . op(b) in fp64-accumulate/fp32-round; a stored [K,M] when ta,
    b stored [N,K] when tb.  ``rows`` = (r0, r1) restricts to a row band."""
    a, b = _f(a), _f(b)
    M = a.shape[1] if ta else a.shape[0]
    K = a.shape[0] if ta else a.shape[1]
    N = b.shape[0] if tb else b.shape[1]
    r0, r1 = rows or (0, M)
    c = np.empty((r1 - r0, N), np.float32)
    lib.orc_sgemm_rows(a.ctypes.data, b.ctypes.data, c, M, N, K, a.shape[1],
                       b.shape[1], int(ta), int(tb), r0, r1)
    return c


def conv2d(x, w, rows=None):
    """x [N,H,W,C] NHWC, w [C_out,K,K,C] OHWI -> [N*H*W, C_out] (stride 1,
    padding K/2); ``rows`` = (m0, m1) restricts to a band of output pixels."""
    x, w = _f(x), _f(w)
    N, H, W, C = x.shape
    C_out, K = w.shape[0], w.shape[1]
    m0, m1 = rows or (0, N * H * W)
    out = np.empty((m1 - m0, C_out), np.float32)
    lib.orc_conv2d_f32(x.ravel(), w.ravel(), out, N, H, W, C, K, C_out, m0, m1)
    return out


def dot_i32(a, b):
    a, b = _i(a), _i(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), np.int32)
    lib.orc_dot_i32(a, b, c, M, N, K)
    return c


# ------------------------------------------------ the reference's own build
class _Ref:
    """The reference CPU path (oracle/_ref/libsilref.so)."""

    def __init__(self, dll):
        self.dll = dll
        dll.silref_last_error.restype = C.c_char_p
        for n in ["silref_binary_f32", "silref_dot_nd_f32", "silref_sum_axis_f32"]:
            getattr(dll, n).restype = C.c_int
        self.dll.silref_reduce_f32.argtypes = [C.c_int, _f32p, _sz, C.POINTER(C.c_float)]
        self.dll.silref_reduce_i32.argtypes = [C.c_int, _i32p, _sz, C.POINTER(C.c_int)]

    def _chk(self, rc):
        if rc:
            raise RuntimeError(self.dll.silref_last_error().decode())

    @staticmethod
    def _shape(x):
        return np.ascontiguousarray(x.shape, dtype=np.uintp)

    def binary(self, op, a, b):
        isint = a.dtype == np.int32
        conv = _i if isint else _f
        a, b = conv(a), conv(b)
        cap = max(a.size, b.size) * 4 + 16
        out = np.empty(cap, a.dtype)
        n = _sz()
        fn = self.dll.silref_binary_i32 if isint else self.dll.silref_binary_f32
        self._chk(fn(OPS[op], a.ctypes.data_as(C.c_void_p), self._shape(a).ctypes.data_as(C.c_void_p),
                     a.ndim, b.ctypes.data_as(C.c_void_p), self._shape(b).ctypes.data_as(C.c_void_p),
                     b.ndim, out.ctypes.data_as(C.c_void_p), _sz(cap), C.byref(n)))
        return out[: n.value]

    def scalar_chain(self, x, chain):
        x = _f(x).ravel()
        ops = np.array([OPS[o] for o, _, _ in chain], np.int32)
        sc = np.array([s for _, s, _ in chain], np.float32)
        left = np.array([int(lf) for _, _, lf in chain], np.int32)
        out = np.empty_like(x)
        self._chk(self.dll.silref_scalar_chain_f32(
            x.ctypes.data_as(C.c_void_p), _sz(x.size), ops.ctypes.data_as(C.c_void_p),
            sc.ctypes.data_as(C.c_void_p), left.ctypes.data_as(C.c_void_p),
            C.c_int(len(chain)), out.ctypes.data_as(C.c_void_p)))
        return out

    def unary(self, which, x):
        x = _f(x)
        y = np.empty_like(x)
        self._chk(self.dll.silref_unary_f32(C.c_int({"sigmoid": 0, "relu": 1}[which]),
                                            x.ctypes.data_as(C.c_void_p), _sz(x.size),
                                            y.ctypes.data_as(C.c_void_p)))
        return y

    def sigmoid_backward(self, s, dout):
        s, dout = _f(s), _f(dout)
        y = np.empty_like(s)
        self._chk(self.dll.silref_sigmoid_backward_f32(
            s.ctypes.data_as(C.c_void_p), dout.ctypes.data_as(C.c_void_p), _sz(s.size),
            y.ctypes.data_as(C.c_void_p)))
        return y

    def dot(self, a, b, ta=False, tb=False):
        a, b = _f(a), _f(b)
        M = a.shape[1] if ta else a.shape[0]
        K = a.shape[0] if ta else a.shape[1]
        N = b.shape[0] if tb else b.shape[1]
        c = np.empty((M, N), np.float32)
        self._chk(self.dll.silref_dot_f32(a.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p),
                                          c.ctypes.data_as(C.c_void_p), _sz(M), _sz(N), _sz(K),
                                          C.c_int(int(ta)), C.c_int(int(tb))))
        return c

    def dot_nd(self, a, b):
        a, b = _f(a), _f(b)
        cap = max(a.size, b.size) * max(a.size, b.size) + 16
        out = np.empty(cap, np.float32)
        n = _sz()
        self._chk(self.dll.silref_dot_nd_f32(
            a.ctypes.data_as(C.c_void_p), self._shape(a).ctypes.data_as(C.c_void_p), a.ndim,
            b.ctypes.data_as(C.c_void_p), self._shape(b).ctypes.data_as(C.c_void_p), b.ndim,
            out.ctypes.data_as(C.c_void_p), _sz(cap), C.byref(n)))
        return out[: n.value]

    def dot_i32(self, a, b):
        a, b = _i(a), _i(b)
        M, K = a.shape
        N = b.shape[1]
        c = np.empty((M, N), np.int32)
        self._chk(self.dll.silref_dot_i32(a.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p),
                                          c.ctypes.data_as(C.c_void_p), _sz(M), _sz(N), _sz(K)))
        return c

    def linear(self, x, w, b, sigmoid=False):
        x, w, b = _f(x), _f(w), _f(b)
        M, K = x.shape
        N = w.shape[1]
        y = np.empty((M, N), np.float32)
        self._chk(self.dll.silref_linear_f32(
            C.c_int(int(sigmoid)), x.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p),
            b.ctypes.data_as(C.c_void_p), _sz(b.size), y.ctypes.data_as(C.c_void_p),
            _sz(M), _sz(N), _sz(K)))
        return y

    def batched_dot(self, a, b):
        a, b = _f(a), _f(b)
        B, M, K = a.shape
        N = b.shape[2]
        c = np.empty((B, M, N), np.float32)
        self._chk(self.dll.silref_batched_dot_f32(
            a.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p), c.ctypes.data_as(C.c_void_p),
            _sz(B), _sz(M), _sz(N), _sz(K)))
        return c

    def softmax(self, x):
        x = _f(x)
        y = np.empty_like(x)
        if x.ndim == 1:
            self._chk(self.dll.silref_softmax1d_f32(x.ctypes.data_as(C.c_void_p),
                                                    y.ctypes.data_as(C.c_void_p), _sz(x.size)))
        else:
            self._chk(self.dll.silref_softmax_f32(x.ctypes.data_as(C.c_void_p),
                                                  y.ctypes.data_as(C.c_void_p),
                                                  _sz(x.shape[0]), _sz(x.shape[1])))
        return y

    def layer_norm(self, x, g, b, eps=1e-5):
        x, g, b = _f(x), _f(g), _f(b)
        y = np.empty_like(x)
        self._chk(self.dll.silref_layer_norm_f32(
            x.ctypes.data_as(C.c_void_p), g.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p),
            y.ctypes.data_as(C.c_void_p), _sz(x.shape[0]), _sz(x.shape[1]), C.c_float(eps)))
        return y

    def argmax(self, x):
        rows, cols = x.shape
        idx = np.empty(rows, np.int32)
        if x.dtype == np.int32:
            x = _i(x)
            fn = self.dll.silref_argmax_i32
        else:
            x = _f(x)
            fn = self.dll.silref_argmax_f32
        self._chk(fn(x.ctypes.data_as(C.c_void_p), idx.ctypes.data_as(C.c_void_p),
                     _sz(rows), _sz(cols)))
        return idx

    def sum_axis(self, x, axis):
        isint = x.dtype == np.int32
        x = _i(x) if isint else _f(x)
        cap = x.size + 16
        out = np.empty(cap, x.dtype)
        n = _sz()
        fn = self.dll.silref_sum_axis_i32 if isint else self.dll.silref_sum_axis_f32
        self._chk(fn(x.ctypes.data_as(C.c_void_p), self._shape(x).ctypes.data_as(C.c_void_p),
                     x.ndim, _sz(axis), out.ctypes.data_as(C.c_void_p), _sz(cap), C.byref(n)))
        shape = list(x.shape)
        del shape[axis]
        return out[: n.value].reshape(shape)

    def reduce(self, which, x):
        w = {"sum": 0, "min": 1, "max": 2}[which]
        if x.dtype == np.int32:
            r = C.c_int()
            self._chk(self.dll.silref_reduce_i32(w, _i(x).ravel(), x.size, C.byref(r)))
            return int(r.value)
        r = C.c_float()
        self._chk(self.dll.silref_reduce_f32(w, _f(x).ravel(), x.size, C.byref(r)))
        return np.float32(r.value)

    def transformer_block(self, x, batch, seq, d, heads, dff, p):
        out = np.empty((batch * seq, d), np.float32)
        args = [p[k] for k in ("g1", "be1", "wq", "bq", "wk", "bk", "wv", "bv",
                               "wo", "bo", "g2", "be2", "w1", "b1", "w2", "b2")]
        args = [_f(a) for a in args]
        x = _f(x)
        self._chk(self.dll.silref_transformer_block_f32(
            x.ctypes.data_as(C.c_void_p), _sz(batch), _sz(seq), _sz(d), _sz(heads), _sz(dff),
            *[a.ctypes.data_as(C.c_void_p) for a in args], out.ctypes.data_as(C.c_void_p)))
        return out


def _load_ref():
    path = os.path.join(_HERE, "_ref", "libsilref.so")
    if not os.path.exists(path):
        return None
    return _Ref(C.CDLL(path))


ref = _load_ref()
