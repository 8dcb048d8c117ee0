"""Host mirror of silarray's `class gpu` (include/gpu.h:266-1036) over libsilcu.

Each function keeps the reference's name and argument meaning; a `storage`
(shared buffer + element offset + length) is a CUDA torch tensor here, whose
data pointer already includes the offset and whose numel() is `len`.
Outputs are preallocated by the caller (as array.h does with make_uninit_)
or allocated here when omitted.  Work is queued on torch's current stream;
`synchronize()` replaces the reference's flush (include/gpu.h:1375-1377).

There is no CPU fallback: a CPU tensor or a missing library raises.
"""
import ctypes as ct

import torch

from . import _lib
from ._lib import check, lib

_F32 = torch.float32
_I32 = torch.int32


def _stream():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dev(t, dtype=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("silarray_b200.gpu: operands must be CUDA tensors (no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"silarray_b200.gpu: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError("silarray_b200.gpu: storage must be contiguous")
    return t


def _p(t):
    return ct.c_void_p(t.data_ptr()) if t is not None else ct.c_void_p(0)


# ------------------------------------------------------------------ workspace
_ws_cache = {}


def workspace(nbytes, device=None):
    """Per-device scratch buffer for multi-pass kernels (grown on demand).
    Kernels never allocate; this host-side cache is the only allocator."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    buf = _ws_cache.get(dev.index)
    if nbytes == 0:
        return buf if buf is not None else None
    if buf is None or buf.numel() < nbytes:
        size = max(int(nbytes * 1.25), 1 << 20)
        buf = torch.empty(size, dtype=torch.uint8, device=dev)
        _ws_cache[dev.index] = buf
    return buf


def _ws_args(nbytes, device):
    buf = workspace(nbytes, device)
    if buf is None:
        return ct.c_void_p(0), 0
    return ct.c_void_p(buf.data_ptr()), buf.numel()


def synchronize():
    check(lib().silcu_synchronize(_stream()))


def device_status():
    check(lib().silcu_device_status(_stream()))


# ---------------------------------------------------------------- elementwise
def _binary(op, A, B, OUT=None, n=None):
    dtype = A.dtype
    _dev(A, dtype), _dev(B, dtype)
    if n is None:
        n = OUT.numel() if OUT is not None else max(A.numel(), B.numel())
    if OUT is None:
        OUT = torch.empty(n, dtype=dtype, device=A.device)
    _dev(OUT, dtype)
    if OUT.numel() < n:
        raise ValueError("output storage too small")
    suffix = {_F32: "f32", _I32: "i32"}[dtype]
    fn = getattr(lib(), f"silcu_{op}_{suffix}")
    check(fn(_p(A), A.numel(), _p(B), B.numel(), _p(OUT), n, _stream()))
    return OUT


def add(A, B, OUT=None, n=None):
    return _binary("add", A, B, OUT, n)


def sub(A, B, OUT=None, n=None):
    return _binary("sub", A, B, OUT, n)


def mul(A, B, OUT=None, n=None):
    return _binary("mul", A, B, OUT, n)


def div(A, B, OUT=None, n=None):
    return _binary("div", A, B, OUT, n)


def pow(A, B, OUT=None, n=None):  # noqa: A001 - mirrors gpu::pow
    return _binary("pow", A, B, OUT, n)


def sigmoid(IN, OUT=None):
    _dev(IN, _F32)
    OUT = torch.empty_like(IN) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_sigmoid_f32(_p(IN), _p(OUT), IN.numel(), _stream()))
    return OUT


def relu(IN, OUT=None):
    _dev(IN, _F32)
    OUT = torch.empty_like(IN) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_relu_f32(_p(IN), _p(OUT), IN.numel(), _stream()))
    return OUT


def sigmoid_backward(dout, x, OUT=None):
    _dev(dout, _F32), _dev(x, _F32)
    OUT = torch.empty_like(x) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_sigmoid_backward_f32(_p(dout), _p(x), _p(OUT), x.numel(), _stream()))
    return OUT


def bias_sigmoid(data, bias, n=None, cols=None):
    _dev(data, _F32), _dev(bias, _F32)
    n = data.numel() if n is None else n
    cols = bias.numel() if cols is None else cols
    check(lib().silcu_bias_sigmoid_f32(_p(data), _p(bias), n, cols, _stream()))
    return data


def affine(IN, OUT=None, n=None, scale=1.0, offset=0.0, fused=False):
    _dev(IN, _F32)
    OUT = torch.empty_like(IN) if OUT is None else _dev(OUT, _F32)
    n = IN.numel() if n is None else n
    check(lib().silcu_affine_f32(_p(IN), _p(OUT), n, float(scale), float(offset), int(fused), _stream()))
    return OUT


OPCODES = {"load": 0, "add": 1, "sub": 2, "mul": 3, "div": 4, "pow": 5, "affine": 6,
           "affine_fma": 7, "sigmoid": 8, "relu": 9, "sigmoid_bwd": 10, "rdiv_imm": 11, "store": 12}


def _program(program, inputs):
    if len(program) > _lib.MAX_PROGRAM or len(inputs) > _lib.MAX_INPUTS:
        raise ValueError("program or input list too long")
    prog = _lib.Program()
    prog.n_instr = len(program)
    prog.n_inputs = len(inputs)
    for i, ins in enumerate(program):
        op, dst, a, b, imm0, imm1 = (list(ins) + [0, 0, 0.0, 0.0])[:6]
        prog.code[i] = _lib.Instr(OPCODES[op] if isinstance(op, str) else op, dst, a, b, imm0, imm1)
    for t in inputs:
        _dev(t, _F32)
    ptrs = (ct.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
    lens = (ct.c_size_t * max(1, len(inputs)))(*[t.numel() for t in inputs])
    return prog, ptrs, lens


def fused_multi(program, inputs, outputs, n):
    """A fused elementwise program with explicit ("store", 0, reg, k) writes
    into outputs[k] (each of n floats)."""
    prog, ptrs, lens = _program(program, inputs)
    for t in outputs:
        _dev(t, _F32)
    outs = (ct.c_void_p * max(1, len(outputs)))(*[t.data_ptr() for t in outputs])
    check(lib().silcu_fused_multi_f32(ct.byref(prog), ptrs, lens, outs, len(outputs), n, _stream()))
    return outputs


def fused(program, inputs, n, OUT=None):
    """Runs a fused elementwise program: `program` is a list of
    (op, dst, a, b, imm0, imm1) tuples; `inputs` CUDA float tensors."""
    prog, ptrs, lens = _program(program, inputs)
    if OUT is None:
        OUT = torch.empty(n, dtype=_F32, device=inputs[0].device)
    _dev(OUT, _F32)
    check(lib().silcu_fused_f32(ct.byref(prog), ptrs, lens, _p(OUT), n, _stream()))
    return OUT


# ----------------------------------------------------------------- reductions
def _reduce(name, IN, out_dtype):
    _dev(IN)
    out = torch.empty((), dtype=out_dtype, device=IN.device)
    wp, wn = _ws_args(lib().silcu_reduce_workspace_bytes(IN.numel()), IN.device)
    check(getattr(lib(), name)(_p(IN), IN.numel(), _p(out), wp, wn, _stream()))
    return out


def sum_f32(IN):
    """Whole-array sum as a 0-d device tensor (gpu::sum_f32 + host finish)."""
    _dev(IN, _F32)
    return _reduce("silcu_sum_f32", IN, _F32)


def sum_i32(IN):
    _dev(IN, _I32)
    return _reduce("silcu_sum_i32", IN, _I32)


def min_f32(IN):
    _dev(IN, _F32)
    return _reduce("silcu_min_f32", IN, _F32)


def max_f32(IN):
    _dev(IN, _F32)
    return _reduce("silcu_max_f32", IN, _F32)


def argmax_all_f32(IN):
    """(index int64, value f32) of the first maximum over the whole array."""
    _dev(IN, _F32)
    idx = torch.empty((), dtype=torch.int64, device=IN.device)
    val = torch.empty((), dtype=_F32, device=IN.device)
    wp, wn = _ws_args(lib().silcu_reduce_workspace_bytes(IN.numel()), IN.device)
    check(lib().silcu_argmax_all_f32(_p(IN), IN.numel(), _p(idx), _p(val), wp, wn, _stream()))
    return idx, val


def softmax(IN, OUT=None, rows=None, cols=None):
    _dev(IN, _F32)
    rows, cols = (IN.shape[0], IN.shape[-1]) if rows is None else (rows, cols)
    OUT = torch.empty_like(IN) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_softmax_f32(_p(IN), _p(OUT), rows, cols, _stream()))
    return OUT


def layer_norm(IN, OUT=None, gamma=None, beta=None, rows=None, cols=None, eps=1e-5):
    _dev(IN, _F32), _dev(gamma, _F32), _dev(beta, _F32)
    rows, cols = (IN.shape[0], IN.shape[-1]) if rows is None else (rows, cols)
    OUT = torch.empty_like(IN) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_layer_norm_f32(_p(IN), _p(OUT), _p(gamma), _p(beta), rows, cols, float(eps), _stream()))
    return OUT


def softmax_split(IN, rows, cols, OUT_hi=None, OUT_lo=None):
    """softmax whose result is written as its exact tf32 split (hi, lo)."""
    _dev(IN, _F32)
    OUT_hi = torch.empty_like(IN) if OUT_hi is None else _dev(OUT_hi, _F32)
    OUT_lo = torch.empty_like(IN) if OUT_lo is None else _dev(OUT_lo, _F32)
    check(lib().silcu_softmax_split_f32(_p(IN), _p(OUT_hi), _p(OUT_lo), rows, cols, _stream()))
    return OUT_hi, OUT_lo


def layer_norm_split(IN, gamma, beta, rows, cols, eps=1e-5, OUT_hi=None, OUT_lo=None):
    """layer_norm whose result is written as its exact tf32 split (hi, lo)."""
    _dev(IN, _F32), _dev(gamma, _F32), _dev(beta, _F32)
    OUT_hi = torch.empty_like(IN) if OUT_hi is None else _dev(OUT_hi, _F32)
    OUT_lo = torch.empty_like(IN) if OUT_lo is None else _dev(OUT_lo, _F32)
    check(lib().silcu_layer_norm_split_f32(_p(IN), _p(OUT_hi), _p(OUT_lo), _p(gamma), _p(beta), rows, cols,
                                           float(eps), _stream()))
    return OUT_hi, OUT_lo


def split(src, rows, cols, ld=None, transpose=False):
    """Exact tf32 split (hi, lo) of a [rows, cols] matrix, optionally transposed."""
    _dev(src, _F32)
    n = rows * cols
    hi = torch.empty(n, dtype=_F32, device=src.device)
    lo = torch.empty(n, dtype=_F32, device=src.device)
    check(lib().silcu_split_f32(_p(src), rows, cols, cols if ld is None else ld, int(transpose), _p(hi), _p(lo),
                                _stream()))
    return hi, lo


def transpose_split(src, rows, cols, ld, batch=1, heads=1, s_b=0, s_h=0, src_lo=None, out=None):
    """(hi, lo) of the per-(b, h) transposes of [rows, cols] blocks (see silcu_transpose_split_f32)."""
    _dev(src, _F32)
    n = batch * heads * rows * cols
    if out is None:
        hi = torch.empty(n, dtype=_F32, device=src.device)
        lo = torch.empty(n, dtype=_F32, device=src.device)
    else:
        hi, lo = _dev(out[0], _F32), _dev(out[1], _F32)
    check(lib().silcu_transpose_split_f32(_p(src), _p(src_lo), rows, cols, ld, batch, heads, s_b, s_h,
                                          _p(hi), _p(lo), _stream()))
    return hi, lo


def attention(Q, K, Vt, *, Sq, Sk, batch, heads, ldq, sq_b, sq_h, ldk, sk_b, sk_h, ldv, sv_b, sv_h,
              scale, O=None, O_split=None, ldo=None, so_b=None, so_h=None, D=64, V=None):
    """Fused softmax(Q.K^T * scale).V; Q, K and Vt (V^T [D, Sk] rows) are
    (hi, lo) split pairs.  Or pass Vt=None and V, V's [Sk, D] rows (e.g. the
    V columns of a QKV projection in place); ldv / sv_b / sv_h then describe
    V's rows."""
    a = _lib.AttnArgs()
    if (Vt is None) == (V is None):
        raise ValueError("attention: give exactly one of Vt and V")
    for nm, pair in (("Q", Q), ("K", K), ("Vt", Vt) if Vt is not None else ("V", V)):
        _dev(pair[0], _F32), _dev(pair[1], _F32)
        setattr(a, nm + "_hi", pair[0].data_ptr())
        setattr(a, nm + "_lo", pair[1].data_ptr())
    if O is None and O_split is None:
        O = torch.empty(batch * heads * Sq * D, dtype=_F32, device=Q[0].device)
    if O is not None:
        a.O = _dev(O, _F32).data_ptr()
    if O_split is not None:
        a.O_hi, a.O_lo = _dev(O_split[0], _F32).data_ptr(), _dev(O_split[1], _F32).data_ptr()
    a.Sq, a.Sk, a.D, a.batch, a.heads = Sq, Sk, D, batch, heads
    a.ldq, a.sq_b, a.sq_h = ldq, sq_b, sq_h
    a.ldk, a.sk_b, a.sk_h = ldk, sk_b, sk_h
    a.ldv, a.sv_b, a.sv_h = ldv, sv_b, sv_h
    a.ldo = D if ldo is None else ldo
    a.so_h = Sq * D if so_h is None else so_h
    a.so_b = heads * Sq * D if so_b is None else so_b
    a.scale = float(scale)
    wp, wn = _ws_args(lib().silcu_attention_workspace_bytes(ct.byref(a)), Q[0].device)
    check(lib().silcu_attention_ex(ct.byref(a), wp, wn, _stream()))
    return O


def argmax_f32(IN, OUT=None, rows=None, cols=None):
    _dev(IN, _F32)
    rows, cols = (IN.shape[0], IN.shape[-1]) if rows is None else (rows, cols)
    OUT = torch.empty(rows, dtype=_I32, device=IN.device) if OUT is None else _dev(OUT, _I32)
    wp, wn = _ws_args(lib().silcu_argmax_workspace_bytes(rows, cols), IN.device)
    check(lib().silcu_argmax_f32(_p(IN), _p(OUT), rows, cols, wp, wn, _stream()))
    return OUT


def sum_axis_f32(IN, outer, length, inner, OUT=None):
    _dev(IN, _F32)
    OUT = torch.empty(outer * inner, dtype=_F32, device=IN.device) if OUT is None else _dev(OUT, _F32)
    wp, wn = _ws_args(lib().silcu_sum_axis_workspace_bytes(outer, length, inner), IN.device)
    check(lib().silcu_sum_axis_f32(_p(IN), _p(OUT), outer, length, inner, wp, wn, _stream()))
    return OUT


def sum_axis_seq_f32(IN, outer, length, inner, OUT=None):
    """Sum over an axis in the reference CPU loop's order (bit-identical)."""
    _dev(IN, _F32)
    OUT = torch.empty(outer * inner, dtype=_F32, device=IN.device) if OUT is None else _dev(OUT, _F32)
    check(lib().silcu_sum_axis_seq_f32(_p(IN), _p(OUT), outer, length, inner, _stream()))
    return OUT


def sum_axis0_f32(IN, OUT=None, rows=None, cols=None):
    """gpu::sum_axis0_f32 (include/gpu.h:385-406): column sums of [rows, cols]."""
    rows, cols = (IN.shape[0], IN.shape[1]) if rows is None else (rows, cols)
    return sum_axis_f32(IN, 1, rows, cols, OUT)


# ---------------------------------------------------------------------- GEMM
ALGO = {"auto": 0, "ffma": 1, "tc": 2}
ACT = {None: 0, "none": 0, "relu": 1, "sigmoid": 2}


def gemm(A, B, C=None, *, M, N, K, lda=None, ldb=None, ldc=None, trans_a=False, trans_b=False,
         batch=1, stride_a=0, stride_b=0, stride_c=0, batch_inner=1, stride_a_inner=0,
         stride_b_inner=0, stride_c_inner=0, alpha=1.0, bias=None, act=None,
         residual=None, ldr=None, algo="auto", C_split=None, no_c=False, acc_chunk_k=0):
    """C = act(alpha * op(A).op(B) + bias) + residual (silcu_sgemm_ex).

    A and B are CUDA float tensors, or (hi, lo) pairs holding the exact tf32
    split of the operand (what the tensor-core path consumes; written by
    producers with a split output).  C_split=(hi, lo) additionally writes the
    split of the result; no_c=True writes only the split.  acc_chunk_k: k
    values per TMEM accumulation chunk on the tensor-core path (0 = 128; see
    silcu_gemm_args)."""
    def ops(X):
        if isinstance(X, (tuple, list)):
            _dev(X[0], _F32), _dev(X[1], _F32)
            return None, X[0], X[1]
        _dev(X, _F32)
        return X, None, None
    Ad, Ah, Al = ops(A)
    Bd, Bh, Bl = ops(B)
    dev = (Ad if Ad is not None else Ah).device
    if C is None and not no_c:
        C = torch.empty(batch * batch_inner * M * N, dtype=_F32, device=dev)
        if batch_inner > 1 and stride_c_inner == 0:
            stride_c_inner = M * N
        if batch > 1 and stride_c == 0:
            stride_c = batch_inner * M * N
    a = _lib.GemmArgs()
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    a.A, a.B = ptr(Ad), ptr(Bd)
    a.A_hi, a.A_lo, a.B_hi, a.B_lo = ptr(Ah), ptr(Al), ptr(Bh), ptr(Bl)
    if C is not None:
        _dev(C, _F32)
        a.C = C.data_ptr()
    if C_split is not None:
        _dev(C_split[0], _F32), _dev(C_split[1], _F32)
        a.C_hi, a.C_lo = C_split[0].data_ptr(), C_split[1].data_ptr()
    a.M, a.N, a.K = M, N, K
    a.lda = lda if lda is not None else (M if trans_a else K)
    a.ldb = ldb if ldb is not None else (K if trans_b else N)
    a.ldc = ldc if ldc is not None else N
    a.trans_a, a.trans_b = int(trans_a), int(trans_b)
    a.batch = batch
    a.stride_a, a.stride_b, a.stride_c = stride_a, stride_b, stride_c
    a.batch_inner = batch_inner
    a.stride_a_inner, a.stride_b_inner, a.stride_c_inner = stride_a_inner, stride_b_inner, stride_c_inner
    a.alpha = float(alpha)
    if bias is not None:
        _dev(bias, _F32)
        a.bias, a.bias_len = bias.data_ptr(), bias.numel()
    a.act = ACT[act]
    if residual is not None:
        _dev(residual, _F32)
        a.residual = residual.data_ptr()
        a.ldr = ldr if ldr is not None else N
    a.algo = ALGO[algo]
    a.acc_chunk_k = int(acc_chunk_k)
    need = lib().silcu_sgemm_workspace_bytes(ct.byref(a))
    wp, wn = _ws_args(need, dev)
    check(lib().silcu_sgemm_ex(ct.byref(a), wp, wn, _stream()))
    return C


def sgemm(A, B, C, M, N, K, lda, ldb, tA=False, tB=False):
    """gpu::sgemm (include/gpu.h:509-514) with the reference argument list."""
    return gemm(A, B, C, M=M, N=N, K=K, lda=lda, ldb=ldb, trans_a=tA, trans_b=tB)


def sgemm_batched(A, B, C, M, N, K, lda, ldb, batch, strideA, strideB, strideC):
    """gpu::sgemm_batched / sgemm_steel_batched (include/gpu.h:518-535)."""
    return gemm(A, B, C, M=M, N=N, K=K, lda=lda, ldb=ldb, batch=batch, stride_a=strideA,
                stride_b=strideB, stride_c=strideC)


def sgemm_bias(A, B, C, bias, bias_len, M, N, K, lda, ldb):
    """gpu::sgemm_bias_steel (include/gpu.h:584-590)."""
    return gemm(A, B, C, M=M, N=N, K=K, lda=lda, ldb=ldb, bias=bias[:bias_len])


def sgemm_bias_sigmoid(A, B, C, bias, bias_len, M, N, K, lda, ldb):
    """gpu::sgemm_bias_sigmoid_steel (include/gpu.h:609-615)."""
    return gemm(A, B, C, M=M, N=N, K=K, lda=lda, ldb=ldb, bias=bias[:bias_len], act="sigmoid")


def conv2d(input, weight, output=None, N=None, H=None, W=None, C_in=None, K=None, C_out=None):
    """gpu::conv2d (include/gpu.h:815-833): NHWC input, OHWI weight, stride 1,
    padding K/2; output [N*H*W, C_out]."""
    _dev(input, _F32), _dev(weight, _F32)
    if N is None:
        N, H, W, C_in = input.shape
        C_out, K = weight.shape[0], weight.shape[1]
    if output is None:
        output = torch.empty(N * H * W * C_out, dtype=_F32, device=input.device)
    _dev(output, _F32)
    wp, wn = _ws_args(lib().silcu_conv2d_workspace_bytes(N, H, W, C_in, K, C_out), input.device)
    check(lib().silcu_conv2d_f32(_p(input), _p(weight), _p(output), N, H, W, C_in, K, C_out, wp, wn, _stream()))
    return output


def sgemv(x, W, y, N, K, bias=None):
    """gpu::sgemv (include/gpu.h:549-574): y[N] = x[K] . W[K,N] (+ bias)."""
    _dev(x, _F32), _dev(W, _F32), _dev(y, _F32)
    wp, wn = _ws_args(lib().silcu_sgemv_workspace_bytes(N, K), x.device)
    check(lib().silcu_sgemv(_p(x), _p(W), _p(y), _p(bias), N, K, wp, wn, _stream()))
    return y
