"""ctypes binding of libsilcu.so (include/silcu.h).

The library is built in-tree by silarray_b200._build.  There is no fallback:
if the shared library is missing or does not load, every call raises.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsilcu.so")

vp = C.c_void_p
sz = C.c_size_t
i32 = C.c_int32
u32 = C.c_uint32
u64 = C.c_uint64
i64 = C.c_int64
f32 = C.c_float

OK = 0
STATUS_NAMES = {0: "OK", 1: "INVALID_ARGUMENT", 2: "CUDA_ERROR", 3: "TIMEOUT",
                4: "WORKSPACE_TOO_SMALL", 5: "UNSUPPORTED"}


class SilcuError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"silcu {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class Instr(C.Structure):
    _fields_ = [("op", i32), ("dst", i32), ("a", i32), ("b", i32), ("imm0", f32), ("imm1", f32)]


MAX_PROGRAM = 32
MAX_INPUTS = 8


class Program(C.Structure):
    _fields_ = [("n_instr", i32), ("n_inputs", i32), ("code", Instr * MAX_PROGRAM)]


class GemmArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("C", vp),
                ("M", i64), ("N", i64), ("K", i64),
                ("lda", i64), ("ldb", i64), ("ldc", i64),
                ("trans_a", i32), ("trans_b", i32),
                ("batch", i64), ("stride_a", i64), ("stride_b", i64), ("stride_c", i64),
                ("batch_inner", i64), ("stride_a_inner", i64), ("stride_b_inner", i64),
                ("stride_c_inner", i64),
                ("alpha", f32), ("bias", vp), ("bias_len", i64), ("act", i32),
                ("residual", vp), ("ldr", i64), ("algo", i32),
                ("A_hi", vp), ("A_lo", vp), ("B_hi", vp), ("B_lo", vp), ("C_hi", vp), ("C_lo", vp),
                ("acc_chunk_k", i32)]


class GemmPlan(C.Structure):
    _fields_ = [("path", i32), ("pair", i32), ("tile_n", i32), ("ksplit", i32), ("tiles", i64), ("whole_tiles", i64)]


class AttnArgs(C.Structure):
    _fields_ = [("Q_hi", vp), ("Q_lo", vp), ("K_hi", vp), ("K_lo", vp), ("Vt_hi", vp), ("Vt_lo", vp),
                ("O", vp), ("O_hi", vp), ("O_lo", vp),
                ("Sq", i64), ("Sk", i64), ("D", i64), ("batch", i64), ("heads", i64),
                ("ldq", i64), ("sq_b", i64), ("sq_h", i64),
                ("ldk", i64), ("sk_b", i64), ("sk_h", i64),
                ("ldv", i64), ("sv_b", i64), ("sv_h", i64),
                ("ldo", i64), ("so_b", i64), ("so_h", i64),
                ("scale", f32), ("V_hi", vp), ("V_lo", vp)]


_SIGS = {
    "silcu_last_error": ([], C.c_char_p),
    "silcu_abi_version": ([], C.c_int),
    "silcu_kernel_launches": ([], C.c_ulonglong),
    "silcu_synchronize": ([vp], C.c_int),
    "silcu_device_status": ([vp], C.c_int),
    "silcu_check_bounded_wait": ([u32, vp], C.c_int),
    "silcu_conv2d_workspace_bytes": ([u32, u32, u32, u32, u32, u32], sz),
    "silcu_conv2d_f32": ([vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, sz, vp], C.c_int),
    "silcu_sigmoid_f32": ([vp, vp, sz, vp], C.c_int),
    "silcu_relu_f32": ([vp, vp, sz, vp], C.c_int),
    "silcu_sigmoid_backward_f32": ([vp, vp, vp, sz, vp], C.c_int),
    "silcu_bias_sigmoid_f32": ([vp, vp, sz, sz, vp], C.c_int),
    "silcu_affine_f32": ([vp, vp, sz, f32, f32, C.c_int, vp], C.c_int),
    "silcu_fused_f32": ([C.POINTER(Program), C.POINTER(vp), C.POINTER(sz), vp, sz, vp], C.c_int),
    "silcu_fused_multi_f32": ([C.POINTER(Program), C.POINTER(vp), C.POINTER(sz), C.POINTER(vp), C.c_int, sz, vp],
                              C.c_int),
    "silcu_reduce_workspace_bytes": ([sz], sz),
    "silcu_sum_f32": ([vp, sz, vp, vp, sz, vp], C.c_int),
    "silcu_sum_f32_noalloc": ([vp, sz, vp, vp], C.c_int),
    "silcu_min_f32": ([vp, sz, vp, vp, sz, vp], C.c_int),
    "silcu_max_f32": ([vp, sz, vp, vp, sz, vp], C.c_int),
    "silcu_sum_i32": ([vp, sz, vp, vp, sz, vp], C.c_int),
    "silcu_argmax_all_f32": ([vp, sz, vp, vp, vp, sz, vp], C.c_int),
    "silcu_softmax_f32": ([vp, vp, sz, sz, vp], C.c_int),
    "silcu_layer_norm_f32": ([vp, vp, vp, vp, sz, sz, f32, vp], C.c_int),
    "silcu_argmax_f32": ([vp, vp, sz, sz, vp, sz, vp], C.c_int),
    "silcu_softmax_split_f32": ([vp, vp, vp, sz, sz, vp], C.c_int),
    "silcu_layer_norm_split_f32": ([vp, vp, vp, vp, vp, sz, sz, f32, vp], C.c_int),
    "silcu_split_f32": ([vp, sz, sz, sz, C.c_int, vp, vp, vp], C.c_int),
    "silcu_transpose_split_f32": ([vp, vp, sz, sz, sz, sz, sz, sz, sz, vp, vp, vp], C.c_int),
    "silcu_attention_f32": ([C.POINTER(AttnArgs), vp], C.c_int),
    "silcu_attention_workspace_bytes": ([C.POINTER(AttnArgs)], C.c_size_t),
    "silcu_attention_ex": ([C.POINTER(AttnArgs), vp, C.c_size_t, vp], C.c_int),
    "silcu_argmax_workspace_bytes": ([sz, sz], sz),
    "silcu_sum_axis_workspace_bytes": ([sz, sz, sz], sz),
    "silcu_sum_axis_f32": ([vp, vp, sz, sz, sz, vp, sz, vp], C.c_int),
    "silcu_sum_axis_seq_f32": ([vp, vp, sz, sz, sz, vp], C.c_int),
    "silcu_sgemm_workspace_bytes": ([C.POINTER(GemmArgs)], sz),
    "silcu_sgemm_plan": ([C.POINTER(GemmArgs), C.POINTER(GemmPlan)], C.c_int),
    "silcu_sgemm_ex": ([C.POINTER(GemmArgs), vp, sz, vp], C.c_int),
    "silcu_sgemm": ([vp, vp, vp, u32, u32, u32, u32, u32, C.c_int, C.c_int, vp, sz, vp], C.c_int),
    "silcu_sgemm_batched": ([vp, vp, vp, u32, u32, u32, u32, u32, u32, u64, u64, u64, vp, sz, vp], C.c_int),
    "silcu_sgemm_bias": ([vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, sz, vp], C.c_int),
    "silcu_sgemm_bias_sigmoid": ([vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, sz, vp], C.c_int),
    "silcu_sgemv_workspace_bytes": ([u32, u32], sz),
    "silcu_sgemv": ([vp, vp, vp, vp, u32, u32, vp, sz, vp], C.c_int),
}
for _op in ("add", "sub", "mul", "div", "pow"):
    for _t in ("f32", "i32"):
        _SIGS[f"silcu_{_op}_{_t}"] = ([vp, sz, vp, sz, vp, sz, vp], C.c_int)

_lib = None


def lib():
    """Loads libsilcu.so once; raises if it is absent (no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m silarray_b200._build` "
                "(the B200 backend has no CPU fallback)")
        dll = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(dll, name)
            fn.argtypes = args
            fn.restype = res
        _lib = dll
    return _lib


def check(status):
    if status != OK:
        raise SilcuError(status, lib().silcu_last_error().decode(errors="replace"))


def declared_symbols():
    """Every function name declared in include/silcu.h (parsed from the header)."""
    import re
    hdr = os.path.join(os.path.dirname(_HERE), "include", "silcu.h")
    text = open(hdr).read()
    return sorted(set(re.findall(r"\b(silcu_[a-z0-9_]+)\s*\(", text)))
