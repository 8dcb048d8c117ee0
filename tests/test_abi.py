"""C-ABI checks that need no GPU: the library loads, exports every entry
point include/silcu.h declares, and rejects bad arguments with a status
(no exception, no abort) before touching the device."""
import ctypes as C

import pytest

from silarray_b200 import _build, _lib


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    names = _lib.declared_symbols()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version(lib):
    assert lib.silcu_abi_version() == 2


def test_null_pointers_are_rejected_with_status(lib):
    st = lib.silcu_add_f32(None, 4, None, 4, None, 4, None)
    assert st == 1  # SILCU_INVALID_ARGUMENT
    assert b"null" in lib.silcu_last_error()


def test_zero_length_is_a_no_op(lib):
    assert lib.silcu_sigmoid_f32(None, None, 0, None) == 0
    assert lib.silcu_softmax_f32(None, None, 0, 5, None) == 0


def test_gemm_validation(lib):
    a = _lib.GemmArgs()
    a.A = a.B = a.C = 16  # never dereferenced: validation fails first
    a.M, a.N, a.K = 4, 4, 4
    a.lda, a.ldb, a.ldc = 2, 4, 4  # lda < K
    a.batch = 1
    a.alpha = 1.0
    assert lib.silcu_sgemm_ex(C.byref(a), None, 0, None) == 1
    assert b"lda" in lib.silcu_last_error()


def test_fused_program_validation(lib):
    p = _lib.Program()
    p.n_instr = 1
    p.n_inputs = 1
    p.code[0] = _lib.Instr(0, 0, 3, 0, 0.0, 0.0)  # loads input 3 of 1
    ptrs = (C.c_void_p * 1)(16)
    lens = (C.c_size_t * 1)(4)
    assert lib.silcu_fused_f32(C.byref(p), ptrs, lens, C.c_void_p(16), 4, None) == 1


def test_workspace_queries_need_no_device(lib):
    assert lib.silcu_reduce_workspace_bytes(1 << 28) >= 8 * 148
    a = _lib.GemmArgs()
    a.M = a.N = a.K = 8192
    a.lda = a.ldb = a.ldc = 8192
    a.batch = 1
    a.alpha = 1.0
    a.algo = 2
    assert lib.silcu_sgemm_workspace_bytes(C.byref(a)) >= 2 * 8192 * 8192 * 2 * 4


def test_python_mirror_refuses_cpu_tensors():
    import torch
    from silarray_b200 import gpu
    with pytest.raises(TypeError):
        gpu.add(torch.ones(4), torch.ones(4))
