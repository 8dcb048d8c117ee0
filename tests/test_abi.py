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


def _plan(lib, M, N, K, split_in=True, c=True, split_out=False, residual=False, trans_b=1):
    a = _lib.GemmArgs()
    a.M, a.N, a.K = M, N, K
    a.lda, a.ldb, a.ldc, a.ldr = K, (K if trans_b else N), N, N
    a.trans_b = trans_b
    a.batch, a.batch_inner = 1, 1
    a.alpha = 1.0
    fake = C.c_void_p(1 << 20)  # never dereferenced by the planner
    if split_in:
        a.A_hi = a.A_lo = a.B_hi = a.B_lo = fake
    else:
        a.A = a.B = fake
    if c:
        a.C = fake
    if split_out:
        a.C_hi = a.C_lo = fake
    if residual:
        a.residual = fake
    p = _lib.GemmPlan()
    assert lib.silcu_sgemm_plan(C.byref(a), C.byref(p)) == 0
    return p


def _visible_sms():
    import torch
    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(0).multi_processor_count
    return 148  # no device: the library plans for a 148-SM B200


def test_gemm_plan_split_k_choice(lib):
    """The 3xTF32 path's tiling and split-K choice on a 148-SM B200 (the
    library assumes 148 SMs when it cannot query a device) for the
    transformer's GEMMs: at a 4-sequence shard (M = 2048) Wo splits every
    single-CTA tile in 3 K parts, FFN-down (K = 3072) runs CTA pairs with every
    tile in 3 parts, QKV's 72 pair tiles run whole and FFN-up splits only its
    last wave's 22 pair tiles; at the full batch (M = 16384) FFN-down splits
    its last wave's 44 tiles in 5 parts, the other GEMMs none."""
    if _visible_sms() != 148:
        pytest.skip("the pinned plans are those of a 148-SM B200; this device has another SM count")
    p = _plan(lib, 2048, 768, 768, residual=True)  # Wo
    assert (p.path, p.pair, p.tile_n, p.ksplit, p.tiles, p.whole_tiles) == (2, 0, 256, 3, 48, 0)
    p = _plan(lib, 2048, 2304, 768, c=False, split_out=True)  # QKV, split output
    assert (p.pair, p.ksplit, p.tiles, p.whole_tiles) == (1, 1, 72, 72)
    p = _plan(lib, 2048, 3072, 768, c=False, split_out=True)  # FFN-up, split output
    assert (p.pair, p.ksplit, p.tiles, p.whole_tiles) == (1, 3, 96, 74)
    p = _plan(lib, 2048, 768, 3072, residual=True)  # FFN-down
    assert (p.pair, p.ksplit, p.tiles, p.whole_tiles) == (1, 3, 24, 0)
    p = _plan(lib, 16384, 768, 3072, residual=True)  # FFN-down, full batch
    assert (p.pair, p.ksplit, p.tiles, p.whole_tiles) == (1, 5, 192, 148)
    for M, N, K in [(16384, 2304, 768), (16384, 3072, 768), (16384, 768, 768)]:
        p = _plan(lib, M, N, K, c=False, split_out=True)
        assert (p.pair, p.ksplit, p.whole_tiles) == (1, 1, p.tiles), (M, N, K)
    p = _plan(lib, 8192, 8192, 8192, split_in=False)  # the 8192^3 SGEMM: plain operands, no split
    assert (p.path, p.pair, p.ksplit) == (2, 1, 1)
    p = _plan(lib, 1, 4096, 4096, split_in=False, trans_b=0)  # GEMV: x . W[K, N]
    assert p.path == 1
