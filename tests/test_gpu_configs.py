"""Parity at the benchmark configurations' own shapes and seeded inputs.

Each test generates the configuration's synthetic inputs (host numpy RNG,
seeded), runs the B200 path on the full shape, and checks it against the
oracle (the reference CPU restatement), the reference's own CPU build where
present (oracle/_ref) and an fp64 recomputation:
  * SGEMM C = A.B, A, B ~ U[-1,1) seed 0: 1024^3 in full, 8192^3 on 24 sampled
    rows that straddle the 128-row tiles and 256-row CTA pairs
    (reference include/array.h:1375-1403);
  * GEMV / linear 1x4096 . 4096x4096 + b and the small batch 32x4096 . 4096x768
    (include/array.h:1405-1416);
  * BMM attention, B*H = 128, S = 1024, d = 64: softmax(Q.K^T / 8).V with K^T
    stored as its own N(0,1) tensor, 6 sampled (b, h) against the oracle chain
    sgemm -> scalar mul -> softmax -> sgemm (include/array.h:1359-1373, 1676-1709);
  * global sum / min / max / argmax over 2^28 U[-1,1) (include/array.h:1523-1658,
    1711-1750): min, max and argmax bit-exact;
  * row ops on 4096 x {1024, 8192, 32768} N(0, 2^2): argmax bit-exact on every
    row, sum(axis=1) on every row against fp64, softmax / layer_norm on sampled
    rows against the oracle;
  * the transformer block at its full batch of 32: two sequences of the batch-32
    forward against the reference build's block.
Tolerances are those of tests/_tol.py (the north star's)."""
import numpy as np
import pytest
import torch

import oracle as O
from silarray_b200 import gpu, transformer
from tests._tol import assert_close, assert_dot_close, assert_sum_close

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def uniform(rng, shape):
    return rng.uniform(-1.0, 1.0, shape).astype(np.float32)


def normal(rng, shape, std):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def test_sgemm_1024_full(cuda):
    n = 1024
    rng = np.random.default_rng(0)
    a, b = uniform(rng, (n, n)), uniform(rng, (n, n))
    got = host(gpu.gemm(dev(a), dev(b), M=n, N=n, K=n)).reshape(n, n)
    assert_dot_close(got, O.sgemm(a, b), n, what="sgemm 1024^3 vs oracle")
    assert_dot_close(got, a.astype(np.float64) @ b.astype(np.float64), n, what="sgemm 1024^3 vs fp64")
    if O.ref is not None:
        assert_dot_close(got, O.ref.dot(a, b), n, what="sgemm 1024^3 vs reference build")
    gpu.device_status()


def test_sgemm_8192_sampled_rows(cuda):
    n = 8192
    rng = np.random.default_rng(0)
    a, b = uniform(rng, (n, n)), uniform(rng, (n, n))
    got = gpu.gemm(dev(a), dev(b), M=n, N=n, K=n).reshape(n, n)
    rows = [0, 1, 63, 64, 127, 128, 129, 255, 256, 257, 511, 512, 1023, 1024, 2047, 2048, 4095, 4096, 4097,
            6143, 8063, 8064, 8190, 8191]
    g = host(got[rows])
    ref64 = a[rows].astype(np.float64) @ b.astype(np.float64)
    assert_dot_close(g, ref64, n, what="sgemm 8192^3 vs fp64")
    if O.ref is not None:
        assert_dot_close(g, O.ref.dot(np.ascontiguousarray(a[rows]), b), n, what="sgemm 8192^3 vs reference build")
    err = np.abs(g - ref64).max()
    print(f"sgemm 8192^3: max |g - fp64| over {len(rows)} rows = {err:.3e}")
    gpu.device_status()


def test_gemv_and_small_batch(cuda):
    rng = np.random.default_rng(16)
    x = normal(rng, (1, 4096), 1.0)
    W = normal(rng, (4096, 4096), 0.02)
    bb = normal(rng, (4096,), 0.01)
    y = torch.empty(4096, device="cuda")
    gpu.sgemv(dev(x.ravel()), dev(W), y, 4096, 4096, bias=dev(bb))
    ref = O.binary("add", O.sgemm(x, W).ravel(), bb)
    assert_dot_close(host(y), ref, 4096, what="gemv 1x4096.4096x4096+b")
    if O.ref is not None:
        assert_dot_close(host(y), O.ref.linear(x, W, bb).ravel(), 4096, what="gemv vs reference linear")
    X = normal(rng, (32, 4096), 1.0)
    W2 = normal(rng, (4096, 768), 0.02)
    got = host(gpu.gemm(dev(X), dev(W2), M=32, N=768, K=4096)).reshape(32, 768)
    assert_dot_close(got, O.sgemm(X, W2), 4096, what="small batch 32x4096.4096x768")
    gpu.device_status()


def test_bmm_attention_config(cuda):
    BH, S, d = 128, 1024, 64
    rng = np.random.default_rng(48)
    q = normal(rng, (BH, S, d), 1.0)
    kt = normal(rng, (BH, d, S), 1.0)  # K^T stored as its own tensor, as the config supplies it
    v = normal(rng, (BH, S, d), 1.0)
    qs = gpu.split(dev(q.ravel()), BH * S, d)
    ks = gpu.transpose_split(dev(kt.ravel()), d, S, S, batch=BH, s_b=d * S)
    vt = gpu.transpose_split(dev(v.ravel()), S, d, d, batch=BH, s_b=S * d)
    scale = float(np.float32(1.0) / np.float32(8.0))
    out = gpu.attention(qs, ks, vt, Sq=S, Sk=S, batch=BH, heads=1, ldq=d, sq_b=S * d, sq_h=S * d, ldk=d,
                        sk_b=S * d, sk_h=S * d, ldv=S, sv_b=d * S, sv_h=d * S, scale=scale)
    got = host(out).reshape(BH, S, d)
    worst = 0.0
    for bh in (0, 1, 37, 64, 100, 127):
        sc = O.scalar_op("mul", np.float32(scale), O.sgemm(q[bh], kt[bh])).reshape(S, S)
        ref = O.sgemm(O.softmax(sc), v[bh])
        assert_dot_close(got[bh], ref, S, what=f"bmm attention (b*h={bh})")
        worst = max(worst, float(np.abs(got[bh] - ref).max()))
    print(f"bmm attention: max |g - oracle chain| = {worst:.3e}")
    gpu.device_status()


def test_global_reductions_2_28(cuda):
    n = 1 << 28
    rng = np.random.default_rng(80)
    x = uniform(rng, n)
    t = dev(x)
    s = float(host(gpu.sum_f32(t)))
    assert_sum_close(s, x, what="global sum 2^28")
    assert float(host(gpu.min_f32(t))) == float(x.min())
    assert float(host(gpu.max_f32(t))) == float(x.max())
    idx, val = gpu.argmax_all_f32(t)
    i = int(host(idx))
    assert i == int(np.argmax(x)) and float(host(val)) == float(x[i])
    if O.ref is not None:  # the reference's own sum (sequential fp32) differs by its own rounding only
        r = O.ref.reduce("sum", x)
        print(f"global sum 2^28: gpu {s!r}, fp64 {x.astype(np.float64).sum()!r}, reference build {r!r}")
    del t
    gpu.device_status()


@pytest.mark.parametrize("C", [1024, 8192, 32768])
def test_row_ops_config(cuda, C):
    R = 4096
    rng = np.random.default_rng(64 + C)
    x = normal(rng, (R, C), 2.0)
    g = (1.0 + normal(rng, (C,), 0.1)).astype(np.float32)
    b = normal(rng, (C,), 0.1)
    X = dev(x)
    np.testing.assert_array_equal(host(gpu.argmax_f32(X)), O.argmax(x))
    s1 = host(gpu.sum_axis_f32(X, R, C, 1))
    x64 = x.astype(np.float64)
    lim = 1e-5 * np.abs(x64).sum(1) + 1e-6
    assert (np.abs(s1 - x64.sum(1)) <= lim).all(), "sum(axis=1) vs fp64"
    rows = np.array([0, 1, 2, 511, 512, 1023, 2048, 3333, 4094, 4095])
    sm = host(gpu.softmax(X))[rows]
    assert_close(sm, O.softmax(x[rows]), rel=1e-5 if C <= 4096 else 3e-5, abs_=1e-6, what=f"softmax 4096x{C}")
    ln = host(gpu.layer_norm(X, gamma=dev(g), beta=dev(b)))[rows]
    assert_close(ln, O.layer_norm(x[rows], g, b), rel=1e-5, abs_=2e-6, what=f"layer_norm 4096x{C}")
    if O.ref is not None:
        np.testing.assert_array_equal(host(gpu.argmax_f32(X))[rows], O.ref.argmax(x[rows]))
    gpu.device_status()


def test_transformer_full_batch(cuda):
    """The bench's own workload: batch 32 x 512, d 768, 12 heads, FFN 3072,
    weights seed 0, input seed 1 (bench.py's); sequences 0 and 31 of the
    batch-32 forward against the reference build's block.  The measured
    worst error is printed beside the bound it is held to."""
    from oracle import transformer_ref as TR
    cfg = transformer.Config()
    p = transformer.init_params(cfg, seed=0)
    x = transformer.init_input(cfg, seed=1)
    blk = transformer.Block(cfg, p, device="cuda")
    out = host(blk.forward(dev(x)))
    one = transformer.Config(batch=1)
    S = cfg.seq
    worst = 0.0
    for sq in (0, 31):
        ref = TR.reference_forward(one, p, x[sq * S:(sq + 1) * S])
        got = out[sq * S:(sq + 1) * S]
        worst = max(worst, TR.check_parity(got, ref, one))
        worst_rel = float((np.abs(got.astype(np.float64) - ref) / (1 + np.abs(ref))).max())
        assert worst_rel <= TR.BLOCK_TOL
    print(f"transformer batch 32: max |g - reference build| = {worst:.3e}")
    gpu.device_status()
