"""Fused attention (silcu_attention_f32) vs the node-by-node oracle chain:
scores = fl(Q.K^T * scale) (fp64-accumulated GEMM), softmax (the reference's
CPU softmax), O = P.V; tolerance |g - r| <= sqrt(Sk) * (1e-6 + 1e-5 |r|)."""
import numpy as np
import pytest
import torch

import oracle as O
from silarray_b200 import gpu
from tests._tol import assert_dot_close

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale):
    s = O.scalar_op("mul", scale, O.sgemm(q, k, tb=True)).reshape(q.shape[0], k.shape[0])
    return O.sgemm(O.softmax(s), v)


@pytest.mark.parametrize("B,H,S", [(1, 1, 64), (2, 3, 200), (1, 2, 300), (1, 2, 512), (1, 1, 1000)])
def test_attention_matches_chain(cuda, B, H, S):
    D = 64
    rng = np.random.default_rng(S + H)
    q = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    k = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    v = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    dq, dk, dv = (torch.from_numpy(t).cuda().reshape(-1) for t in (q, k, v))
    qs = gpu.split(dq, B * H * S, D)
    ks = gpu.split(dk, B * H * S, D)
    vt = gpu.transpose_split(dv, S, D, D, batch=B, heads=H, s_b=H * S * D, s_h=S * D)
    scale = float(np.float32(0.125))
    hi = torch.empty(B * H * S * D, device="cuda")
    lo = torch.empty(B * H * S * D, device="cuda")
    out = gpu.attention(qs, ks, vt, Sq=S, Sk=S, batch=B, heads=H, ldq=D, sq_b=H * S * D, sq_h=S * D,
                        ldk=D, sk_b=H * S * D, sk_h=S * D, ldv=S, sv_b=H * D * S, sv_h=D * S,
                        scale=scale, O_split=(hi, lo), O=torch.empty(B * H * S * D, device="cuda"))
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(B, H, S, D)
    np.testing.assert_array_equal((hi + lo).cpu().numpy().reshape(B, H, S, D), got)
    for b in range(B):
        for h in range(H):
            assert_dot_close(got[b, h], _ref(q[b, h], k[b, h], v[b, h], np.float32(scale)), S,
                             what=f"attention b{b} h{h}")
    gpu.device_status()


@pytest.mark.parametrize("B,H,S", [(1, 1, 64), (2, 3, 200), (1, 2, 300), (1, 1, 1000)])
def test_attention_v_rows(cuda, B, H, S):
    """V given as its [Sk, D] rows (read in place, e.g. from a QKV projection)
    instead of V^T: the same products in the same order, so the output equals
    the V^T form bit for bit, and the oracle chain within tolerance."""
    D = 64
    rng = np.random.default_rng(S * 3 + H)
    q = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    k = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    v = rng.normal(0, 1, (B, H, S, D)).astype(np.float32)
    dq, dk, dv = (torch.from_numpy(t).cuda().reshape(-1) for t in (q, k, v))
    qs, ks, vs = (gpu.split(t, B * H * S, D) for t in (dq, dk, dv))
    vt = gpu.transpose_split(dv, S, D, D, batch=B, heads=H, s_b=H * S * D, s_h=S * D)
    common = dict(Sq=S, Sk=S, batch=B, heads=H, ldq=D, sq_b=H * S * D, sq_h=S * D, ldk=D, sk_b=H * S * D,
                  sk_h=S * D, scale=float(np.float32(0.125)))
    o_t = gpu.attention(qs, ks, vt, ldv=S, sv_b=H * D * S, sv_h=D * S, **common)
    o_r = gpu.attention(qs, ks, None, V=vs, ldv=D, sv_b=H * S * D, sv_h=S * D, **common)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o_r.cpu().numpy(), o_t.cpu().numpy())
    got = o_r.cpu().numpy().reshape(B, H, S, D)
    for b in range(B):
        for h in range(H):
            assert_dot_close(got[b, h], _ref(q[b, h], k[b, h], v[b, h], np.float32(0.125)), S,
                             what=f"attention (V rows) b{b} h{h}")
    gpu.device_status()


def _attn_inputs(B, H, Sq, Sk, seed):
    D = 64
    rng = np.random.default_rng(seed)
    q = rng.normal(0, 1, (B, H, Sq, D)).astype(np.float32)
    k = rng.normal(0, 1, (B, H, Sk, D)).astype(np.float32)
    v = rng.normal(0, 1, (B, H, Sk, D)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("splits", [1, 2, 3, 4])
@pytest.mark.parametrize("B,H,Sq,Sk", [(2, 3, 200, 700), (1, 2, 128, 1024), (1, 1, 64, 300)])
def test_attention_split_kv(cuda, monkeypatch, splits, B, H, Sq, Sk):
    """Split-KV: each (batch, head, query tile) as up to 4 key ranges on
    separate CTAs plus the combine pass, forced by SILCU_ATTN_SPLITS, ragged
    Sq and Sk (tail key block inside the last range).  Within the chain's
    tolerance of the oracle; the split output (hi + lo) equals the plain
    output; one range is the unsplit kernel bit for bit."""
    D = 64
    q, k, v = _attn_inputs(B, H, Sq, Sk, Sq + Sk + splits)
    dq, dk, dv = (torch.from_numpy(t).cuda().reshape(-1) for t in (q, k, v))
    qs = gpu.split(dq, B * H * Sq, D)
    ks = gpu.split(dk, B * H * Sk, D)
    vs = gpu.split(dv, B * H * Sk, D)
    common = dict(Sq=Sq, Sk=Sk, batch=B, heads=H, ldq=D, sq_b=H * Sq * D, sq_h=Sq * D, ldk=D, sk_b=H * Sk * D,
                  sk_h=Sk * D, scale=float(np.float32(0.125)), ldv=D, sv_b=H * Sk * D, sv_h=Sk * D)
    monkeypatch.setenv("SILCU_ATTN_SPLITS", "1")
    o1 = gpu.attention(qs, ks, None, V=vs, **common)
    monkeypatch.setenv("SILCU_ATTN_SPLITS", str(splits))
    hi = torch.empty(B * H * Sq * D, device="cuda")
    lo = torch.empty_like(hi)
    o = gpu.attention(qs, ks, None, V=vs, O=torch.empty_like(hi), O_split=(hi, lo), **common)
    torch.cuda.synchronize()
    got = o.cpu().numpy().reshape(B, H, Sq, D)
    np.testing.assert_array_equal((hi + lo).cpu().numpy().reshape(B, H, Sq, D), got)
    if splits == 1:
        np.testing.assert_array_equal(got, o1.cpu().numpy().reshape(B, H, Sq, D))
    for b in range(B):
        for h in range(H):
            r = _ref(q[b, h], k[b, h], v[b, h], np.float32(0.125))
            assert_dot_close(got[b, h], r, Sk, what=f"split {splits} attention b{b} h{h}")
    gpu.device_status()


@pytest.mark.parametrize("splits", [2, 3])
def test_attention_split_kv_vt(cuda, monkeypatch, splits):
    """Split-KV with V given as V^T (K-major) and Sq != Sk, ragged: within the
    oracle chain's tolerance, and a workspace smaller than the split needs
    runs the call unsplit (the same result as one range, bit for bit)."""
    import ctypes as ct
    from silarray_b200 import _lib
    B, H, Sq, Sk, D = 1, 2, 150, 900, 64
    q, k, v = _attn_inputs(B, H, Sq, Sk, 77 + splits)
    dq, dk, dv = (torch.from_numpy(t).cuda().reshape(-1) for t in (q, k, v))
    qs = gpu.split(dq, B * H * Sq, D)
    ks = gpu.split(dk, B * H * Sk, D)
    vt = gpu.transpose_split(dv, Sk, D, D, batch=B, heads=H, s_b=H * Sk * D, s_h=Sk * D)
    common = dict(Sq=Sq, Sk=Sk, batch=B, heads=H, ldq=D, sq_b=H * Sq * D, sq_h=Sq * D, ldk=D, sk_b=H * Sk * D,
                  sk_h=Sk * D, scale=float(np.float32(0.125)), ldv=Sk, sv_b=H * D * Sk, sv_h=D * Sk)
    monkeypatch.setenv("SILCU_ATTN_SPLITS", str(splits))
    got = gpu.attention(qs, ks, vt, **common)
    torch.cuda.synchronize()
    g = got.cpu().numpy().reshape(B, H, Sq, D)
    for h in range(H):
        assert_dot_close(g[0, h], _ref(q[0, h], k[0, h], v[0, h], np.float32(0.125)), Sk,
                         what=f"split {splits} attention (V^T) h{h}")
    # the same arguments through silcu_attention_ex with no workspace: unsplit
    a = _lib.AttnArgs()
    a.Q_hi, a.Q_lo = qs[0].data_ptr(), qs[1].data_ptr()
    a.K_hi, a.K_lo = ks[0].data_ptr(), ks[1].data_ptr()
    a.Vt_hi, a.Vt_lo = vt[0].data_ptr(), vt[1].data_ptr()
    o2 = torch.empty(B * H * Sq * D, device="cuda")
    a.O = o2.data_ptr()
    a.Sq, a.Sk, a.D, a.batch, a.heads = Sq, Sk, D, B, H
    a.ldq, a.sq_b, a.sq_h = D, H * Sq * D, Sq * D
    a.ldk, a.sk_b, a.sk_h = D, H * Sk * D, Sk * D
    a.ldv, a.sv_b, a.sv_h = Sk, H * D * Sk, D * Sk
    a.ldo, a.so_b, a.so_h = D, H * Sq * D, Sq * D
    a.scale = float(np.float32(0.125))
    assert gpu.lib().silcu_attention_workspace_bytes(ct.byref(a)) > 0
    _lib.check(gpu.lib().silcu_attention_ex(ct.byref(a), None, 0, gpu._stream()))
    monkeypatch.setenv("SILCU_ATTN_SPLITS", "1")
    o1 = gpu.attention(qs, ks, vt, **common)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o2.cpu().numpy(), o1.cpu().numpy())
    gpu.device_status()


def test_attention_split_choice(cuda, monkeypatch):
    """The split is taken by shape: one query tile over 4096 keys splits (a
    workspace is asked for); the benchmark's 12 heads x 4 query tiles x batch
    32 does not."""
    import ctypes as ct
    from silarray_b200 import _lib
    monkeypatch.delenv("SILCU_ATTN_SPLITS", raising=False)
    a = _lib.AttnArgs()
    a.Sq, a.Sk, a.D, a.batch, a.heads = 128, 4096, 64, 1, 1
    assert gpu.lib().silcu_attention_workspace_bytes(ct.byref(a)) > 0
    a.Sq, a.Sk, a.batch, a.heads = 512, 512, 32, 12
    assert gpu.lib().silcu_attention_workspace_bytes(ct.byref(a)) == 0
