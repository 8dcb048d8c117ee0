"""Test infrastructure only: CPU reference of the pre-norm transformer block
(the reference's bench/composite/bench_transformer.cpp:56-67 generalised to a
batch of sequences and multi-head attention) and the end-to-end tolerance the
B200 forward is held to.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU leg; the product package never imports it."""
import numpy as np

import oracle as O


def reference_forward(cfg, params, x):
    """CPU reference of the B200 block (silarray_b200.transformer.Block): the reference's own CPU build when it
    is present (oracle/_ref, every op a sil:: array op), else the oracle
    restatement composed the same way.  Test infrastructure only."""
    if O.ref is not None:
        return O.ref.transformer_block(x, cfg.batch, cfg.seq, cfg.d_model, cfg.heads, cfg.d_ff, params)
    return _restated_forward(cfg, params, x)


def _restated_forward(cfg, p, x):
    S, d, H, hd = cfg.seq, cfg.d_model, cfg.heads, cfg.head_dim
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    out = np.empty_like(x)
    lin = lambda a, w, b: O.binary("add", O.sgemm(a, w), b).reshape(a.shape[0], w.shape[1])  # noqa: E731
    for bi in range(cfg.batch):
        X = x[bi * S:(bi + 1) * S]
        h = O.layer_norm(X, p["g1"], p["be1"])
        Q, K, V = lin(h, p["wq"], p["bq"]), lin(h, p["wk"], p["bk"]), lin(h, p["wv"], p["bv"])
        ctx = np.empty((S, d), np.float32)
        for hh in range(H):
            sl = slice(hh * hd, (hh + 1) * hd)
            q, k, v = (np.ascontiguousarray(m[:, sl]) for m in (Q, K, V))
            sc = O.scalar_op("mul", scale, O.sgemm(q, k, tb=True)).reshape(S, S)
            at = O.softmax(sc)
            ctx[:, sl] = O.sgemm(at, v)
        r1 = O.binary("add", X, lin(ctx, p["wo"], p["bo"])).reshape(S, d)
        h2 = O.layer_norm(r1, p["g2"], p["be2"])
        ff = O.relu(lin(h2, p["w1"], p["b1"]))
        out[bi * S:(bi + 1) * S] = O.binary("add", r1, lin(ff, p["w2"], p["b2"])).reshape(S, d)
    return out


BLOCK_TOL = 2e-5  # |g - r| <= BLOCK_TOL * (1 + |r|) end to end; measured worst 4.1e-6 at the bench shape


def check_parity(got, ref, cfg):
    """End-to-end tolerance for the 6-GEMM chain: |g - r| <= BLOCK_TOL * (1 + |r|)
    (each GEMM is within sqrt(K) * (1e-6 + 1e-5|r|) of the oracle; layer_norm
    and softmax amplify the differences by O(1) factors)."""
    got = np.asarray(got, np.float64).reshape(ref.shape)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    lim = BLOCK_TOL * (1.0 + np.abs(ref))
    if not (err <= lim).all():
        i = int(np.argmax(err - lim))
        raise AssertionError(f"transformer parity: {(err > lim).sum()} of {err.size} outside; worst "
                             f"got {got.ravel()[i]!r} ref {ref.ravel()[i]!r}; max err {err.max():.3e}")
    return float(err.max())
