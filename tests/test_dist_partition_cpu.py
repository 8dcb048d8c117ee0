"""Host logic of the partitioner (silarray_b200.dist) on CPU: gloo ranks
(world 2 and a ragged world 3) each compute their shard of dot / GEMV /
row ops / batched dot / BMM attention / the transformer batch split, with
the oracle standing in for the kernels (`ops=`), and gather_rows assembles
the whole result, which must equal the whole-array oracle.  The GPU runs use
the same code with the silcu kernels and NCCL (tests/test_gpu_multi.py).

Also the failure path: a rank that raises before a combine makes the other
ranks' combine end with CombineTimeout within its deadline (no hang)."""
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from silarray_b200 import dist as sd


class OracleOps:
    """The subset of silarray_b200.gpu the partitioner calls, on CPU tensors
    through the oracle (test stand-in only)."""

    @staticmethod
    def _np(t):
        return t.detach().cpu().numpy().astype(np.float32, copy=False)

    def gemm(self, A, B, C=None, *, M, N, K, batch=1, stride_a=0, stride_b=0, stride_c=0, **kw):
        import oracle as O
        a, b = self._np(A), self._np(B)
        out = np.empty(batch * M * N, np.float32)
        for i in range(batch):
            ai = a[i * stride_a: i * stride_a + M * K].reshape(M, K)
            bi = b[i * stride_b: i * stride_b + K * N].reshape(K, N)
            out[i * M * N:(i + 1) * M * N] = O.sgemm(ai, bi).ravel()
        return torch.from_numpy(out)

    def sgemv(self, x, W, y, N, K, bias=None):
        import oracle as O
        r = O.sgemm(self._np(x).reshape(1, K), self._np(W).reshape(K, N)).ravel()
        if bias is not None:
            r = O.binary("add", r, self._np(bias))
        y[:] = torch.from_numpy(r)
        return y

    def softmax(self, x, rows, cols):
        import oracle as O
        return torch.from_numpy(O.softmax(self._np(x).reshape(rows, cols)).ravel())

    def layer_norm(self, x, gamma, beta, rows, cols, eps=1e-5):
        import oracle as O
        return torch.from_numpy(O.layer_norm(self._np(x).reshape(rows, cols), self._np(gamma), self._np(beta),
                                             eps).ravel())

    def argmax_f32(self, x, rows, cols):
        import oracle as O
        return torch.from_numpy(O.argmax(self._np(x).reshape(rows, cols)).astype(np.int32))

    def sum_axis_f32(self, x, outer, length, inner):
        import oracle as O
        return torch.from_numpy(O.sum_axis(self._np(x).reshape(outer, length), 1).ravel())

    def split(self, x, rows, cols):
        return x, torch.zeros_like(x)

    def transpose_split(self, src, rows, cols, ld, batch=1, s_b=0, **kw):
        a = self._np(src)
        t = np.concatenate([a[i * s_b: i * s_b + rows * cols].reshape(rows, cols).T.ravel()
                            for i in range(batch)])
        t = torch.from_numpy(np.ascontiguousarray(t))
        return t, torch.zeros_like(t)

    def attention(self, Q, K, Vt, *, Sq, Sk, batch, scale, D=64, **kw):
        import oracle as O
        q, k, vt = self._np(Q[0]), self._np(K[0]), self._np(Vt[0])
        out = []
        for i in range(batch):
            qi = q[i * Sq * D:(i + 1) * Sq * D].reshape(Sq, D)
            ki = k[i * Sk * D:(i + 1) * Sk * D].reshape(Sk, D)
            vti = vt[i * D * Sk:(i + 1) * D * Sk].reshape(D, Sk)
            s = O.scalar_op("mul", np.float32(scale), O.sgemm(qi, ki, tb=True)).reshape(Sq, Sk)
            out.append(O.sgemm(O.softmax(s), vti, tb=True).ravel())
        return torch.from_numpy(np.concatenate(out))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(11)
    return {
        "A": rng.uniform(-1, 1, (37, 24)).astype(np.float32),
        "B": rng.uniform(-1, 1, (24, 19)).astype(np.float32),
        "x": rng.normal(0, 1, 64).astype(np.float32),
        "W": rng.normal(0, 0.02, (64, 45)).astype(np.float32),
        "b": rng.normal(0, 0.01, 45).astype(np.float32),
        "X": rng.normal(0, 2, (29, 130)).astype(np.float32),
        "g": rng.normal(1, 0.1, 130).astype(np.float32),
        "be": rng.normal(0, 0.1, 130).astype(np.float32),
        "BA": rng.normal(0, 1, (7, 5, 6)).astype(np.float32),
        "BB": rng.normal(0, 1, (7, 6, 4)).astype(np.float32),
        "Q": rng.normal(0, 1, (5, 16, 64)).astype(np.float32),
        "Kt": rng.normal(0, 1, (5, 64, 16)).astype(np.float32),
        "V": rng.normal(0, 1, (5, 16, 64)).astype(np.float32),
    }


def _worker(rank, world, port, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ops = OracleOps()
        I = {k: torch.from_numpy(v) for k, v in _inputs().items()}
        res = {}
        c, (r0, r1) = sd.dot(I["A"], I["B"], 37, 19, 24, ops=ops)
        res["dot"] = sd.gather_rows(c, 37, 19).numpy()
        gv = sd.GemvColumns(I["W"], I["b"], 64, 45, ops=ops)
        y = gv(I["x"])
        # columns are gathered as rows of a [45, 1] matrix
        res["gemv"] = sd.gather_rows(y, 45, 1).numpy()
        s, _ = sd.softmax_rows(I["X"], 29, 130, ops=ops)
        res["softmax"] = sd.gather_rows(s, 29, 130).numpy()
        ln, _ = sd.layer_norm_rows(I["X"], I["g"], I["be"], 29, 130, ops=ops)
        res["layer_norm"] = sd.gather_rows(ln, 29, 130).numpy()
        am, _ = sd.argmax_rows(I["X"], 29, 130, ops=ops)
        res["argmax"] = sd.gather_rows(am, 29, 1).numpy()
        sr, _ = sd.sum_rows(I["X"], 29, 130, ops=ops)
        res["sum_rows"] = sd.gather_rows(sr, 29, 1).numpy()
        bd, _ = sd.batched_dot(I["BA"], I["BB"], 7, 5, 4, 6, ops=ops)
        res["batched_dot"] = sd.gather_rows(bd, 7, 20).numpy()
        at, _ = sd.bmm_attention(I["Q"], I["Kt"], I["V"], 5, 16, 64, 0.125, ops=ops)
        res["attention"] = sd.gather_rows(at, 5, 16 * 64).numpy()
        q.put((rank, res, None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _spawn(target, world, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + tuple(extra)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return res, procs


@pytest.mark.parametrize("world", [2, 3])
def test_partitioned_ops_match_whole_array_oracle(world):
    import oracle as O
    I = _inputs()
    want = {
        "dot": O.sgemm(I["A"], I["B"]).ravel(),
        "gemv": O.binary("add", O.sgemm(I["x"].reshape(1, -1), I["W"]).ravel(), I["b"]),
        "softmax": O.softmax(I["X"]).ravel(),
        "layer_norm": O.layer_norm(I["X"], I["g"], I["be"]).ravel(),
        "argmax": O.argmax(I["X"]).ravel(),
        "sum_rows": O.sum_axis(I["X"], 1).ravel(),
        "batched_dot": np.concatenate([O.sgemm(I["BA"][i], I["BB"][i]).ravel() for i in range(7)]),
        "attention": np.concatenate([
            O.sgemm(O.softmax(O.scalar_op("mul", np.float32(0.125), O.sgemm(I["Q"][i], I["Kt"][i])).reshape(16, 16)),
                    I["V"][i]).ravel() for i in range(5)]),
    }
    res, procs = _spawn(_worker, world)
    for rank, got, err in res:
        assert err is None, f"rank {rank}: {err}"
        for k, v in want.items():
            np.testing.assert_array_equal(got[k].ravel(), v, err_msg=f"{k} (world {world}, rank {rank})")
    for p in procs:
        assert p.exitcode == 0


def test_sharded_block_spans():
    """The transformer batch split: every sequence of the global batch on
    exactly one rank, contiguous token rows, for 1/2/4/8 ranks and a ragged 3."""
    from silarray_b200 import transformer
    cfg = transformer.Config()
    for world in (1, 2, 3, 4, 8):
        spans = []
        for r in range(world):
            s0, s1 = sd.shard(cfg.batch, r, world)
            spans.append((s0 * cfg.seq, s1 * cfg.seq))
        assert spans[0][0] == 0 and spans[-1][1] == cfg.tokens
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def _failing_worker(rank, world, port, q, deadline):
    sd.init("gloo", timeout_s=30, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    if rank == world - 1:
        # this rank fails before the combine and leaves without joining it
        q.put((rank, "raised", 0.0))
        raise SystemExit(3)
    t0 = time.monotonic()
    try:
        sd.combine_sum(1.0, deadline_s=deadline)
        q.put((rank, "completed", time.monotonic() - t0))
    except sd.CombineTimeout:
        q.put((rank, "timeout", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error: " + repr(e), time.monotonic() - t0))


@pytest.mark.parametrize("world", [2, 3])
def test_failed_rank_ends_combine_within_deadline(world):
    deadline = 3.0
    res, procs = _spawn(_failing_worker, world, extra=(deadline,))
    for rank, what, dt in res:
        if rank == world - 1:
            assert what == "raised"
            continue
        assert what == "timeout", (rank, what)
        assert dt <= deadline + 5.0, f"rank {rank} took {dt:.1f} s"
    assert procs[-1].exitcode == 3
