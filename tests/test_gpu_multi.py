"""Multi-GPU path on >= 2 GPUs (skipped on one): each rank reduces its shard
of a 2^24-element array with the silcu kernels and the NCCL combine of
silarray_b200.dist gives the whole-array sum / min / max / argmax."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from silarray_b200 import dist as sd
    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        x = np.random.default_rng(5).uniform(-1, 1, 1 << 24).astype(np.float32)
        x[123456] = 9.0
        x[15000000] = 9.0
        s0, s1 = sd.shard(x.size, rank, world)
        xs = torch.from_numpy(x[s0:s1]).cuda()
        q.put((rank, sd.global_sum(xs), sd.global_min(xs), sd.global_max(xs), sd.global_argmax(xs, s0)))
    finally:
        dist.destroy_process_group()


def test_two_gpu_global_reductions(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = np.random.default_rng(5).uniform(-1, 1, 1 << 24).astype(np.float32)
    x[123456] = 9.0
    x[15000000] = 9.0
    for _, s, mn, mx, (gi, gv) in res:
        assert abs(s - float(x.astype(np.float64).sum())) <= 1e-5 * float(np.abs(x).sum())
        assert mn == float(x.min()) and mx == 9.0
        assert gi == 123456 and gv == 9.0


def _partition_inputs():
    rng = np.random.default_rng(21)
    return {
        "A": rng.uniform(-1, 1, (1000, 768)).astype(np.float32),
        "B": rng.uniform(-1, 1, (768, 640)).astype(np.float32),
        "x": rng.normal(0, 1, 4096).astype(np.float32),
        "W": rng.normal(0, 0.02, (4096, 4096)).astype(np.float32),
        "b": rng.normal(0, 0.01, 4096).astype(np.float32),
        "X": rng.normal(0, 2, (515, 8192)).astype(np.float32),
        "g": rng.normal(1, 0.1, 8192).astype(np.float32),
        "be": rng.normal(0, 0.1, 8192).astype(np.float32),
        "Q": rng.normal(0, 1, (6, 256, 64)).astype(np.float32),
        "Kt": rng.normal(0, 1, (6, 64, 256)).astype(np.float32),
        "V": rng.normal(0, 1, (6, 256, 64)).astype(np.float32),
    }


def _partition_worker(rank, world, port, q):
    import torch.distributed as dist
    from silarray_b200 import dist as sd, gpu, transformer
    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    try:
        sd.init("nccl", timeout_s=120, device=dev, init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                world_size=world)
        I = {k: torch.from_numpy(v).to(dev) for k, v in _partition_inputs().items()}
        res = {}
        c, _ = sd.dot(I["A"], I["B"], 1000, 640, 768)
        res["dot"] = sd.gather_rows(c, 1000, 640).cpu().numpy()
        res["gemv"] = sd.gather_rows(sd.GemvColumns(I["W"], I["b"], 4096, 4096)(I["x"]), 4096, 1).cpu().numpy()
        res["softmax"] = sd.gather_rows(sd.softmax_rows(I["X"], 515, 8192)[0], 515, 8192).cpu().numpy()
        res["layer_norm"] = sd.gather_rows(sd.layer_norm_rows(I["X"], I["g"], I["be"], 515, 8192)[0], 515,
                                           8192).cpu().numpy()
        res["argmax"] = sd.gather_rows(sd.argmax_rows(I["X"], 515, 8192)[0], 515, 1).cpu().numpy()
        res["sum_rows"] = sd.gather_rows(sd.sum_rows(I["X"], 515, 8192)[0], 515, 1).cpu().numpy()
        res["attention"] = sd.gather_rows(sd.bmm_attention(I["Q"], I["Kt"], I["V"], 6, 256, 64, 0.125)[0], 6,
                                          256 * 64).cpu().numpy()
        cfg = transformer.Config(batch=4, seq=256, d_model=256, heads=4, d_ff=1024)
        p = transformer.init_params(cfg, seed=3)
        x = torch.from_numpy(transformer.init_input(cfg, seed=4)).to(dev)
        blk = sd.ShardedBlock(cfg, p, dev)
        out = blk.forward(blk.local_input(x))
        res["block"] = sd.gather_rows(out, cfg.tokens, cfg.d_model).cpu().numpy()
        gpu.device_status()
        q.put((rank, res, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, None, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_two_gpu_partitioner(cuda):
    """dot (row shard), GEMV (column shard), softmax / layer_norm / argmax /
    sum(axis=1) (row shard), BMM attention (batch shard) and the transformer
    batch split on 2 GPUs with the silcu kernels; the gathered results
    against the whole-array oracle within the single-GPU tolerances."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import oracle as O
    from oracle import transformer_ref as TR
    from silarray_b200 import transformer
    from tests._tol import assert_close, assert_dot_close
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_partition_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    I = _partition_inputs()
    for rank, got, err in res:
        assert err is None, f"rank {rank}: {err}"
    got = res[0][1]
    assert_dot_close(got["dot"].reshape(1000, 640), O.sgemm(I["A"], I["B"]), 768, what="dot row shard")
    assert_dot_close(got["gemv"], O.binary("add", O.sgemm(I["x"].reshape(1, -1), I["W"]).ravel(), I["b"]), 4096,
                     what="gemv column shard")
    X = I["X"]
    assert_close(got["softmax"].reshape(X.shape), O.softmax(X), rel=3e-5, what="softmax row shard")
    assert_close(got["layer_norm"].reshape(X.shape), O.layer_norm(X, I["g"], I["be"]), abs_=2e-6,
                 what="layer_norm row shard")
    np.testing.assert_array_equal(got["argmax"].ravel(), O.argmax(X))
    x64 = X.astype(np.float64)
    assert (np.abs(got["sum_rows"].ravel() - x64.sum(1)) <= 1e-5 * np.abs(x64).sum(1) + 1e-6).all()
    for i in range(6):
        s = O.scalar_op("mul", np.float32(0.125), O.sgemm(I["Q"][i], I["Kt"][i])).reshape(256, 256)
        assert_dot_close(got["attention"].reshape(6, 256, 64)[i], O.sgemm(O.softmax(s), I["V"][i]), 256,
                         what=f"attention batch shard {i}")
    cfg = transformer.Config(batch=4, seq=256, d_model=256, heads=4, d_ff=1024)
    p = transformer.init_params(cfg, seed=3)
    x = transformer.init_input(cfg, seed=4)
    TR.check_parity(got["block"].reshape(cfg.tokens, cfg.d_model), TR.reference_forward(cfg, p, x), cfg)
    np.testing.assert_array_equal(res[0][1]["block"], res[1][1]["block"])
