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
