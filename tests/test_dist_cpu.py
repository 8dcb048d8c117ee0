"""Host logic of the multi-GPU path on CPU: world_size-2 gloo ranks, each
reducing its shard with the oracle and combining through silarray_b200.dist,
against the whole-array oracle (the GPU runs use the same combine over NCCL)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from silarray_b200 import dist as sd


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, x, q):
    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        s0, s1 = sd.shard(x.size, rank, world)
        part = x[s0:s1]
        total = sd.combine_sum(float(np.asarray(part, np.float64).sum()))
        mn = sd.combine_min(O.min_all(part))
        mx = sd.combine_max(O.max_all(part))
        li = int(O.argmax(part.reshape(1, -1))[0])
        has = sd.argmax_key(part[li], 0) != 0
        gi, gv = sd.combine_argmax(part[li], li if has else None, s0)
        q.put((rank, total, mn, mx, gi, gv))
    finally:
        dist.destroy_process_group()


def _run(x, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_shard_covers_everything():
    for total in (0, 1, 7, 100, 2 ** 28):
        for world in (1, 2, 3, 8):
            spans = [sd.shard(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def test_argmax_key_order():
    assert sd.argmax_key(-1.0, 3) == 0 and sd.argmax_key(0.0, 3) == 0
    assert sd.argmax_key(2.0, 5) > sd.argmax_key(1.0, 1)
    assert sd.argmax_key(2.0, 5) > sd.argmax_key(2.0, 9)  # ties: first index wins


@pytest.mark.parametrize("case", ["random", "ties_across_ranks", "no_candidate"])
def test_two_rank_reductions(case):
    import oracle as O
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, 10001).astype(np.float32)
    if case == "ties_across_ranks":
        x[9000] = 7.0
        x[1234] = 7.0
    if case == "no_candidate":
        x = -np.abs(x) - 1
    res = _run(x)
    ref_idx = int(O.argmax(x.reshape(1, -1))[0])
    for rank, total, mn, mx, gi, gv in res:
        assert abs(total - float(x.astype(np.float64).sum())) <= 1e-5 * float(np.abs(x).sum())
        assert mn == float(x.min()) and mx == float(x.max())
        assert gi == ref_idx
        if case != "no_candidate":
            assert gv == float(x[ref_idx])
