"""Multi-GPU partitioning for the hot path (one process per GPU).

The hot path's work is independent per row / sequence / (batch, head), so
the partitioner hands each rank a contiguous shard and no data moves between
GPUs.  The one exchange step is the combine of whole-array reductions
(sum / min / max / argmax over an array split across ranks): each rank
reduces its shard with the silcu kernels and one all-reduce of a scalar
combines them (NCCL over NVLink on GPUs, gloo in the CPU tests).

Combining rules:
  sum     fp64 all-reduce SUM of the per-rank fp32 sums;
  min/max all-reduce MIN/MAX;
  argmax  all-reduce MAX of a 64-bit key (orderable value << 32 | ~global
          index), so the largest value wins and ties go to the first index;
          values <= FLT_MIN are never candidates and an empty result is
          index 0, the reference CPU branch's rule (include/array.h:1733-1740).
"""
import struct

import torch
import torch.distributed as dist

FLT_MIN = struct.unpack("<f", struct.pack("<I", 0x00800000))[0]


def shard(total, rank, world):
    """[start, stop) of `rank`'s contiguous share of `total` units (the first
    total % world ranks get one extra)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("bad rank/world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _ord32(v):
    u = struct.unpack("<I", struct.pack("<f", float(v)))[0]
    return (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000


def _unord32(u):
    b = u & 0x7FFFFFFF if u & 0x80000000 else (~u) & 0xFFFFFFFF
    return struct.unpack("<f", struct.pack("<I", b))[0]


def argmax_key(value, global_index):
    """64-bit key of a local argmax result (0 = no candidate)."""
    v = float(value)
    if not (v > FLT_MIN):
        return 0
    return (_ord32(v) << 32) | (0xFFFFFFFF - (int(global_index) & 0xFFFFFFFF))


def _to_signed64(k):
    return k - (1 << 64) if k >= (1 << 63) else k


def _from_signed64(k):
    return k + (1 << 64) if k < 0 else k


def _device():
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def combine_sum(local_sum):
    t = torch.tensor([float(local_sum)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def combine_min(local_min):
    t = torch.tensor([float(local_min)], dtype=torch.float32, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def combine_max(local_max):
    t = torch.tensor([float(local_max)], dtype=torch.float32, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def combine_argmax(local_value, local_index, offset):
    """Global (index, value) from each rank's local first-argmax; the keys are
    offset by the one bit flip that keeps signed int64 ordering == unsigned."""
    key = argmax_key(local_value, offset + local_index) if local_index is not None else 0
    t = torch.tensor([_to_signed64(key ^ (1 << 63))], dtype=torch.int64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    k = _from_signed64(int(t.item())) ^ (1 << 63)
    if k == 0:
        return 0, None
    return 0xFFFFFFFF - (k & 0xFFFFFFFF), _unord32(k >> 32)


# ----------------------------------------------------- whole-array on GPUs
def global_sum(x_shard):
    """Sum of an array split across ranks; x_shard is this rank's CUDA shard."""
    from . import gpu
    return combine_sum(gpu.sum_f32(x_shard).item())


def global_min(x_shard):
    from . import gpu
    return combine_min(gpu.min_f32(x_shard).item())


def global_max(x_shard):
    from . import gpu
    return combine_max(gpu.max_f32(x_shard).item())


def global_argmax(x_shard, offset):
    """First index of the maximum over the whole array; `offset` is this
    shard's first global index."""
    from . import gpu
    idx, val = gpu.argmax_all_f32(x_shard)
    i, v = int(idx.item()), float(val.item())
    return combine_argmax(v, i if argmax_key(v, 0) else None, offset)
