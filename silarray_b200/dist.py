"""Multi-GPU partitioning for the hot path (one process per GPU).

The hot path's work is independent per row / column / sequence / (batch,
head), so the partitioner hands each rank a contiguous shard and no data moves
between GPUs on the data path:
  dot          C = A.B, rows of A (and C) split, B replicated
               (reference include/array.h:1375-1403);
  GEMV/linear  y = x.W + b with W's columns split, x replicated; each rank
               keeps only its column block of W (include/array.h:1405-1416,
               2669-2670);
  row ops      softmax / layer_norm / argmax / sum(axis=1), rows split
               (include/array.h:1486-1505, 1554-1583, 1676-1750);
  BMM          batched products and the fused attention chain, the batch
               (batch x heads) split (include/array.h:1359-1373);
  transformer  the block's batch of sequences split (ShardedBlock).
Inputs are the caller's replicated arrays (each rank reads only its rows /
columns / batch entries through views); outputs are this rank's share, and
`gather_rows` assembles the whole result where a caller wants it on every
rank (one all-gather; not part of the sharded computation).

The one exchange step is the combine of whole-array reductions
(sum / min / max / argmax over an array split across ranks): each rank
reduces its shard with the silcu kernels and one all-reduce of a scalar
combines them (NCCL over NVLink on GPUs, gloo in the CPU tests).  Every
combine waits on the host with a deadline: a rank that failed or never
arrives makes the others raise CombineTimeout (after aborting the process
group) instead of hanging.

Combining rules:
  sum     fp64 all-reduce SUM of the per-rank fp32 sums;
  min/max all-reduce MIN/MAX;
  argmax  all-reduce MAX of a 64-bit key (orderable value << 32 | ~global
          index), so the largest value wins and ties go to the first index;
          values <= FLT_MIN are never candidates and an empty result is
          index 0, the reference CPU branch's rule (include/array.h:1733-1740).
"""
import datetime
import struct
import time

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


# ------------------------------------------------------- process group, deadlines
DEFAULT_DEADLINE_S = 60.0


class CombineTimeout(RuntimeError):
    """A collective did not complete within its deadline (a rank failed,
    left, or never arrived); the process group has been aborted."""


def init(backend=None, timeout_s=DEFAULT_DEADLINE_S, device=None, init_method=None, rank=None, world_size=None):
    """One process per GPU: init_process_group from the torchrun environment
    (RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT), or from init_method /
    rank / world_size when given, with a short collective timeout, so that a
    lost rank ends the others' collectives with an error.  backend: "nccl"
    when a device is given or CUDA is available, else "gloo"."""
    if dist.is_initialized():
        return
    if backend is None:
        backend = "nccl" if (device is not None or torch.cuda.is_available()) else "gloo"
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if init_method is not None:
        kw.update(init_method=init_method, rank=rank, world_size=world_size)
    if backend == "nccl":
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        kw["device_id"] = dev
    dist.init_process_group(backend, **kw)


def abort():
    """Abort the default process group (ncclCommAbort for NCCL): pending
    collectives of this rank end and the group cannot be used again."""
    try:
        from torch.distributed.distributed_c10d import _abort_process_group
        _abort_process_group()
    except Exception:  # noqa: BLE001 - best effort on the failure path
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _wait(work, deadline_s, what):
    """Polls an async collective until it completes or the deadline passes
    (the host never blocks inside the library, so a missing peer cannot hang
    it); on expiry the group is aborted and CombineTimeout raised."""
    t_end = time.monotonic() + deadline_s
    while True:
        try:
            if work.is_completed():
                break
        except RuntimeError as e:  # the backend already failed the collective
            abort()
            raise CombineTimeout(f"{what}: collective failed: {e}") from e
        if time.monotonic() > t_end:
            abort()
            raise CombineTimeout(f"{what}: no completion within {deadline_s:.1f} s (a rank failed or left)")
        time.sleep(50e-6)
    try:
        work.wait()
    except RuntimeError as e:
        abort()
        raise CombineTimeout(f"{what}: collective failed: {e}") from e


def _all_reduce(t, op, deadline_s, what):
    work = dist.all_reduce(t, op=op, async_op=True)
    _wait(work, deadline_s, what)
    return t


def combine_sum(local_sum, deadline_s=DEFAULT_DEADLINE_S):
    t = torch.tensor([float(local_sum)], dtype=torch.float64, device=_device())
    _all_reduce(t, dist.ReduceOp.SUM, deadline_s, "combine_sum")
    return float(t.item())


def combine_min(local_min, deadline_s=DEFAULT_DEADLINE_S):
    t = torch.tensor([float(local_min)], dtype=torch.float32, device=_device())
    _all_reduce(t, dist.ReduceOp.MIN, deadline_s, "combine_min")
    return float(t.item())


def combine_max(local_max, deadline_s=DEFAULT_DEADLINE_S):
    t = torch.tensor([float(local_max)], dtype=torch.float32, device=_device())
    _all_reduce(t, dist.ReduceOp.MAX, deadline_s, "combine_max")
    return float(t.item())


def combine_argmax(local_value, local_index, offset, deadline_s=DEFAULT_DEADLINE_S):
    """Global (index, value) from each rank's local first-argmax; the keys are
    offset by the one bit flip that keeps signed int64 ordering == unsigned."""
    key = argmax_key(local_value, offset + local_index) if local_index is not None else 0
    t = torch.tensor([_to_signed64(key ^ (1 << 63))], dtype=torch.int64, device=_device())
    _all_reduce(t, dist.ReduceOp.MAX, deadline_s, "combine_argmax")
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


# ------------------------------------------------------------- partitioner
def _rank_world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def span(total, rank=None, world=None):
    """This rank's [start, stop) of `total` units (shard() of the current
    process group's rank / size when not given)."""
    r, w = _rank_world()
    return shard(total, r if rank is None else rank, w if world is None else world)


def _ops(ops):
    if ops is None:
        from . import gpu as ops
    return ops


def gather_rows(local, total_rows, row_elems, deadline_s=DEFAULT_DEADLINE_S):
    """The whole [total_rows, row_elems] result on every rank from each
    rank's contiguous rows (shares from shard(); one all-gather of equal,
    padded blocks, then the padding is dropped)."""
    rank, world = _rank_world()
    if world == 1:
        return local.reshape(-1)[: total_rows * row_elems]
    per = -(-total_rows // world) * row_elems
    buf = torch.zeros(per, dtype=local.dtype, device=local.device)
    flat = local.reshape(-1)
    buf[: flat.numel()] = flat
    out = torch.empty(per * world, dtype=local.dtype, device=local.device)
    _wait(dist.all_gather_into_tensor(out, buf, async_op=True), deadline_s, "gather_rows")
    parts = []
    for r in range(world):
        a, b = shard(total_rows, r, world)
        parts.append(out[r * per: r * per + (b - a) * row_elems])
    return torch.cat(parts)


def dot(A, B, M, N, K, ops=None, **gemm_kw):
    """Row-sharded C = A.B (+ the gemm epilogue keywords): this rank computes
    rows [r0, r1) of C from the same rows of A (a view) and all of B.
    Returns (C_local [(r1 - r0) * N], (r0, r1))."""
    ops = _ops(ops)
    r0, r1 = span(M)
    a = A.reshape(-1)[r0 * K: r1 * K]
    if r1 == r0:
        return torch.empty(0, dtype=A.dtype, device=A.device), (r0, r1)
    return ops.gemm(a, B, M=r1 - r0, N=N, K=K, **gemm_kw), (r0, r1)


class GemvColumns:
    """Column-sharded GEMV / linear, y = x.W + b for W [K, N]: this rank keeps
    only its block of columns [c0, c1) of W and b (copied once, contiguous:
    1/world of the weight bytes stream per call), and each call writes
    y[c0:c1]; no collective."""

    def __init__(self, W, b, K, N, ops=None):
        self.ops = _ops(ops)
        self.K, self.N = K, N
        self.c0, self.c1 = span(N)
        n = self.c1 - self.c0
        self.W = W.reshape(K, N)[:, self.c0:self.c1].contiguous().reshape(-1)
        self.b = None if b is None else b.reshape(-1)[self.c0:self.c1].contiguous()
        self.n = n

    def __call__(self, x, y=None):
        if y is None:
            y = torch.empty(self.n, dtype=torch.float32, device=self.W.device)
        if self.n:
            self.ops.sgemv(x.reshape(-1), self.W, y, self.n, self.K, bias=self.b)
        return y


def _rows_view(X, rows, cols):
    r0, r1 = span(rows)
    return X.reshape(-1)[r0 * cols: r1 * cols], r0, r1


def softmax_rows(X, rows, cols, ops=None):
    """Row-sharded softmax(axis=1): (rows [r0, r1) of the result, (r0, r1))."""
    ops = _ops(ops)
    x, r0, r1 = _rows_view(X, rows, cols)
    return (ops.softmax(x, rows=r1 - r0, cols=cols) if r1 > r0 else x.clone()), (r0, r1)


def layer_norm_rows(X, gamma, beta, rows, cols, eps=1e-5, ops=None):
    ops = _ops(ops)
    x, r0, r1 = _rows_view(X, rows, cols)
    if r1 == r0:
        return x.clone(), (r0, r1)
    return ops.layer_norm(x, gamma=gamma, beta=beta, rows=r1 - r0, cols=cols, eps=eps), (r0, r1)


def argmax_rows(X, rows, cols, ops=None):
    """Row-sharded argmax(axis=1): column indices (int32) of rows [r0, r1)."""
    ops = _ops(ops)
    x, r0, r1 = _rows_view(X, rows, cols)
    if r1 == r0:
        return torch.empty(0, dtype=torch.int32, device=X.device), (r0, r1)
    return ops.argmax_f32(x, rows=r1 - r0, cols=cols), (r0, r1)


def sum_rows(X, rows, cols, ops=None):
    """Row-sharded sum(axis=1) of a [rows, cols] matrix."""
    ops = _ops(ops)
    x, r0, r1 = _rows_view(X, rows, cols)
    if r1 == r0:
        return torch.empty(0, dtype=X.dtype, device=X.device), (r0, r1)
    return ops.sum_axis_f32(x, r1 - r0, cols, 1), (r0, r1)


def batched_dot(A, B, batch, M, N, K, ops=None):
    """Batch-sharded C[b] = A[b].B[b] (contiguous [batch, M, K] and
    [batch, K, N]): (C of batches [b0, b1), (b0, b1))."""
    ops = _ops(ops)
    b0, b1 = span(batch)
    if b1 == b0:
        return torch.empty(0, dtype=A.dtype, device=A.device), (b0, b1)
    a = A.reshape(-1)[b0 * M * K: b1 * M * K]
    b = B.reshape(-1)[b0 * K * N: b1 * K * N]
    return ops.gemm(a, b, M=M, N=N, K=K, batch=b1 - b0, stride_a=M * K, stride_b=K * N,
                    stride_c=M * N), (b0, b1)


def bmm_attention(Q, Kt, V, BH, S, d, scale, ops=None):
    """The BMM-attention configuration, O[b] = softmax(Q[b].Kt[b] * scale).V[b]
    for Q, V [BH, S, d] and Kt [BH, d, S], sharded over BH: this rank runs the
    fused kernel on its (batch x head) entries.  (O of [b0, b1), (b0, b1))."""
    ops = _ops(ops)
    b0, b1 = span(BH)
    nb = b1 - b0
    if nb == 0:
        return torch.empty(0, dtype=Q.dtype, device=Q.device), (b0, b1)
    q = Q.reshape(-1)[b0 * S * d: b1 * S * d]
    kt = Kt.reshape(-1)[b0 * d * S: b1 * d * S]
    v = V.reshape(-1)[b0 * S * d: b1 * S * d]
    qs = ops.split(q, nb * S, d)
    ks = ops.transpose_split(kt, d, S, S, batch=nb, s_b=d * S)
    vt = ops.transpose_split(v, S, d, d, batch=nb, s_b=S * d)
    O = ops.attention(qs, ks, vt, Sq=S, Sk=S, batch=nb, heads=1, ldq=d, sq_b=S * d, sq_h=S * d, ldk=d,
                      sk_b=S * d, sk_h=S * d, ldv=S, sv_b=d * S, sv_h=d * S, scale=scale)
    return O, (b0, b1)


class ShardedBlock:
    """The transformer block over a global batch split by sequence: this rank
    holds the replicated weights and runs sequences [s0, s1) of every global
    batch (a Block of s1 - s0 sequences); no collective in the forward."""

    def __init__(self, cfg, params, device, rank=None, world=None, **block_kw):
        from . import transformer
        r, w = _rank_world()
        self.rank = r if rank is None else rank
        self.world = w if world is None else world
        self.full = cfg
        self.s0, self.s1 = shard(cfg.batch, self.rank, self.world)
        self.local = transformer.Config(batch=self.s1 - self.s0, seq=cfg.seq, d_model=cfg.d_model,
                                        heads=cfg.heads, d_ff=cfg.d_ff, eps=cfg.eps)
        self.block = transformer.Block(self.local, params, device=device, **block_kw) if self.local.batch else None

    @property
    def token_span(self):
        """[t0, t1) of this rank's rows in the global [batch * seq, d_model] input."""
        return self.s0 * self.full.seq, self.s1 * self.full.seq

    def local_input(self, x_full):
        """This rank's rows of a replicated global input (a view)."""
        t0, t1 = self.token_span
        return x_full.reshape(-1)[t0 * self.full.d_model: t1 * self.full.d_model]

    def forward(self, x_local, out=None):
        """Forward of this rank's sequences (x_local: its rows, on its GPU)."""
        if self.block is None:
            return x_local.new_empty(0)
        return self.block.forward(x_local, out)
