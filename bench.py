"""Benchmark of the B200 backend on BASELINE.json's metric.

Workload (one "step"): one pre-norm transformer-block forward, fp32, batch 32
x seq 512, d_model 768, 12 heads x 64, FFN 3072 relu,
batch-sharded over the ranks (global batch fixed at 32: strong scaling).
Synthetic data: weights ~ N(0, 0.02^2), biases 0, gamma 1, beta 0,
activations ~ N(0, 1), seeded.  Reported alongside: the 8192^3 fp32-faithful
SGEMM of the same metric (rank 0, N = 1 only).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun (one process per GPU, NCCL for the barrier and
the max-over-ranks time; the forward itself needs no collective).
Timing: CUDA events on the launching stream around each step; the 126 MB L2
is flushed (256 MiB write) before every timed step; W >= 3 untimed warm-ups;
nvidia-smi clocks are sampled during the timed region.  Block.forward runs
eagerly once per buffer set (warm-up) and then replays a CUDA graph of the
same launches; gpu_launches counts the kernels those replays launch.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
os.environ.setdefault("OPENBLAS_NUM_THREADS", str(os.cpu_count() or 1))

METRIC = "fp32 SGEMM TFLOP/s (8192³); transformer-block tokens/s at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-sgemm", action="store_true", help="skip the 8192^3 SGEMM side measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-suite", action="store_true", help="skip the per-configuration suite in the headline line")
    ap.add_argument("--suite", action="store_true",
                    help="measure every configuration of the metric (one JSON line each) instead of the headline")
    ap.add_argument("--profile-case", default=None, choices=["gemm", "block", "shard", "attention", "hbm", "sgemm", "conv"],
                    help="run only a small case for ncu: the FFN-up GEMM of the workload, a 2-sequence block, "
                         "or the 8-GPU per-rank forward (4 sequences)")
    return ap.parse_args()


def ffn_up_case(dev, T=16384, d=768, f=3072):
    """Arguments of the forward's FFN-up GEMM (one tc_gemm_kernel launch):
    A = split layer_norm output [T, d], B = split K-major W1^T [f, d], bias +
    relu epilogue, split output [T, f], the block's accumulation chunk."""
    import torch
    from silarray_b200 import gpu, transformer
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(T * d, device=dev, generator=g)
    W = torch.randn(d * f, device=dev, generator=g) * 0.02
    return dict(A=gpu.split(A, T, d), B=gpu.split(W, d, f, transpose=True), M=T, N=f, K=d, trans_b=True,
                bias=torch.zeros(f, device=dev), act="relu", no_c=True,
                C_split=(torch.empty(T * f, device=dev), torch.empty(T * f, device=dev)),
                acc_chunk_k=transformer.Block.ACC_CHUNK_K)


def profile_case(args):
    """Small, self-terminating cases for ncu captures (one GPU): `gemm` runs the
    dominant kernel as the forward does (FFN-up, M=16384 N=3072 K=768, ~600 MB
    on the device) warmup+1 times; `block` runs a 2-sequence transformer forward;
    `shard` the 8-GPU per-rank forward (4 sequences, ~200 MB);
    `conv` the ResNet mid-layer conv2d of the suite (16x56x56x64 k3 -> 128);
    `attention` the fused attention on a quarter of the BMM-attention config;
    `hbm` the HBM-bound kernels of the suite once each after the warm-ups
    (GEMV 1x4096.4096x4096, small batch 32x4096.4096x768, softmax /
    layer_norm 4096x8192 and 4096x32768, argmax 4096x32768, global sum 2^28:
    ~2.5 GB on the device); `sgemm` the 8192^3 SGEMM (~1 GB)."""
    import torch
    from silarray_b200 import gpu, transformer
    dev = torch.device("cuda", 0)
    if args.profile_case == "gemm":
        gargs = ffn_up_case(dev)
        for _ in range(args.warmup + 1):
            gpu.gemm(**gargs)
    elif args.profile_case == "attention":
        BH, S, d = 32, 1024, 64  # the BMM-attention config at a quarter of its batch
        g = torch.Generator(device=dev).manual_seed(0)
        qs = gpu.split(torch.randn(BH * S * d, device=dev, generator=g), BH * S, d)
        ks = gpu.split(torch.randn(BH * S * d, device=dev, generator=g), BH * S, d)
        vt = gpu.transpose_split(torch.randn(BH * S * d, device=dev, generator=g), S, d, d, batch=BH, s_b=S * d)
        Ob = torch.empty(BH * S * d, device=dev)
        for _ in range(args.warmup + 1):
            gpu.attention(qs, ks, vt, Sq=S, Sk=S, batch=BH, heads=1, ldq=d, sq_b=S * d, sq_h=S * d, ldk=d,
                          sk_b=S * d, sk_h=S * d, ldv=S, sv_b=d * S, sv_h=d * S, scale=0.125, O=Ob)
    elif args.profile_case == "conv":
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(16, 56, 56, 64, device=dev, generator=g)
        w = torch.randn(128, 3, 3, 64, device=dev, generator=g) * 0.05
        for _ in range(args.warmup + 1):
            gpu.conv2d(x, w)
    elif args.profile_case == "sgemm":
        n = 8192  # the metric's SGEMM, plain fp32 operands (split pre-pass + tc_gemm), ~1 GB on the device
        g = torch.Generator(device=dev).manual_seed(0)
        Aa = torch.rand(n * n, device=dev, generator=g) * 2 - 1
        Bb = torch.rand(n * n, device=dev, generator=g) * 2 - 1
        Cc = torch.empty(n * n, device=dev)
        for _ in range(args.warmup + 1):
            gpu.gemm(Aa, Bb, Cc, M=n, N=n, K=n)
    elif args.profile_case == "hbm":
        g = torch.Generator(device=dev).manual_seed(0)
        x, W, bb, y = (torch.randn(4096, device=dev, generator=g), torch.randn(4096 * 4096, device=dev, generator=g),
                       torch.randn(4096, device=dev, generator=g), torch.empty(4096, device=dev))
        r8 = torch.randn(4096 * 8192, device=dev, generator=g) * 2
        r32 = torch.randn(4096 * 32768, device=dev, generator=g) * 2
        o32 = torch.empty_like(r32)
        gm, bt = torch.ones(32768, device=dev), torch.zeros(32768, device=dev)
        flat = torch.rand(1 << 28, device=dev, generator=g) * 2 - 1
        X32, W32, Y32 = (torch.randn(32 * 4096, device=dev, generator=g), torch.randn(4096 * 768, device=dev, generator=g),
                         torch.empty(32 * 768, device=dev))
        for _ in range(args.warmup + 1):
            gpu.sgemv(x, W, y, 4096, 4096, bias=bb)
            gpu.gemm(X32, W32, Y32, M=32, N=768, K=4096)
            gpu.softmax(r8, o32[: r8.numel()], rows=4096, cols=8192)
            gpu.layer_norm(r8, o32[: r8.numel()], gamma=gm[:8192], beta=bt[:8192], rows=4096, cols=8192)
            gpu.softmax(r32, o32, rows=4096, cols=32768)
            gpu.layer_norm(r32, o32, gamma=gm, beta=bt, rows=4096, cols=32768)
            gpu.argmax_f32(r32, rows=4096, cols=32768)
            gpu.sum_f32(flat)
    else:
        cfg = transformer.Config(batch=4 if args.profile_case == "shard" else 2)
        blk = transformer.Block(cfg, transformer.init_params(cfg), device=dev)
        x = torch.from_numpy(transformer.init_input(cfg)).to(dev)
        for _ in range(args.warmup + 1):
            blk.forward(x)
    torch.cuda.synchronize()
    gpu.device_status()
    print("profile case done", flush=True)
    return 0


def run_suite(args, sink=None):
    """Every configuration of BASELINE.json's metric on one GPU: algorithmic
    bytes or FLOPs per call / CUDA-event time (L2 flushed before each timed
    call), against the measured HBM copy bandwidth or the 3xTF32 ceiling.
    Prints one JSON line per configuration, or appends them to `sink`."""
    import numpy as np
    import torch
    from silarray_b200 import gpu
    dev = torch.device("cuda", 0)
    hbm, bf16, src = peaks()
    ceiling = bf16 / 6.0
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)

    def timed(fn, iters=max(3, args.steps)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            flush.zero_()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            fn()
            e0.record()
            torch.cuda.synchronize()
            ts.append(s0.elapsed_time(e0))
        return float(np.median(ts)) / 1e3

    def timed_graph(make_fn, set_bytes, reps=20):
        """Short kernels: `reps` calls captured in one CUDA graph, each on its
        own input set (make_fn(i) returns the call), so that the sets in
        rotation exceed twice the L2 and host launch latency is not timed."""
        nsets = max(2, int(np.ceil(2 * 126e6 / max(1, set_bytes))))
        calls = [make_fn(i % nsets) for i in range(reps)]
        for c in calls[:nsets]:
            c()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(gr, stream=st):
                for c in calls:
                    c()
        torch.cuda.current_stream().wait_stream(st)
        gr.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, args.steps)):
            flush.zero_()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            gr.replay()
            e0.record()
            torch.cuda.synchronize()
            ts.append(s0.elapsed_time(e0))
        return float(np.median(ts)) / 1e3 / reps

    def emit(name, sec, nbytes=None, flops=None, **extra):
        line = {"config": name, "ms": sec * 1e3}
        if nbytes is not None:
            line.update({"GB/s": nbytes / sec / 1e9, "frac_of_hbm": nbytes / sec / 1e9 / hbm, "bytes": nbytes})
        if flops is not None:
            line.update({"TFLOP/s": flops / sec / 1e12, "frac_of_3xtf32_ceiling": flops / sec / 1e12 / ceiling})
        line.update(extra)
        if sink is not None:
            sink.append(line)
        else:
            print(json.dumps(line), flush=True)

    U = lambda *sh: torch.rand(*sh, device=dev, generator=g) * 2 - 1  # noqa: E731
    Nn = lambda std, *sh: torch.randn(*sh, device=dev, generator=g) * std  # noqa: E731
    for n in (1024, 8192):
        a, b, c = U(n, n), U(n, n), torch.empty(n * n, device=dev)
        emit(f"sgemm {n}^3", timed(lambda: gpu.gemm(a, b, c, M=n, N=n, K=n)), flops=2.0 * n ** 3)
        del a, b, c
    gv_bytes = 4.0 * (4096 * 4096 + 4096 + 2 * 4096)
    gsets = {}

    def gemv_set(i):
        if i not in gsets:
            gsets[i] = (Nn(1, 4096), Nn(0.02, 4096, 4096), Nn(0.01, 4096), torch.empty(4096, device=dev))
        x, W, bb, y = gsets[i]
        return lambda: gpu.sgemv(x, W, y, 4096, 4096, bias=bb)
    emit("gemv 1x4096 . 4096x4096 + b", timed_graph(gemv_set, gv_bytes), nbytes=gv_bytes, timing="graph")
    gsets.clear()
    sb_bytes = 4.0 * (32 * 4096 + 4096 * 768 + 32 * 768)

    def sb_set(i):
        if i not in gsets:
            gsets[i] = (Nn(1, 32, 4096), Nn(0.02, 4096, 768), torch.empty(32 * 768, device=dev))
        X, W2, Y = gsets[i]
        return lambda: gpu.gemm(X, W2, Y, M=32, N=768, K=4096)
    emit("small batch 32x4096 . 4096x768", timed_graph(sb_set, sb_bytes), nbytes=sb_bytes,
         flops=2.0 * 32 * 4096 * 768, timing="graph")
    gsets.clear()
    for C in (1024, 8192, 32768):
        R = 4096
        gm, bt = 1 + Nn(0.1, C), Nn(0.1, C)
        if C < 32768:  # < 2 x L2 per call: graph replays over rotating inputs
            sets = {}

            def rows_set(i):
                if i not in sets:
                    sets[i] = (Nn(2, R, C), torch.empty(R, C, device=dev), torch.empty(R, dtype=torch.int32,
                                                                                      device=dev))
                return sets[i]
            for name, nb, mk in (
                    ("softmax", 8.0 * R * C, lambda i: (lambda X=rows_set(i): gpu.softmax(X[0], X[1]))),
                    ("layer_norm", 8.0 * R * C + 8.0 * C,
                     lambda i: (lambda X=rows_set(i): gpu.layer_norm(X[0], X[1], gm, bt))),
                    ("argmax(axis=1)", 4.0 * R * C + 4.0 * R,
                     lambda i: (lambda X=rows_set(i): gpu.argmax_f32(X[0], X[2]))),
                    ("sum(axis=1)", 4.0 * R * C + 4.0 * R,
                     lambda i: (lambda X=rows_set(i): gpu.sum_axis_f32(X[0], R, C, 1, X[1].view(-1)[:R]))),
                    ("sum(axis=1) in the reference's order (drop-in)", 4.0 * R * C + 4.0 * R,
                     lambda i: (lambda X=rows_set(i): gpu.sum_axis_seq_f32(X[0], R, C, 1, X[1].view(-1)[:R])))):
                emit(f"{name} 4096x{C}", timed_graph(mk, nb), nbytes=nb, timing="graph")
            sets.clear()
            continue
        X = Nn(2, R, C)
        Y = torch.empty_like(X)
        emit(f"softmax 4096x{C}", timed(lambda: gpu.softmax(X, Y)), nbytes=8.0 * R * C)
        emit(f"layer_norm 4096x{C}", timed(lambda: gpu.layer_norm(X, Y, gm, bt)), nbytes=8.0 * R * C + 8.0 * C)
        emit(f"argmax(axis=1) 4096x{C}", timed(lambda: gpu.argmax_f32(X)), nbytes=4.0 * R * C + 4.0 * R)
        emit(f"sum(axis=1) 4096x{C}", timed(lambda: gpu.sum_axis_f32(X, R, C, 1)), nbytes=4.0 * R * C + 4.0 * R)
        emit(f"sum(axis=1) in the reference's order (drop-in) 4096x{C}", timed(lambda: gpu.sum_axis_seq_f32(X, R, C, 1)),
             nbytes=4.0 * R * C + 4.0 * R)
        del X, Y
    Z = U(1 << 28)
    for name, fn in (("sum", gpu.sum_f32), ("min", gpu.min_f32), ("max", gpu.max_f32),
                     ("argmax", gpu.argmax_all_f32)):
        emit(f"global {name} 2^28", timed(lambda: fn(Z)), nbytes=4.0 * (1 << 28))
    del Z
    BH, S, d = 128, 1024, 64
    Q, Kt, V = Nn(1, BH, S, d), Nn(1, BH, d, S), Nn(1, BH, S, d)
    Ob = torch.empty(BH * S * d, device=dev)

    def attention():
        # operands to their split K-major forms (K from the stored K^T, V^T from V), then one fused kernel
        qs = gpu.split(Q, BH * S, d)
        ks = gpu.transpose_split(Kt, d, S, S, batch=BH, s_b=d * S)
        vt = gpu.transpose_split(V, S, d, d, batch=BH, s_b=S * d)
        gpu.attention(qs, ks, vt, Sq=S, Sk=S, batch=BH, heads=1, ldq=d, sq_b=S * d, sq_h=S * d,
                      ldk=d, sk_b=S * d, sk_h=S * d, ldv=S, sv_b=d * S, sv_h=d * S, scale=0.125, O=Ob)
    emit("bmm attention 128x1024x1024x64 (fused)", timed(attention), flops=4.0 * BH * S * S * d,
         note="includes the splits of Q, K^T->K and V->V^T")
    del Q, Kt, V, Ob
    # beyond the metric's configurations: conv2d of the reference's bench/micro/bench_nn_ops.cpp
    for (Nb, Ci, Co, Hh, Ww, Kk, desc) in ((1, 3, 32, 224, 224, 3, "ImageNet first layer"),
                                           (16, 64, 128, 56, 56, 3, "ResNet mid layer"),
                                           (16, 128, 256, 28, 28, 3, "ResNet deep layer")):
        x = Nn(1, Nb, Hh, Ww, Ci)
        wt = Nn(0.1, Co, Kk, Kk, Ci)
        y = torch.empty(Nb * Hh * Ww * Co, device=dev)
        emit(f"conv2d {desc} {Nb}x{Ci}x{Hh}x{Ww} k{Kk} -> {Co} (extra)", timed(lambda: gpu.conv2d(x, wt, y)),
             flops=2.0 * Nb * Hh * Ww * Co * Kk * Kk * Ci, note="implicit GEMM, patch split included")
        del x, wt, y
    return 0


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9:
                    rows.append(f)
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        import statistics
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ peaks
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------ CPU baseline
def workload_config(full, world):
    """The `config` both arms report (identical keys and values at a given N)."""
    return {"workload": "transformer_block_fwd", "global_batch": full.batch, "seq_len": full.seq,
            "d_model": full.d_model, "heads": full.heads, "d_ff": full.d_ff, "parallelism": f"dp{world}",
            "l2": "GPU arm: flushed (256 MiB write) before every timed step"}


def _reference_sequence(one, params, x, k):
    """One bounded sample of the workload on the reference CPU path: sequence
    k % batch of the batch (512 tokens through the whole block)."""
    from oracle import transformer_ref as TR
    n = x.shape[0] // one.seq
    i = k % n
    TR.reference_forward(one, params, x[i * one.seq:(i + 1) * one.seq])


def cpu_baseline(cfg, params, x, budget_s=12.0):
    """The reference's own CPU implementation of the block (oracle/_ref, all
    host threads for cblas_sgemm) on a bounded sample: whole sequences of the
    same workload, as many as fit in ~budget_s (at least one)."""
    import oracle as O
    from silarray_b200 import transformer
    kind = "reference" if O.ref is not None else "port"
    one = transformer.Config(batch=1, seq=cfg.seq, d_model=cfg.d_model, heads=cfg.heads, d_ff=cfg.d_ff)
    n, t0 = 0, time.perf_counter()
    while True:
        _reference_sequence(one, params, x, n)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= cfg.batch:
            break
    return {"value": n * cfg.seq / el, "unit": "tokens/s", "cores": int(os.environ["OPENBLAS_NUM_THREADS"]),
            "kind": kind, "sample": f"{n} of {cfg.batch} sequences ({n * cfg.seq} tokens) in {el:.1f} s; "
                                    f"cblas_sgemm threads = OPENBLAS_NUM_THREADS, other ops single-threaded "
                                    f"as in the reference"}


def run_reference(args):
    """The reference arm: silarray's own CPU path (oracle/_ref, built from the
    reference sources) on the host cores, rank 0 only.  One step = one whole
    512-token sequence of the batch (a bounded sample of the workload, ~0.4 s
    on 16 cores); W untimed warm-up steps, then K timed steps; the value is
    tokens processed / wall time of the K steps."""
    import oracle as O
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from silarray_b200 import transformer
    full = transformer.Config()
    params = transformer.init_params(full, seed=0)
    x = transformer.init_input(full, seed=1)
    one = transformer.Config(batch=1, seq=full.seq, d_model=full.d_model, heads=full.heads, d_ff=full.d_ff)
    for k in range(args.warmup):
        _reference_sequence(one, params, x, k)
    t0 = time.perf_counter()
    for k in range(args.steps):
        _reference_sequence(one, params, x, args.warmup + k)
    el = time.perf_counter() - t0
    v = args.steps * full.seq / el
    cores = int(os.environ["OPENBLAS_NUM_THREADS"])
    cb = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "reference" if O.ref is not None else "port",
          "sample": f"one {full.seq}-token sequence of the batch-{full.batch} workload per step, {args.steps} "
                    f"timed steps in {el:.1f} s; cblas_sgemm on {cores} threads, other ops single-threaded as "
                    f"in the reference"}
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": full.tokens / v * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": workload_config(full, world),
            "timed_region_s": el, "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- our arm
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from silarray_b200 import _lib, gpu, transformer
    from silarray_b200 import dist as sd

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        sd.init("nccl", timeout_s=300, device=dev)
    lib = _lib.lib()

    full = transformer.Config()
    params = transformer.init_params(full, seed=0)
    x_all = transformer.init_input(full, seed=1)
    shard = sd.ShardedBlock(full, params, dev, rank=rank, world=world)  # this rank's sequences of the batch
    cfg, blk = shard.local, shard.block
    t0, t1 = shard.token_span
    x_local = np.ascontiguousarray(x_all[t0:t1])
    x_dev = torch.from_numpy(x_local).to(dev)
    out = torch.empty(cfg.tokens * cfg.d_model, dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        blk.forward(x_dev, out)
    barrier()
    # ---------------- device-resident timed region
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches0 = lib.silcu_kernel_launches() + blk.replayed_launches
    with ClockSampler(local) as clk:
        barrier()
        for s, e in ev:
            flush.zero_()
            s.record(stream)
            blk.forward(x_dev, out)
            e.record(stream)
        barrier()
    launches = lib.silcu_kernel_launches() + blk.replayed_launches - launches0
    ms = sum(s.elapsed_time(e) for s, e in ev) / len(ev)
    ms = max_over_ranks(ms)
    tokens = full.tokens
    value = tokens / (ms / 1e3)
    clocks = clk.summary()

    # ---------------- end to end through the public API with host buffers
    # Block.forward_host_stream: args.steps consecutive batches from pinned host
    # input to pinned host output, every batch copied in and its result copied
    # out, the copies of batch k +- 1 overlapping the compute of batch k.  One
    # timed region over the stream (no L2 flush inside it: each step's working
    # set, e.g. the 302 MB split QKV activations, exceeds the 126 MB L2).
    x_host = torch.from_numpy(x_local).pin_memory()
    o_hosts = [torch.empty(cfg.tokens * cfg.d_model, dtype=torch.float32).pin_memory() for _ in range(2)]
    xs_in = [x_host] * args.steps
    outs = [o_hosts[k % 2] for k in range(args.steps)]
    # warm-up over 4 batches: every (buffer, whole / half batch) combination
    # the timed stream uses runs once eagerly and is captured before timing
    blk.forward_host_stream([x_host] * 4, o_hosts * 2)
    barrier()
    flush.zero_()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    blk.forward_host_stream(xs_in, outs)
    e2.record(stream)
    barrier()
    ev2 = [(s2, e2)]
    o_host = o_hosts[0]
    ms_e2e = max_over_ranks(sum(s.elapsed_time(e) for s, e in ev2) / len(ev2) / args.steps)
    e2e = {"value": tokens / (ms_e2e / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": int(x_host.numel() * 4 * world), "d2h_bytes_per_step": int(o_host.numel() * 4 * world),
           "api": "Block.forward_host_stream over %d consecutive batches (pinned host buffers; copies of "
                  "neighbouring batches overlap the compute; per-step time = region / steps)" % args.steps}

    hbm, bf16, src = peaks()
    result = None
    if rank == 0:
        # ---------------- dominant kernel: the 3xTF32 GEMM as the forward runs it (FFN-up:
        # split activations x split K-major weights, bias + relu, split output) -- one launch
        T, d, f = cfg.tokens, cfg.d_model, cfg.d_ff
        gargs = ffn_up_case(dev, T, d, f)
        for _ in range(3):
            gpu.gemm(**gargs)
        torch.cuda.synchronize()
        ge = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
        for s, e in ge:
            flush.zero_()
            s.record(stream)
            gpu.gemm(**gargs)
            e.record(stream)
        torch.cuda.synchronize()
        gms = sum(s.elapsed_time(e) for s, e in ge) / len(ge)
        gflop = 2.0 * T * f * d
        ceiling = bf16 / 2.0 / 3.0  # tf32 runs at half the bf16 rate; 3 MMAs per product
        achieved = gflop / (gms / 1e3) / 1e12
        traffic_path = os.path.join(ROOT, "profiles", "traffic.json")
        traffic = None
        if os.path.exists(traffic_path):
            # captured at the full single-GPU shape (M = 16384); scaled by rows otherwise
            traffic = json.load(open(traffic_path)).get("tc_gemm_kernel_ffn_up")
            if traffic is not None and T != 16384:
                traffic = traffic * T / 16384.0
        roofline = {"bound": "tensor", "kernel": "tc_gemm_kernel<256, pair> M=%d N=%d K=%d (FFN-up of the forward)" % (T, f, d),
                    "achieved": achieved, "peak": ceiling, "unit": "TFLOP/s", "frac": achieved / ceiling,
                    "traffic": traffic,
                    "peak_note": f"3xTF32 ceiling = {src} bf16 {bf16} TFLOP/s / 2 (tf32 rate) / 3 (MMAs per product)",
                    "frac_of_bf16_peak": achieved * 6.0 / bf16}
        sg = None
        if not args.no_sgemm and world == 1:
            n = 8192
            Aa = torch.rand(n, n, device=dev) * 2 - 1
            Bb = torch.rand(n, n, device=dev) * 2 - 1
            Cc = torch.empty(n * n, device=dev)
            for _ in range(2):
                gpu.gemm(Aa, Bb, Cc, M=n, N=n, K=n)
            torch.cuda.synchronize()
            se = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(5)]
            for s, e in se:
                s.record(stream)
                gpu.gemm(Aa, Bb, Cc, M=n, N=n, K=n)
                e.record(stream)
            torch.cuda.synchronize()
            sms = sorted(s.elapsed_time(e) for s, e in se)[len(se) // 2]
            sg = {"tflops": 2.0 * n ** 3 / (sms / 1e3) / 1e12, "ms": sms, "unit": "TFLOP/s",
                  "frac_of_3xtf32_ceiling": 2.0 * n ** 3 / (sms / 1e3) / 1e12 / ceiling,
                  "note": "inputs U[-1,1) 768 MiB > L2; median of 5; includes the hi/lo split pre-pass"}
            del Aa, Bb, Cc
        cpu = None
        if not args.no_cpu and world == 1:
            cpu = cpu_baseline(cfg, params, x_local, budget_s=12.0)
        suite = None
        if not args.no_suite and world == 1:
            # every other configuration of the metric, one entry each (~15 s)
            del gargs
            torch.cuda.empty_cache()
            suite = []
            run_suite(argparse.Namespace(steps=5, warmup=3), sink=suite)
        result = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(full, world),
            "timing": {"launch": "CUDA-graph replay of the forward's kernels (captured after its first eager run)"},
            "clocks": clocks, "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline,
            "sgemm_8192": sg, "cpu_baseline": cpu, "suite": suite,
        }
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        return profile_case(args)
    if args.suite:
        return run_suite(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
