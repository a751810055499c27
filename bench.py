"""Benchmark: W4A16 GEMM HBM GB/s at M=1 (and TFLOP/s at M=4096) on 1/2/4/8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

One JSON line (rank 0). ``value`` is:

* N = 1: the decode configuration, M=1, K=4096, N=11008, G=128 (X ~ N(0,1),
  W ~ N(0, 0.02) quantised to uint4 on the GPU). One step = one fused GEMM.
* N > 1: the batched-decode sweep configuration at M=1, K=8192, N=28672, G=128
  (W ~ N(0, 0.015) with 0.1% outliers ~ N(0, 0.2^2)), column-sharded: rank r owns
  columns [r*N/p, (r+1)*N/p) and computes its slice of Y (strong scaling: the
  total work is fixed). ``value`` = the bytes all ranks read and write (the
  reference's byte model per rank: X + its weight columns + scales + zeros + its
  Y columns) / the slowest rank's time.

Extra keys carry every other configuration of the benchmark list: ``sweep``
(M in {1,4,8,16,32} at K=8192, N=28672/p, at every N; ``mid_m`` adds M in {48, 96} at N = 1),
``gather`` (N > 1: the
same GEMM with the full Y on every rank, through the fused GEMM + all-gather
kernel and through GEMM + NCCL all-gather), ``mlp_stack`` (80 decoder MLP blocks,
gate/up column-parallel with SwiGLU fused into its epilogue, down row-parallel with
its all-reduce, M=1 and M=2048),
``prefill`` (N = 1: M in {512,2048,4096,8192} at K=4096, N=14336 on the prefill
kernel the per-shape choice picks, with the other prefill kernel's time beside it;
``secondary`` repeats M=4096). Each has a roofline against the measured
peaks. Before anything is timed, every rank checks its outputs (its shard, the
gathered Y, the MLP block's activations and reduced output) against the numpy
oracle on sampled columns; a mismatch on any rank ends the run non-zero.

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and a device
synchronise, timed with CUDA events on the launching stream, max over ranks.
Inputs are larger than L2: each step uses the next of R distinct weight copies
totalling > 2 x 126 MB. The K steps are replayed from a CUDA graph captured
beforehand so the host's launch rate does not cap a ~5-20 us kernel.

``e2e`` is the headline metric through the public Python API with host buffers:
every step stages X in from pinned host memory and reads Y (this rank's columns)
back into pinned host memory, inside the timed region.

``--impl reference`` times the reference's CPU path (dequantise, then fp32
matmul: reference.py:43-53) restated in numpy by the oracle, on all host cores,
on the same workload and with the same ``config`` as this arm at the same N.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200"))
sys.path.insert(0, ROOT)

METRIC = "W4A16 GEMM HBM GB/s at M=1 & TFLOPS at M=4096, 1/2/4/8 B200"
DECODE = dict(M=1, K=4096, N=11008, G=128, sigma=0.02, outliers=0.0)
SWEEP = dict(K=8192, N=28672, G=128, sigma=0.015, outliers=0.001, Ms=(1, 4, 8, 16, 32))
PREFILL = dict(K=4096, N=14336, G=128, sigma=0.02, Ms=(512, 2048, 4096, 8192))
MLP = dict(D=8192, H=28672, G=128, layers=80, sets=4, Ms=(1, 2048))
L2_BYTES = 126 * 1024 * 1024
PUBLISHED_T4_GBS = 31.0  # README.md:186, the reference's Triton kernel, same metric and shape, on a T4
ORACLE_COLS = 256        # columns of each checked output compared with the oracle


def gemm_bytes(M, K, N, G):
    """Algorithmic bytes per GEMM (the reference's byte model, bench_gemm.py:61-67):
    X + packed weights + scales + zeros + Y."""
    return M * K * 2 + (K // 8) * N * 4 + 2 * (K // G) * N * 2 + M * N * 2


def workload(world):
    """(K, N, N per rank, G, sigma, outlier fraction, config dict) of `value` (M = 1) at
    `world` GPUs. The reference arm prints the same config dict."""
    if world == 1:
        c = DECODE
        cfg = {"workload": "decode GEMM M=1 K=4096 N=11008 G=128 (BASELINE configs[1])",
               "M": 1, "K": c["K"], "N": c["N"], "group_size": c["G"], "parallelism": "single GPU"}
        cfg.update(_TIMING_CFG)
        return c["K"], c["N"], c["N"], c["G"], c["sigma"], c["outliers"], cfg
    c = SWEEP
    cfg = {"workload": f"batched-decode sweep M=1 K=8192 N=28672 G=128 column-sharded over {world} GPUs "
                       f"(BASELINE configs[2]), no gather",
           "M": 1, "K": c["K"], "N": c["N"], "N_per_gpu": c["N"] // world, "group_size": c["G"],
           "parallelism": f"column-parallel x{world}"}
    cfg.update(_TIMING_CFG)
    return c["K"], c["N"], c["N"] // world, c["G"], c["sigma"], c["outliers"], cfg


_TIMING_CFG = {"l2": "inputs larger than L2: rotating weight copies, > 2 x 126 MiB per rank",
               "timing": "GPU arm: CUDA graph of the K steps, CUDA events on the launching stream, "
                         "max over ranks; reference arm: wall clock per CPU step"}


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        p = {"hbm_gbs": float(m["hbm_gbs"]), "bf16_tflops": float(m["bf16_tflops"]),
             "bf16_tflops_sustained": float(m.get("bf16_tflops_sustained", m["bf16_tflops"])),
             "source": "measured"}
    except (OSError, KeyError, ValueError):
        pass
    return p


def profile_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>), or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def hbm_roofline(bytes_per_launch, seconds_per_launch, pk, kernel, traffic=None, traffic_source=None):
    achieved = bytes_per_launch / seconds_per_launch / 1e9
    r = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
         "frac": achieved / pk["hbm_gbs"],
         "peak_source": "measured hbm_gbs (MEASURED_PEAKS.json)" if pk["source"] == "measured"
         else "fallback 6650 GB/s", "traffic": traffic, "algorithmic_bytes_per_launch": bytes_per_launch,
         "kernel": kernel}
    if traffic_source:
        r["traffic_source"] = traffic_source
    return r


def tensor_roofline(flops, seconds, pk, kernel, sustained=False):
    tf = flops / seconds / 1e12
    peak = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
    return {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
            "peak_source": ("measured bf16_tflops" + ("_sustained" if sustained else " (burst)")
                            + ", fp16 proxy") if pk["source"] == "measured" else "fallback",
            "frac_of_2250_nominal": tf / 2250.0, "kernel": kernel}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# --------------------------------------------------------------------------------------
# CPU side: the reference's dequantise-then-matmul (numpy restatement in oracle/)
# --------------------------------------------------------------------------------------
def cpu_dequant_then_matmul(X, qw, s, z, G, threads):
    """The reference's CPU path (reference.py:43-53), restated in numpy by the oracle,
    run over column blocks on `threads` host threads (numpy releases the GIL)."""
    import oracle
    from concurrent.futures import ThreadPoolExecutor
    N = qw.shape[1]
    nb = max(1, threads)
    bounds = np.linspace(0, N, nb + 1).astype(int)
    out = np.empty((X.shape[0], N), dtype=np.float16)

    def work(i):
        a, b = bounds[i], bounds[i + 1]
        if b > a:
            out[:, a:b] = oracle.dequant_then_matmul(X, np.ascontiguousarray(qw[:, a:b]),
                                                     np.ascontiguousarray(s[:, a:b]),
                                                     np.ascontiguousarray(z[:, a:b]), G)
    with ThreadPoolExecutor(nb) as ex:
        list(ex.map(work, range(nb)))
    return out


def cpu_inputs(M, K, N, G, sigma, outliers, seed=0):
    import oracle
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(sigma)
    if outliers > 0:
        mask = rng.random((K, N), dtype=np.float32) < outliers
        W[mask] = rng.standard_normal(int(mask.sum()), dtype=np.float32) * np.float32(0.2)
    qw, s, z = oracle.quantize_weight(W.astype(np.float16), G)
    return X, qw, s, z


def cpu_model() -> str:
    """The host CPU's model name (Linux), for the baseline's record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_cpu(M, K, N, G, sigma, outliers, min_seconds=10.0, max_iters=50, steps=None, threads=None):
    """Time the CPU path; returns (median seconds per GEMM, iterations, threads).

    Runs for at least ``min_seconds`` (bounded by ``max_iters``) or exactly
    ``steps`` iterations. BLAS is pinned to one thread per worker; the column
    blocks give the parallelism (all host cores unless ``threads`` is given)."""
    from threadpoolctl import threadpool_limits
    threads = threads or os.cpu_count() or 1
    X, qw, s, z = cpu_inputs(M, K, N, G, sigma, outliers)
    times = []
    with threadpool_limits(limits=1):
        cpu_dequant_then_matmul(X, qw, s, z, G, threads)   # warm-up
        t_end = time.perf_counter() + min_seconds
        while (len(times) < steps) if steps is not None else \
                (time.perf_counter() < t_end and len(times) < max_iters):
            t0 = time.perf_counter()
            cpu_dequant_then_matmul(X, qw, s, z, G, threads)
            times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), threads


CPU_KIND_NOTE = ("numpy restatement (oracle/) of the reference's CPU dequant_then_matmul "
                 "(w4a16-kernel/src/w4a16/reference.py:43-53): fp16 (q - z) * s, then an fp32 matmul; "
                 "the reference's own PyTorch code is not on the GPU box")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = args.gpus
    K, N, _, G, sigma, outliers, cfg = workload(world)
    M = 1
    # each step is one full GEMM of the workload on the CPU (~0.1-0.5 s); cap the count
    # so the whole run stays within a few minutes
    t, n, threads = time_cpu(M, K, N, G, sigma, outliers, steps=max(1, min(args.steps, 40)))
    gbs = gemm_bytes(M, K, N, G) / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n} full GEMMs of the workload (each one bounded step), numpy over "
                                   f"{threads} column blocks", "what": CPU_KIND_NOTE,
                         "cpu_model": cpu_model()},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------
# GPU side
# --------------------------------------------------------------------------------------
class Ctx:
    """Rank, device, process group and the helpers every measurement shares."""

    def __init__(self, torch, dist):
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
        self.stream = torch.cuda.Stream(device=self.dev)
        self.pk = peaks()

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v):
        t = self.torch.tensor([float(v)], device=self.dev, dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_ok(self, ok):
        t = self.torch.tensor([1 if ok else 0], device=self.dev, dtype=self.torch.int32)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN)
        return bool(t.item())

    def time_graph(self, step, steps):
        """Capture `steps` calls of step(i) in one CUDA graph, replay it once untimed,
        then time one replay with CUDA events on the capture stream (max over ranks).
        Returns milliseconds for the whole replay."""
        torch = self.torch
        with torch.cuda.stream(self.stream):
            for i in range(3):
                step(i)   # warm-up on the capture stream (its workspace, peer channels)
        torch.cuda.synchronize(self.dev)
        self.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(self.stream):
            with torch.cuda.graph(g, stream=self.stream):
                for i in range(steps):
                    step(i)
            g.replay()
        torch.cuda.synchronize(self.dev)
        self.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            e0.record(self.stream)
            g.replay()
            e1.record(self.stream)
        torch.cuda.synchronize(self.dev)
        self.barrier()
        ms = self.max_over_ranks(e0.elapsed_time(e1))
        del g
        return ms


def make_weight(torch, K, N, sigma, outliers, seed, dev):
    """sigma * N(0,1) fp16 [K, N], with a Bernoulli(outliers) set redrawn from N(0, 0.2^2);
    the same on every rank (same seed), so every rank can check any column."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    W = torch.randn(K, N, generator=gen, device=dev) * sigma
    if outliers > 0:
        mask = torch.rand(K, N, generator=gen, device=dev) < outliers
        W = torch.where(mask, torch.randn(K, N, generator=gen, device=dev) * 0.2, W)
    return W.half()


def oracle_check(ctx, what, y_cols, X, qw_cols, s_cols, z_cols, G, bias_cols=None):
    """y_cols [M, c] (device, fp16) against the numpy oracle of the same columns."""
    import oracle
    ref = oracle.reference_w4a16(X.cpu().numpy(), qw_cols.cpu().numpy(), s_cols.cpu().numpy(),
                                 z_cols.cpu().numpy(), G).astype(np.float32)
    if bias_cols is not None:
        ref = (ref.astype(np.float16) + bias_cols.cpu().numpy()).astype(np.float32)
    out = y_cols.float().cpu().numpy()
    err = np.abs(out - ref)
    ok = bool(np.all(np.isfinite(out)) and np.all(err <= 1e-2 + 1e-3 * np.abs(ref)))
    if not ok:
        sys.stderr.write(f"[rank {ctx.rank}] oracle mismatch in {what}: max |d| = {float(err.max())}\n")
    return ok, float(err.max())


class ShardedWeights:
    """One column-sharded quantised [K, N] weight: this rank's shard in R copies (so the
    rotation exceeds L2), plus a few sampled columns of the full weight for the oracle."""

    def __init__(self, ctx, K, N, G, sigma, outliers, seed, min_rotation_bytes):
        torch = ctx.torch
        import w4a16
        self.K, self.N, self.G = K, N, G
        self.n = N // ctx.world
        W = make_weight(torch, K, N, sigma, outliers, seed, ctx.dev)
        qw, s, z = w4a16.quantize_weight(W, G)
        del W
        lo, hi = ctx.rank * self.n, (ctx.rank + 1) * self.n
        shard = (qw[:, lo:hi].contiguous(), s[:, lo:hi].contiguous(), z[:, lo:hi].contiguous())
        self.shard_bytes = sum(t.numel() * t.element_size() for t in shard)
        self.R = max(2, -(-min_rotation_bytes // self.shard_bytes))
        self.copies = [shard] + [tuple(t.clone() for t in shard) for _ in range(self.R - 1)]
        gen = np.random.default_rng(seed)
        self.cols_all = torch.from_numpy(np.sort(gen.choice(N, min(ORACLE_COLS, N), replace=False))).to(ctx.dev)
        own = np.arange(lo, hi)
        self.cols_own = torch.from_numpy(np.sort(gen.choice(own, min(ORACLE_COLS, self.n), replace=False))).to(ctx.dev)
        self.sample_all = tuple(t[:, self.cols_all].contiguous() for t in (qw, s, z))
        self.sample_own = tuple(t[:, self.cols_own].contiguous() for t in (qw, s, z))
        self.lo = lo
        del qw, s, z
        torch.cuda.empty_cache()


def measure_sweep(ctx, args, sw, X_by_M, ys):
    """The decode GEMM on this rank's shard for each M: graph-timed, oracle-checked."""
    import w4a16
    out, ok = [], True
    K, n, G = sw.K, sw.n, sw.G
    for M, X in X_by_M.items():
        y = ys[M]
        w4a16.w4a16_matmul(X, *sw.copies[0], G, out=y)
        good, err = oracle_check(ctx, f"sweep M={M} shard", y[:, sw.cols_own - sw.lo], X, *sw.sample_own, G)
        ok &= good

        def step(i, X=X, y=y):
            w4a16.w4a16_matmul(X, *sw.copies[i % sw.R], G, out=y)
        steps = args.steps
        ms = ctx.time_graph(step, steps)
        per = ms / 1e3 / steps
        b_rank = gemm_bytes(M, K, n, G)
        out.append({"M": M, "us_per_call": per * 1e6, "gbs_total": ctx.world * b_rank / per / 1e9,
                    "tflops_total": 2.0 * M * K * sw.N / per / 1e12, "oracle_max_abs_err": err,
                    "roofline_per_gpu": hbm_roofline(b_rank, per, ctx.pk, "decode_gemv_tma_kernel")})
    return out, ok


def measure_gather(ctx, args, sw, X_by_M):
    """N > 1: the same GEMM with the full Y on every rank -- the fused GEMM + all-gather
    kernel (ColumnParallelW4A16Linear(gather=True)) and GEMM + NCCL all-gather."""
    torch = ctx.torch
    from w4a16.parallel import ColumnParallelW4A16Linear, gather_columns
    import w4a16
    out, ok = [], True
    K, N, G = sw.K, sw.N, sw.G
    layers = []
    for r in range(sw.R):
        lin = ColumnParallelW4A16Linear(K, N, G, bias=False, device=ctx.dev)
        for name, t in zip(("qweight", "scales", "zeros"), sw.copies[r]):
            setattr(lin, name, t)   # the shard copies themselves (no extra memory)
        layers.append(lin)
    for M in (1, 32):
        X = X_by_M[M]
        yf = layers[0](X, gather=True)
        good, err_f = oracle_check(ctx, f"fused gather M={M}", yf[:, sw.cols_all], X, *sw.sample_all, G)
        ok &= good
        yn = gather_columns(w4a16.w4a16_matmul(X, *sw.copies[0], G))
        good, err_n = oracle_check(ctx, f"NCCL gather M={M}", yn[:, sw.cols_all], X, *sw.sample_all, G)
        ok &= good
        ok &= bool(torch.equal(yf, yn))

        def fused(i, X=X):
            layers[i % sw.R](X, gather=True)

        def nccl(i, X=X):
            gather_columns(w4a16.w4a16_matmul(X, *sw.copies[i % sw.R], G))
        steps = max(10, min(args.steps, 100))
        t_f = ctx.time_graph(fused, steps) / 1e3 / steps
        t_n = ctx.time_graph(nccl, steps) / 1e3 / steps
        b_rank = gemm_bytes(M, K, sw.n, G)
        out.append({"M": M, "fused_us_per_call": t_f * 1e6, "nccl_us_per_call": t_n * 1e6,
                    "fused_gbs_total": ctx.world * b_rank / t_f / 1e9,
                    "nccl_gbs_total": ctx.world * b_rank / t_n / 1e9,
                    "oracle_max_abs_err": max(err_f, err_n), "fused_equals_nccl": bool(torch.equal(yf, yn)),
                    "gathered_bytes_per_rank": M * N * 2,
                    "path": "fused: w4a16_gemm_allgather (one kernel per rank, peer stores over NVLink); "
                            "nccl: w4a16_gemm + all_gather_into_tensor (+ reorder for M > 1)"})
    from w4a16.parallel import close_peer_channels
    close_peer_channels()
    return out, ok


def measure_mlp(ctx, args):
    """80 decoder MLP blocks (4 distinct weight sets cycled, >= 1.4 GB per GPU at tp1),
    gate/up column-parallel fused into one GEMM with the SwiGLU in its epilogue, down
    row-parallel with its all-reduce (fused over NVLink up to 32 tokens, NCCL beyond),
    one CUDA graph per step.
    Block 0's activations and reduced output are checked against the oracle first."""
    torch = ctx.torch
    import w4a16
    from w4a16.parallel import W4A16MLP, close_peer_channels
    c = MLP
    D, H, G, L = c["D"], c["H"], c["G"], c["layers"]
    blocks, check = [], None
    for i in range(c["sets"]):
        gen = torch.Generator(device=ctx.dev).manual_seed(1000 + i)
        wg = (torch.randn(D, H, generator=gen, device=ctx.dev) * 0.02).half()
        wu = (torch.randn(D, H, generator=gen, device=ctx.dev) * 0.02).half()
        wd = (torch.randn(H, D, generator=gen, device=ctx.dev) * 0.02).half()
        mlp = W4A16MLP(D, H, G, device=ctx.dev)
        gq, uq, dq = (w4a16.quantize_weight(w, G) for w in (wg, wu, wd))
        mlp.load_quantized(gq, uq, dq)
        if i == 0:
            rng = np.random.default_rng(5)
            h_per = H // ctx.world
            hc = torch.from_numpy(np.sort(rng.choice(h_per, 128, replace=False))).to(ctx.dev)
            yc = torch.from_numpy(np.sort(rng.choice(D, 128, replace=False))).to(ctx.dev)
            hcol = hc + ctx.rank * h_per
            check = dict(hc=hc, yc=yc, g=tuple(t[:, hcol].contiguous() for t in gq),
                         u=tuple(t[:, hcol].contiguous() for t in uq), d=tuple(t[:, yc].contiguous() for t in dq))
        blocks.append(mlp)
        del wg, wu, wd, gq, uq, dq
        torch.cuda.empty_cache()
    per_block_bytes = sum(b.numel() * b.element_size() for b in blocks[0].buffers())
    lines, ok = [], True
    for M in c["Ms"]:
        gen = torch.Generator(device=ctx.dev).manual_seed(7)
        x = torch.randn(M, D, generator=gen, device=ctx.dev).half()
        # oracle check of block 0 (first 4 rows): SwiGLU activations on sampled columns of this
        # rank's shard, then the reduced output on sampled columns given every rank's activations
        b0 = blocks[0]
        xs = x[:4]
        h = w4a16.w4a16_matmul_swiglu(xs, b0.gate_up.qweight, b0.gate_up.scales, b0.gate_up.zeros, G,
                                      kernel_order=b0.gate_up_kernel_order)
        y = b0.down(h)
        import oracle
        g_ref = oracle.reference_w4a16(xs.cpu().numpy(), *(t.cpu().numpy() for t in check["g"]), G)
        u_ref = oracle.reference_w4a16(xs.cpu().numpy(), *(t.cpu().numpy() for t in check["u"]), G)
        gf = g_ref.astype(np.float32)
        h_ref = (gf / (1.0 + np.exp(-gf)) * u_ref.astype(np.float32)).astype(np.float16).astype(np.float32)
        h_out = h[:, check["hc"]].float().cpu().numpy()
        # silu(g) * u of g, u within the GEMM tolerance of the oracle's: 4e-2 + 4e-3 |ref|
        h_ok = bool(np.all(np.abs(h_out - h_ref) <= 4e-2 + 4e-3 * np.abs(h_ref)))
        if not h_ok:
            sys.stderr.write(f"[rank {ctx.rank}] MLP M={M}: activations differ from the oracle\n")
        if ctx.world > 1:
            hs = [torch.empty_like(h) for _ in range(ctx.world)]
            ctx.dist.all_gather(hs, h.contiguous())
            h_full = torch.cat(hs, dim=1)
        else:
            h_full = h
        good, err = oracle_check(ctx, f"MLP M={M} reduced output", y[:, check["yc"]], h_full, *check["d"], G)
        ok &= good and h_ok

        def step(i, x=x):
            for l in range(L):
                blocks[l % c["sets"]](x)
        steps = max(1, min(args.steps, 5))
        ms = ctx.time_graph(step, steps) / steps
        flops = 2.0 * M * (2 * D * H + H * D) * L
        line = {"M": M, "ms_per_step": ms, "layers": L, "parallelism": f"tp{ctx.world}",
                "weights_per_gpu_per_block_bytes": per_block_bytes,
                "hbm_gbs_per_gpu": per_block_bytes * L / (ms * 1e-3) / 1e9,
                "tflops_total": flops / (ms * 1e-3) / 1e12, "oracle_max_abs_err": err,
                "timing": "one CUDA graph per step (GEMMs, SwiGLUs, all-reduces)"}
        if M <= 32:
            line["roofline_per_gpu"] = hbm_roofline(per_block_bytes * L, ms * 1e-3, ctx.pk,
                                                    "decode GEMMs + fused all-reduce")
        else:
            line["roofline_per_gpu"] = tensor_roofline(flops / ctx.world, ms * 1e-3, ctx.pk,
                                                       "prefill GEMMs + NCCL all-reduce", sustained=True)
        lines.append(line)
    close_peer_channels()
    del blocks
    torch.cuda.empty_cache()
    return lines, ok


PREFILL_KERNELS = {1: "prefill::w4a16_tcgen05_kernel (weights as the shared-memory operand)",
                   2: "prefill_ts::w4a16_ts_kernel (weights as the TMEM operand)"}


def measure_prefill(ctx, args):
    """N = 1: the tcgen05 prefill GEMM at M in {512, 2048, 4096, 8192}, K=4096, N=14336,
    L2 flushed before every timed launch; oracle-checked on sampled rows and columns."""
    torch = ctx.torch
    import w4a16
    from w4a16 import _lib
    c = PREFILL
    K, N, G = c["K"], c["N"], c["G"]
    W = make_weight(torch, K, N, c["sigma"], 0.0, 99, ctx.dev)
    qw, s, z = w4a16.quantize_weight(W, G)
    del W
    rng = np.random.default_rng(3)
    cols = torch.from_numpy(np.sort(rng.choice(N, ORACLE_COLS, replace=False))).to(ctx.dev)
    sample = tuple(t[:, cols].contiguous() for t in (qw, s, z))
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=ctx.dev)
    out, ok = [], True
    for M in c["Ms"]:
        gen = torch.Generator(device=ctx.dev).manual_seed(M)
        X = torch.randn(M, K, generator=gen, device=ctx.dev).half()
        y = torch.empty(M, N, device=ctx.dev, dtype=torch.float16)
        w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
        rows = torch.from_numpy(np.sort(rng.choice(M, 16, replace=False))).to(ctx.dev)
        good, err = oracle_check(ctx, f"prefill M={M}", y[rows][:, cols], X[rows], *sample, G)
        ok &= good
        iters = max(5, min(args.steps, 20))
        for _ in range(3):
            w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
        torch.cuda.synchronize(ctx.dev)
        times = []
        for _ in range(iters):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
            b.record()
            torch.cuda.synchronize(ctx.dev)
            times.append(a.elapsed_time(b))
        t = statistics.median(times) / 1e3
        flops = 2.0 * M * N * K
        which = _lib.prefill_choice(M, N, K)
        # the other prefill kernel on the same shape, for the record (forced, same timing)
        other = _lib.PREFILL_SMEM_B if which == _lib.PREFILL_TMEM_A else _lib.PREFILL_TMEM_A
        _lib.set_prefill_kernel(other)
        try:
            w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
            alt = []
            for _ in range(iters):
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record()
                w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
                b.record()
                torch.cuda.synchronize(ctx.dev)
                alt.append(a.elapsed_time(b))
        finally:
            _lib.set_prefill_kernel(_lib.PREFILL_AUTO)
        t_alt = statistics.median(alt) / 1e3
        out.append({"M": M, "K": K, "N": N, "us": t * 1e6, "tflops": flops / t / 1e12, "iters": iters,
                    "kernel": PREFILL_KERNELS[which], "oracle_max_abs_err": err,
                    "other_kernel": {"kernel": PREFILL_KERNELS[other], "us": t_alt * 1e6,
                                     "tflops": flops / t_alt / 1e12},
                    "roofline": tensor_roofline(flops, t, ctx.pk, PREFILL_KERNELS[which])})
        del X, y
    return out, ok


def measure_e2e(ctx, args, X, copies, R, G, n):
    """The headline through the public API with host buffers (see the module docstring):
    (a) pipelined, the K steps replayed from one CUDA graph, x staged in by
    w4a16.stage_copy (a kernel, so the GEMM after it still starts under programmatic
    dependent launch) and y copied out on a second stream; (b) eager from Python with
    Tensor.copy_ in and out; (c) eager from Python through w4a16.w4a16_matmul_host."""
    torch = ctx.torch
    import w4a16
    M, K = X.shape
    dev, stream = ctx.dev, ctx.stream
    Xh = X.cpu().pin_memory()
    Yh = torch.empty(M, n, dtype=torch.float16).pin_memory()
    y_bytes = M * n * 2
    ring = max(2, min(args.steps, (256 << 20) // y_bytes))
    Xd = [torch.empty_like(X) for _ in range(2)]
    Yd = [torch.empty(M, n, device=dev, dtype=torch.float16) for _ in range(ring)]
    s_out = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(3):
            w4a16.stage_copy(Xd[i % 2], Xh, src_ready=True)
            w4a16.w4a16_matmul(Xd[i % 2], *copies[i % R], G, out=Yd[i % ring])
            Yh.copy_(Yd[i % ring], non_blocking=True)
    torch.cuda.synchronize(dev)
    k_done = [torch.cuda.Event() for _ in range(ring)]
    out_done = [torch.cuda.Event() for _ in range(ring)]
    ge = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(ge, stream=stream):
            s_out.wait_stream(stream)
            for i in range(args.steps):
                sl = i % ring
                # x of step i from pinned host memory; Xd[i % 2] was last read by GEMM
                # i-2, which has completed once the copy's wait for GEMM i-1 returns
                w4a16.stage_copy(Xd[i % 2], Xh, src_ready=True)
                if i >= ring:
                    stream.wait_event(out_done[sl])      # y of step i-ring has left Yd[sl]
                w4a16.w4a16_matmul(Xd[i % 2], *copies[i % R], G, out=Yd[sl])
                k_done[sl].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(k_done[sl])
                    Yh.copy_(Yd[sl], non_blocking=True)
                    out_done[sl].record(s_out)
            stream.wait_stream(s_out)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        ge.replay()
    torch.cuda.synchronize(dev)
    ctx.barrier()
    s0e = torch.cuda.Event(enable_timing=True)
    s1e = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s0e.record(stream)
        ge.replay()
        s1e.record(stream)
    torch.cuda.synchronize(dev)
    t_pipe = ctx.max_over_ranks(s0e.elapsed_time(s1e))
    del ge
    # the last step's y, read back through the graph, is the GEMM's result
    y_last = w4a16.w4a16_matmul(X, *copies[(args.steps - 1) % R], G)
    torch.cuda.synchronize(dev)
    assert torch.equal(Yh.to(dev), y_last), "e2e: the y read back differs from the GEMM's result"

    with torch.cuda.stream(stream):
        for i in range(3):
            Xd[0].copy_(Xh, non_blocking=True)
            yy = w4a16.w4a16_matmul(Xd[0], *copies[i % R], G)
            Yh.copy_(yy, non_blocking=True)
        torch.cuda.synchronize(dev)
        ctx.barrier()
        s0e.record(stream)
        h0 = time.perf_counter()
        for i in range(args.steps):
            Xd[0].copy_(Xh, non_blocking=True)
            yy = w4a16.w4a16_matmul(Xd[0], *copies[i % R], G)
            Yh.copy_(yy, non_blocking=True)
        ctx.host_submit_copies_us = (time.perf_counter() - h0) * 1e6 / args.steps
        s1e.record(stream)
    torch.cuda.synchronize(dev)
    t_eager = ctx.max_over_ranks(s0e.elapsed_time(s1e))

    # (c) eager through w4a16.w4a16_matmul_host: one call per step, pinned x in and
    # pinned y out (stage-in, GEMM, stage-out kernels chained on the GEMM stream)
    with torch.cuda.stream(stream):
        for i in range(3):
            w4a16.w4a16_matmul_host(Xh, *copies[i % R], G, out=Yh)
        torch.cuda.synchronize(dev)
        ctx.barrier()
        s0e.record(stream)
        h0 = time.perf_counter()
        for i in range(args.steps):
            w4a16.w4a16_matmul_host(Xh, *copies[i % R], G, out=Yh)
        h1 = time.perf_counter()
        s1e.record(stream)
    torch.cuda.synchronize(dev)
    t_host = ctx.max_over_ranks(s0e.elapsed_time(s1e))
    ctx.host_submit_us = (h1 - h0) * 1e6 / args.steps
    y_last = w4a16.w4a16_matmul(X, *copies[(args.steps - 1) % R], G)
    torch.cuda.synchronize(dev)
    assert torch.equal(Yh.to(dev), y_last), "e2e: w4a16_matmul_host's y differs from the GEMM's result"
    return t_pipe, t_eager, t_host


def run_ours(args):
    import torch
    import torch.distributed as dist

    import w4a16
    from w4a16 import _lib

    ctx = Ctx(torch, dist)
    world, rank, dev = ctx.world, ctx.rank, ctx.dev
    K, N, n, G, sigma, outliers, cfg = workload(world)
    M = 1
    rank_bytes = gemm_bytes(M, K, n, G)
    all_ok = True

    # ---- the headline weights: this rank's shard, R copies so the rotation exceeds L2
    hw = ShardedWeights(ctx, K, N, G, sigma, outliers, 1234 if world == 1 else 4321, 2 * L2_BYTES)
    X = torch.randn(M, K, generator=torch.Generator(device=dev).manual_seed(42), device=dev).half()
    y = torch.empty(M, n, device=dev, dtype=torch.float16)
    w4a16.w4a16_matmul(X, *hw.copies[0], G, out=y)
    good, head_err = oracle_check(ctx, "headline", y[:, hw.cols_own - hw.lo], X, *hw.sample_own, G)
    all_ok &= good
    if not ctx.all_ok(all_ok):
        sys.stderr.write("oracle check failed before timing\n")
        return 3

    def step(i):
        w4a16.w4a16_matmul(X, *hw.copies[i % hw.R], G, out=y)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(ctx.stream):
        with torch.cuda.graph(g, stream=ctx.stream):
            for i in range(args.steps):
                step(i)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.local) as clocks:
        # keep the GPU busy ~1 s so the sampled clocks describe the loaded state
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            with torch.cuda.stream(ctx.stream):
                g.replay()
            torch.cuda.synchronize(dev)
        ctx.barrier()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(ctx.stream):
            e0.record(ctx.stream)
            g.replay()
            e1.record(ctx.stream)
        torch.cuda.synchronize(dev)
        ctx.barrier()
        t_ms = e0.elapsed_time(e1)
        time.sleep(0.25)
    del g
    t_ms = ctx.max_over_ranks(t_ms)
    per_launch_s = t_ms / 1e3 / args.steps
    value = world * rank_bytes * args.steps / (t_ms / 1e3) / 1e9
    assert _lib.check_device_errors(dev) == 0

    # the same GEMM on weights repacked once into the kernel nibble order (w4a16.repack_qweight,
    # W4A16Linear.repack_()): a load-time layout, reported beside the drop-in headline
    kcopies = [(w4a16.repack_qweight(q), s_, z_) for (q, s_, z_) in hw.copies]
    yk = torch.empty_like(y)
    w4a16.w4a16_matmul(X, *kcopies[0], G, out=yk, kernel_order=True)
    good, _ = oracle_check(ctx, "headline (kernel nibble order)", yk[:, hw.cols_own - hw.lo], X, *hw.sample_own, G)
    all_ok &= good

    def kstep(i):
        w4a16.w4a16_matmul(X, *kcopies[i % hw.R], G, out=yk, kernel_order=True)
    tk = ctx.time_graph(kstep, args.steps) / 1e3 / args.steps
    kernel_order_line = {"us_per_call": tk * 1e6, "value": world * rank_bytes / tk / 1e9, "unit": "GB/s",
                         "roofline": hbm_roofline(rank_bytes, tk, ctx.pk, "decode_gemv_tma_kernel<1, false, true>"),
                         "what": "the headline GEMM with qweight repacked once into the kernel nibble order"}
    del kcopies, yk

    t_pipe, t_eager, t_host = measure_e2e(ctx, args, X, hw.copies, hw.R, G, n)
    e2e_value = world * rank_bytes * args.steps / (t_pipe / 1e3) / 1e9
    e2e_eager = world * rank_bytes * args.steps / (t_eager / 1e3) / 1e9
    e2e_host = world * rank_bytes * args.steps / (t_host / 1e3) / 1e9
    del hw, y
    torch.cuda.empty_cache()

    # ---- the sweep configuration (column-sharded at N > 1), gather, MLP stack, prefill
    extra = {}
    if not args.no_sweep:
        c = SWEEP
        sw = ShardedWeights(ctx, c["K"], c["N"], c["G"], c["sigma"], c["outliers"], 4321, 2 * L2_BYTES)
        gx = torch.Generator(device=dev).manual_seed(43)
        X_by_M = {m: torch.randn(m, c["K"], generator=gx, device=dev).half() for m in c["Ms"]}
        ys = {m: torch.empty(m, sw.n, device=dev, dtype=torch.float16) for m in c["Ms"]}
        extra["sweep"], good = measure_sweep(ctx, args, sw, X_by_M, ys)
        all_ok &= good
        if world > 1:
            extra["gather"], good = measure_gather(ctx, args, sw, X_by_M)
            all_ok &= good
        else:
            # past the decode route: 48 and 96 tokens on the same weights (prefill kernels;
            # not a BASELINE configuration, reported for the 33-128-token range)
            from w4a16 import _lib
            X_mid = {m: torch.randn(m, c["K"], generator=gx, device=dev).half() for m in (48, 96)}
            y_mid = {m: torch.empty(m, sw.n, device=dev, dtype=torch.float16) for m in X_mid}
            extra["mid_m"], good = measure_sweep(ctx, args, sw, X_mid, y_mid)
            for e in extra["mid_m"]:
                which = _lib.prefill_choice(e["M"], sw.n, c["K"])
                e["roofline_per_gpu"]["kernel"] = PREFILL_KERNELS.get(which, "prefill")
            all_ok &= good
            del X_mid, y_mid
        del sw, X_by_M, ys
        torch.cuda.empty_cache()
    if not args.no_mlp:
        extra["mlp_stack"], good = measure_mlp(ctx, args)
        all_ok &= good
    if world == 1 and not args.no_prefill:
        extra["prefill"], good = measure_prefill(ctx, args)
        all_ok &= good
        p4096 = [p for p in extra["prefill"] if p["M"] == 4096]
        if p4096:
            p = p4096[0]
            extra["secondary"] = {
                "metric": "W4A16 GEMM TFLOP/s at M=4096, K=4096, N=14336, G=128 (tcgen05 prefill kernel)",
                "value": p["tflops"], "unit": "TFLOP/s", "ms": p["us"] / 1e3, "iters": p["iters"],
                "kernel": p["kernel"],
                "l2": "L2 flushed (252 MiB write) before every timed launch", "roofline": p["roofline"]}
    assert _lib.check_device_errors(dev) == 0
    if not ctx.all_ok(all_ok):
        sys.stderr.write("oracle check failed\n")
        return 3

    kernel = "decode_gemv_tma_kernel<1, false>"
    traffic, tsrc = None, None
    if world == 1:
        traffic = profile_traffic("decode_gemv_m1_k4096_n11008.txt")
        tsrc = "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/decode_gemv_m1_k4096_n11008.txt"
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
        "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": value / world / PUBLISHED_T4_GBS if world == 1 else None,
        "vs_baseline_ref": "per-GPU value / 31 GB/s: the reference's Triton kernel on a T4, same metric "
                           "and shape (README.md:186); null at N > 1 (no published sharded number)",
        "dtype": "f16", "data": "synthetic",
        "config": cfg,
        "oracle_check": {"passed": True, "headline_max_abs_err": head_err,
                         "what": f"every rank, every configuration: {ORACLE_COLS} sampled output columns "
                                 "against the numpy oracle (|d| <= 1e-2 + 1e-3 |ref|) before timing"},
        "roofline": hbm_roofline(rank_bytes, per_launch_s, ctx.pk, kernel, traffic, tsrc),
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": world * M * K * 2,
                "d2h_bytes_per_step": world * M * n * 2,
                "path": "pinned host X -> w4a16.stage_copy -> w4a16.w4a16_matmul -> pinned host Y "
                        "(this rank's columns) every step: x staged in by a kernel on the GEMM stream "
                        "(chains under programmatic dependent launch), y copied out on a second stream "
                        "while the next steps compute; the K steps replayed from one CUDA graph",
                "eager": {"value": e2e_host, "unit": "GB/s", "us_per_step": t_host * 1e3 / args.steps,
                          "host_submit_us_per_step": ctx.host_submit_us,
                          "path": "eager from Python, one w4a16.w4a16_matmul_host call per step (pinned X "
                                  "in, pinned Y out: stage-in, GEMM and stage-out kernels chained under "
                                  "programmatic dependent launch on one stream)"},
                "eager_torch_copies": {"value": e2e_eager, "unit": "GB/s",
                                       "us_per_step": t_eager * 1e3 / args.steps,
                                       "host_submit_us_per_step": ctx.host_submit_copies_us,
                                       "path": "eager from Python on one stream: Tensor.copy_ of X in, "
                                               "w4a16.w4a16_matmul, Tensor.copy_ of Y out (copy-engine "
                                               "transfers between the kernels)"}},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "kernel_order": kernel_order_line,
    }
    line.update(extra)
    if rank == 0 and world == 1 and not args.no_cpu:
        c = DECODE
        t_cpu, n_cpu, threads = time_cpu(M, K, N, G, sigma, outliers, min_seconds=args.cpu_seconds)
        t_one, n_one, _ = time_cpu(M, K, N, G, sigma, outliers, steps=3, threads=1)
        line["cpu_baseline"] = {"value": rank_bytes / t_cpu / 1e9, "unit": "GB/s", "cores": threads,
                                "kind": "port", "what": CPU_KIND_NOTE,
                                "sample": f"{n_cpu} full decode GEMMs, numpy over {threads} column blocks, "
                                          f"median {t_cpu * 1e3:.1f} ms",
                                "cpu_model": cpu_model(),
                                "one_core": {"value": rank_bytes / t_one / 1e9, "unit": "GB/s",
                                             "sample": f"{n_one} full decode GEMMs on 1 thread, median "
                                                       f"{t_one * 1e3:.1f} ms"}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        from w4a16.parallel import close_peer_channels
        close_peer_channels()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill sweep")
    ap.add_argument("--no-sweep", action="store_true", help="skip the batched-decode sweep (and gather)")
    ap.add_argument("--no-mlp", action="store_true", help="skip the MLP-stack configuration")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
