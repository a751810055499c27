"""Benchmark: W4A16 GEMM HBM GB/s at M=1 (and TFLOP/s at M=4096) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Headline workload (the decode configuration): M=1, K=4096, N=11008, G=128,
X ~ N(0,1) fp16, W ~ N(0, 0.02) fp16 quantised to uint4 on the GPU. One step =
one fused GEMM over one batch. Weak scaling: with N GPUs every rank owns an
11008-column shard of an (11008*N)-column weight and computes its slice of Y;
there is no collective on the data path (an all-gather of Y is only needed
when a caller wants the full output, and is not part of this metric).

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and a
device synchronise, timed with CUDA events on the launching stream, max over
ranks. Inputs are larger than L2: each step uses the next of R distinct
weight copies totalling > 126 MB. The K steps are replayed from a CUDA graph
captured beforehand so the host's launch rate does not cap a ~4 us kernel.

``e2e`` is the same metric through the public Python API with host buffers:
each step copies X from pinned host memory, calls ``w4a16_matmul`` eagerly and
copies Y back, all inside the timed region.

``--impl reference`` times the reference's CPU path (dequantise, then matmul)
restated in numpy (oracle/), on all host cores, on the same configuration.
"""
from __future__ import annotations

import argparse
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
DECODE = dict(M=1, K=4096, N=11008, G=128, sigma=0.02)
PREFILL = dict(M=4096, K=4096, N=14336, G=128, sigma=0.02)
L2_BYTES = 126 * 1024 * 1024
PUBLISHED_T4_GBS = 31.0  # README.md:186, the reference's Triton kernel, same metric and shape, on a T4


def gemm_bytes(M, K, N, G):
    """Algorithmic bytes per GEMM (the reference's byte model, bench_gemm.py:61-67):
    X + packed weights + scales + zeros + Y."""
    return M * K * 2 + (K // 8) * N * 4 + 2 * (K // G) * N * 2 + M * N * 2


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
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
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


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


def cpu_inputs(cfg, seed=0):
    import oracle
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((cfg["M"], cfg["K"]), dtype=np.float32).astype(np.float16)
    W = (rng.standard_normal((cfg["K"], cfg["N"]), dtype=np.float32) * np.float32(cfg["sigma"])).astype(np.float16)
    qw, s, z = oracle.quantize_weight(W, cfg["G"])
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


def time_cpu(cfg, min_seconds=10.0, max_iters=50, steps=None, threads=None):
    """Time the CPU path; returns (median seconds per GEMM, iterations, threads).

    Runs for at least ``min_seconds`` (bounded by ``max_iters``) or exactly
    ``steps`` iterations. BLAS is pinned to one thread per worker; the column
    blocks give the parallelism (all host cores unless ``threads`` is given)."""
    from threadpoolctl import threadpool_limits
    threads = threads or os.cpu_count() or 1
    X, qw, s, z = cpu_inputs(cfg)
    times = []
    with threadpool_limits(limits=1):
        cpu_dequant_then_matmul(X, qw, s, z, cfg["G"], threads)   # warm-up
        t_end = time.perf_counter() + min_seconds
        while (len(times) < steps) if steps is not None else \
                (time.perf_counter() < t_end and len(times) < max_iters):
            t0 = time.perf_counter()
            cpu_dequant_then_matmul(X, qw, s, z, cfg["G"], threads)
            times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), threads


# --------------------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = DECODE
    # each step is one full decode GEMM on the CPU (~0.1-1 s); cap the count so
    # the whole run stays within a few minutes
    t, n, threads = time_cpu(cfg, steps=max(1, min(args.steps, 60)))
    gbs = gemm_bytes(cfg["M"], cfg["K"], cfg["N"], cfg["G"]) / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": {"workload": "decode GEMM M=1 K=4096 N=11008 G=128 (CPU)",
                                        "M": 1, "K": 4096, "N": 11008, "group_size": 128},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n} full decode GEMMs (dequantise-then-matmul), "
                                   f"numpy oracle over {threads} column blocks",
                         "cpu_model": cpu_model()},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import w4a16
    from w4a16 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    cfg = DECODE
    M, K, N, G = cfg["M"], cfg["K"], cfg["N"], cfg["G"]
    step_bytes = gemm_bytes(M, K, N, G)

    # ---- inputs: this rank's column shard, R copies so the rotation exceeds L2
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    shard_w_bytes = (K // 8) * N * 4 + 2 * (K // G) * N * 2
    R = max(2, -(-2 * L2_BYTES // shard_w_bytes))
    X = torch.randn(M, K, generator=gen, device=dev).half()
    W = (torch.randn(K, N, generator=gen, device=dev) * cfg["sigma"]).half()
    qw0, s0, z0 = w4a16.quantize_weight(W, G)
    copies = [(qw0, s0, z0)] + [(qw0.clone(), s0.clone(), z0.clone()) for _ in range(R - 1)]
    del W
    y = torch.empty(M, N, device=dev, dtype=torch.float16)

    def step(i):
        qw, s, z = copies[i % R]
        w4a16.w4a16_matmul(X, qw, s, z, G, out=y)

    stream = torch.cuda.Stream(device=dev)
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize(dev)
    # capture the K timed steps (and a warm-up replay of the same graph)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for i in range(args.steps):
                step(i)
    torch.cuda.synchronize(dev)

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # keep the GPU busy ~1 s so the sampled clocks describe the loaded state
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            g.replay()
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            e0.record(stream)
            g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t_ms = e0.elapsed_time(e1)
        time.sleep(0.25)
    t_max = torch.tensor([t_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    t_ms = float(t_max.item())
    per_launch_s = t_ms / 1e3 / args.steps
    value = world * step_bytes * args.steps / (t_ms / 1e3) / 1e9
    assert _lib.check_device_errors(dev) == 0

    # ---- e2e through the public API with host buffers. Every step copies its x from
    # pinned host memory to the device and reads its y back to pinned host memory.
    # (a) pipelined, as a serving loop runs its decode steps, the K steps captured
    #     in one CUDA graph (no Python on the timed path): each step's x is staged in
    #     by w4a16.stage_copy -- a kernel, so the GEMM after it still starts under
    #     programmatic dependent launch (a memory-copy node there would make every
    #     GEMM wait for the previous one to finish) -- and its y is copied out by a
    #     memcpy on a second stream while the next steps compute (one device y per
    #     step, up to a 256 MiB ring, so no GEMM waits on a copy-out);
    # (b) eager: copy in, GEMM, copy out from Python on one stream.
    Xh = X.cpu().pin_memory()
    Yh = torch.empty(M, N, dtype=torch.float16).pin_memory()
    y_bytes = M * N * 2
    ring = max(2, min(args.steps, (256 << 20) // y_bytes))
    Xd = [torch.empty_like(X) for _ in range(2)]
    Yd = [torch.empty(M, N, device=dev, dtype=torch.float16) for _ in range(ring)]
    s_out = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(3):   # warm-up on the GEMM stream (creates its workspace)
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
    if world > 1:
        dist.barrier()
    s0e = torch.cuda.Event(enable_timing=True)
    s1e = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s0e.record(stream)
        ge.replay()
        s1e.record(stream)
    torch.cuda.synchronize(dev)
    e2e_t = torch.tensor([s0e.elapsed_time(s1e)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = world * step_bytes * args.steps / (float(e2e_t.item()) / 1e3) / 1e9
    del ge
    # the last step's y, read back through the graph, is the GEMM's result
    y_last = w4a16.w4a16_matmul(X, *copies[(args.steps - 1) % R], G)
    torch.cuda.synchronize(dev)
    assert torch.equal(Yh.to(dev), y_last), "e2e: the y read back differs from the GEMM's result"

    for i in range(3):
        Xd[0].copy_(Xh, non_blocking=True)
        yy = w4a16.w4a16_matmul(Xd[0], *copies[i % R], G)
        Yh.copy_(yy, non_blocking=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    s0e.record()
    for i in range(args.steps):
        Xd[0].copy_(Xh, non_blocking=True)
        yy = w4a16.w4a16_matmul(Xd[0], *copies[i % R], G)
        Yh.copy_(yy, non_blocking=True)
    s1e.record()
    torch.cuda.synchronize(dev)
    eager_t = torch.tensor([s0e.elapsed_time(s1e)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(eager_t, op=dist.ReduceOp.MAX)
    e2e_eager = world * step_bytes * args.steps / (float(eager_t.item()) / 1e3) / 1e9

    # ---- secondary: prefill TFLOP/s at M=4096 (rank 0, N=1 only; not part of `value`)
    secondary = None
    if world == 1 and not args.no_prefill:
        secondary = prefill_secondary(torch, w4a16, dev, args)

    pk = peaks()
    achieved = step_bytes / per_launch_s / 1e9
    traffic = profile_traffic("decode_gemv_m1_k4096_n11008.txt")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": value / world / PUBLISHED_T4_GBS,
        "vs_baseline_ref": "per-GPU value / 31 GB/s: the reference's Triton kernel on a T4, "
                           "same metric and shape (README.md:186)",
        "dtype": "f16", "data": "synthetic",
        "config": {"workload": "decode GEMM M=1 K=4096 N=11008 G=128 per GPU (column shard of an "
                               f"{N * world}-column weight)", "M": M, "K": K, "N_per_gpu": N,
                   "group_size": G, "parallelism": f"column-parallel x{world}, no collective",
                   "l2": f"{R} rotating weight copies, {R * shard_w_bytes / 2**20:.0f} MiB > 126 MiB L2",
                   "timing": "CUDA graph of the K steps, CUDA events on the launching stream"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"],
                     "peak_source": f"{pk['source']} hbm_gbs (MEASURED_PEAKS.json)" if pk["source"] == "measured"
                     else "fallback 6650 GB/s",
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": step_bytes,
                     "kernel": "decode_gemv_tma_kernel<1, false>"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": M * K * 2,
                "d2h_bytes_per_step": M * N * 2,
                "path": "pinned host X -> w4a16.stage_copy -> w4a16.w4a16_matmul -> pinned host Y "
                        "every step: x staged in by a kernel on the GEMM stream (chains under "
                        "programmatic dependent launch), y copied out on a second stream while "
                        "the next steps compute; the K steps replayed from one CUDA graph",
                "eager": {"value": e2e_eager, "unit": "GB/s",
                          "path": "the same three calls per step from Python on one stream"}},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if secondary is not None:
        line["secondary"] = secondary
    if rank == 0 and world == 1 and not args.no_cpu:
        t_cpu, n_cpu, threads = time_cpu(DECODE, min_seconds=args.cpu_seconds)
        cpu_gbs = step_bytes / t_cpu / 1e9
        t_one, n_one, _ = time_cpu(DECODE, steps=3, threads=1)
        line["cpu_baseline"] = {"value": cpu_gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": f"{n_cpu} full decode GEMMs (dequantise-then-matmul, numpy oracle "
                                          f"over {threads} column blocks), median {t_cpu * 1e3:.1f} ms",
                                "cpu_model": cpu_model(),
                                "one_core": {"value": step_bytes / t_one / 1e9, "unit": "GB/s",
                                             "sample": f"{n_one} full decode GEMMs on 1 thread, median "
                                                       f"{t_one * 1e3:.1f} ms"}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def prefill_secondary(torch, w4a16, dev, args):
    cfg = PREFILL
    M, K, N, G = cfg["M"], cfg["K"], cfg["N"], cfg["G"]
    gen = torch.Generator(device=dev).manual_seed(99)
    X = torch.randn(M, K, generator=gen, device=dev).half()
    W = (torch.randn(K, N, generator=gen, device=dev) * cfg["sigma"]).half()
    qw, s, z = w4a16.quantize_weight(W, G)
    del W
    y = torch.empty(M, N, device=dev, dtype=torch.float16)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    iters = max(5, min(args.steps, 20))
    for _ in range(3):
        w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(iters):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        w4a16.w4a16_matmul(X, qw, s, z, G, out=y)
        b.record()
        torch.cuda.synchronize(dev)
        times.append(a.elapsed_time(b))
    t = statistics.median(times) / 1e3
    flops = 2.0 * M * N * K
    tf = flops / t / 1e12
    pk = peaks()
    peak = pk.get("bf16_tflops", 1590.0)
    return {"metric": "W4A16 GEMM TFLOP/s at M=4096, K=4096, N=14336, G=128 (tcgen05 prefill kernel)",
            "value": tf, "unit": "TFLOP/s", "ms": t * 1e3, "iters": iters,
            "l2": "L2 flushed (252 MiB write) before every timed launch",
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak, "peak_source": "measured bf16_tflops (burst), fp16 proxy"
                         if pk["source"] == "measured" else "fallback 1590",
                         "frac_of_2250_nominal": tf / 2250.0,
                         "kernel": "prefill::w4a16_tcgen05_kernel"}}


def run_mlp(args):
    """The decoder MLP-stack configuration: 80 blocks of gate/up [8192->28672]
    (column-parallel, fused into one GEMM), SwiGLU and down [28672->8192]
    (row-parallel, fp32 all-reduce over NCCL), at M=1 and M=2048 tokens.

    Every block reads its own weights from HBM: 4 distinct weight sets are
    cycled over the 80 blocks (>= 1.4 GB per GPU, far above L2). Each block
    gets the same input, so the timed work is exactly the 80 blocks' GEMMs,
    SwiGLUs and all-reduces without an activation-normalisation kernel."""
    import datetime

    import torch
    import torch.distributed as dist

    from w4a16.parallel import W4A16MLP

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    D, H, G, L, NSETS = 8192, 28672, 128, 80, 4
    blocks = []
    for i in range(NSETS):
        gen = torch.Generator(device=dev).manual_seed(1000 + i)
        wg = (torch.randn(D, H, generator=gen, device=dev) * 0.02).half()
        wu = (torch.randn(D, H, generator=gen, device=dev) * 0.02).half()
        wd = (torch.randn(H, D, generator=gen, device=dev) * 0.02).half()
        blocks.append(W4A16MLP.from_dense(wg, wu, wd, G))
        del wg, wu, wd
        torch.cuda.empty_cache()
    per_block_bytes = sum(b.numel() * b.element_size() for b in blocks[0].buffers())
    lines = []
    for M in (1, 2048):
        gen = torch.Generator(device=dev).manual_seed(7)
        x = torch.randn(M, D, generator=gen, device=dev).half()

        def step():
            for l in range(L):
                y = blocks[l % NSETS](x)
            return y

        for _ in range(max(1, args.warmup)):
            step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(1, min(args.steps, 5))
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

        # the same step captured in one CUDA graph (GEMMs, SwiGLUs and, with tp > 1,
        # the NCCL all-reduces): no Python or launch overhead between the 80 blocks
        gst = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(gst):
            for _ in range(2):
                step()   # warm-up on the capture stream (its GEMM workspace)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(gst):
            with torch.cuda.graph(graph, stream=gst):
                step()
            graph.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        with torch.cuda.stream(gst):
            e0.record(gst)
            for _ in range(steps):
                graph.replay()
            e1.record(gst)
        torch.cuda.synchronize(dev)
        tg = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        gms = float(tg.item())
        del graph   # before the process group goes away (it holds NCCL work)

        flops = 2.0 * M * (2 * D * H + H * D) * L
        lines.append({"config": {"workload": f"MLP stack 80 x (gate/up {D}->{H}, down {H}->{D}) G=128",
                                 "M": M, "parallelism": f"tp{world}", "weights_per_gpu_per_block_bytes": per_block_bytes},
                      "ms_per_step": gms, "hbm_gbs_per_gpu": per_block_bytes * L / (gms * 1e-3) / 1e9,
                      "tflops_total": flops / (gms * 1e-3) / 1e12, "timing": "one CUDA graph per step",
                      "eager": {"ms_per_step": ms, "hbm_gbs_per_gpu": per_block_bytes * L / (ms * 1e-3) / 1e9,
                                "tflops_total": flops / (ms * 1e-3) / 1e12},
                      "n_gpus": world, "steps": steps})
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)
    if world > 1:
        from w4a16.parallel import close_peer_channels
        close_peer_channels()   # collective; before the process group goes away
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
    ap.add_argument("--no-prefill", action="store_true", help="skip the M=4096 secondary line")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--config", choices=["decode", "mlp"], default="decode",
                    help="decode: the headline line; mlp: the 80-block MLP-stack configuration")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    if args.config == "mlp":
        return run_mlp(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
