"""Tensor-parallel layers on the GPU: fp32-output GEMM, SwiGLU, the column /
row-parallel layers and the MLP block against the numpy oracle; with two or
more GPUs visible, also as NCCL ranks against the unsharded result."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from helpers import gpu_case, np_
from tolerance import assert_gemm_close
from w4a16 import (interleave_gate_up, quantize_weight, swiglu, w4a16_matmul, w4a16_matmul_f32,
                   w4a16_matmul_swiglu)
from w4a16.parallel import ColumnParallelW4A16Linear, RowParallelW4A16Linear, W4A16MLP

pytestmark = pytest.mark.gpu
ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _oracle_f32(X, qw, s, z, G):
    W = oracle.dequantize_weight(np_(qw), np_(s), np_(z), G).astype(np.float32)
    return np_(X).astype(np.float32) @ W


def _silu_mul(g, u):
    g = g.astype(np.float32)
    return (g / (1.0 + np.exp(-g)) * u.astype(np.float32)).astype(np.float16)


def _mlp_oracle(X, gate, up, down, G):
    g = oracle.reference_w4a16(np_(X), *(np_(t) for t in gate), G)
    u = oracle.reference_w4a16(np_(X), *(np_(t) for t in up), G)
    h = _silu_mul(g, u)
    return oracle.reference_w4a16(h, *(np_(t) for t in down), G)


@pytest.mark.parametrize("M", [1, 5, 40, 300])
def test_fp32_output_gemm(M):
    X, W = gpu_case(M, 1024, 264, 128, sigma=0.05, seed=M)
    qw, s, z = quantize_weight(W, 128)
    y = w4a16_matmul_f32(X, qw, s, z, 128)
    assert y.dtype == torch.float32 and y.shape == (M, 264)
    ref = _oracle_f32(X, qw, s, z, 128)
    err = np.abs(np_(y) - ref)
    assert np.all(err <= 1e-4 + 1e-5 * np.abs(ref)), err.max()


def test_swiglu_matches_fp32_reference():
    gu = torch.randn(7, 2 * 136, device="cuda").half() * 3
    h = swiglu(gu)
    ref = _silu_mul(np_(gu[:, :136]), np_(gu[:, 136:]))
    assert np.max(np.abs(np_(h).astype(np.float32) - ref.astype(np.float32))) <= 2e-3 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("M,K,H", [(1, 1024, 208), (5, 512, 64), (9, 1024, 336), (32, 2048, 512),
                                   (33, 512, 208), (300, 1024, 336)])
def test_fused_swiglu_gemm_matches_gemm_then_swiglu(M, K, H):
    """The SwiGLU epilogue (decode route up to 32 tokens, tcgen05 route beyond) gives
    the bits of the plain GEMM on the same interleaved weights followed by the SwiGLU
    kernel, and agrees with the oracle."""
    G = 128 if K % 128 == 0 else 64
    X, Wg = gpu_case(M, K, H, G, sigma=0.05, seed=M + H)
    _, Wu = gpu_case(1, K, H, G, sigma=0.05, seed=M + H + 1)
    qg, qu = quantize_weight(Wg, G), quantize_weight(Wu, G)
    fused = [interleave_gate_up(a, b) for a, b in zip(qg, qu)]
    h = w4a16_matmul_swiglu(X, *fused, G)
    assert h.shape == (M, H) and h.dtype == torch.float16
    gu = w4a16_matmul(X, *fused, G).view(M, H // 16, 2, 16)
    ref = swiglu(torch.cat([gu[:, :, 0].reshape(M, H), gu[:, :, 1].reshape(M, H)], dim=1))
    assert torch.equal(h, ref), f"max |d| {float((h.float() - ref.float()).abs().max())}"
    g = oracle.reference_w4a16(np_(X), *(np_(t) for t in qg), G)
    u = oracle.reference_w4a16(np_(X), *(np_(t) for t in qu), G)
    want = _silu_mul(g, u).astype(np.float32)
    err = np.abs(np_(h).astype(np.float32) - want)
    assert np.all(err <= 2e-2 + 4e-3 * np.abs(want)), float(err.max())


@pytest.mark.parametrize("M", [1, 64])
def test_single_rank_layers_and_mlp(M):
    D, H, G = 512, 1024, 128
    X, Wg = gpu_case(M, D, H, G, sigma=0.05, seed=1)
    _, Wu = gpu_case(1, D, H, G, sigma=0.05, seed=2)
    _, Wd = gpu_case(1, H, D, G, sigma=0.05, seed=3)
    col = ColumnParallelW4A16Linear.from_quantized(*quantize_weight(Wg, G), G)
    qg = quantize_weight(Wg, G)
    assert_gemm_close(np_(col(X, gather=True)), oracle.reference_w4a16(np_(X), *(np_(t) for t in qg), G), "col")
    qd = quantize_weight(Wd, G)
    row = RowParallelW4A16Linear.from_quantized(*qd, G)
    Xh = torch.randn(M, H, device="cuda").half()
    assert_gemm_close(np_(row(Xh)), oracle.reference_w4a16(np_(Xh), *(np_(t) for t in qd), G), "row")
    mlp = W4A16MLP.from_dense(Wg, Wu, Wd, G)
    y = mlp(X)
    ref = _mlp_oracle(X, qg, quantize_weight(Wu, G), qd, G)
    assert_gemm_close(np_(y), ref, "mlp")


# ----------------------------------------------------------------------------- NCCL ranks
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank: int, world: int, port: int, q) -> None:
    try:
        for p in (os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200"), ROOT,
                  os.path.join(ROOT, "tests")):
            sys.path.insert(0, p)
        import datetime
        import torch.distributed as dist
        from helpers import gpu_case as case
        from w4a16 import quantize_weight as quant, w4a16_matmul
        from w4a16.parallel import ColumnParallelW4A16Linear as Col, W4A16MLP as MLP

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        D, H, G, M = 1024, 2048, 128, 4
        X, Wg = case(M, D, H, G, sigma=0.05, seed=1, device=dev)
        _, Wu = case(1, D, H, G, sigma=0.05, seed=2, device=dev)
        _, Wd = case(1, H, D, G, sigma=0.05, seed=3, device=dev)
        qg = quant(Wg, G)
        full = w4a16_matmul(X, *qg, G)
        y = Col.from_quantized(*qg, G)(X, gather=True)
        col_err = float((y.float() - full.float()).abs().max())
        mlp = MLP.from_dense(Wg, Wu, Wd, G)(X)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, (col_err, y.cpu().numpy()), mlp.cpu().numpy(), None))
    except Exception as e:
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_column_gather_and_mlp():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, col, _, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert col[0] <= 1e-2, f"rank {rank}: gathered shards differ by {col[0]}"
    # the same block unsharded on one GPU
    D, H, G, M = 1024, 2048, 128, 4
    X, Wg = gpu_case(M, D, H, G, sigma=0.05, seed=1)
    _, Wu = gpu_case(1, D, H, G, sigma=0.05, seed=2)
    _, Wd = gpu_case(1, H, D, G, sigma=0.05, seed=3)
    qg = quantize_weight(Wg, G)
    col_ref = oracle.reference_w4a16(np_(X), *(np_(t) for t in qg), G)
    for rank, col, _, _ in res:
        assert_gemm_close(col[1], col_ref, f"NCCL column gather vs oracle, rank {rank}")
    ref = _mlp_oracle(X, qg, quantize_weight(Wu, G), quantize_weight(Wd, G), G)
    for rank, _, y, _ in res:
        assert_gemm_close(y, ref, f"tp mlp rank {rank}")


def _fused_row_rank(rank: int, world: int, port: int, q) -> None:
    try:
        for p in (os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200"), ROOT,
                  os.path.join(ROOT, "tests")):
            sys.path.insert(0, p)
        import datetime
        import torch.distributed as dist
        from helpers import gpu_case as case
        from w4a16 import _lib, quantize_weight as quant
        from w4a16.parallel import RowParallelW4A16Linear as Row, close_peer_channels

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        K, N, G = 2048, 1024, 128
        results = {}
        for M in (1, 5, 32):
            X, Wd = case(M, K, N, G, sigma=0.05, seed=11 + M, device=dev)
            qd = quant(Wd, G)
            bias = (torch.randn(N, generator=torch.Generator(device=dev).manual_seed(3), device=dev)
                    * 0.1).half()
            for use_bias in (False, True):
                fused = Row.from_quantized(*qd, G, bias=bias if use_bias else None)
                nccl = Row.from_quantized(*qd, G, bias=bias if use_bias else None)
                nccl.fused_allreduce = False
                k = K // world
                xl = X[:, rank * k:(rank + 1) * k].contiguous()
                outs = [fused(xl) for _ in range(3)]           # several epochs: both halves
                ref = nccl(xl)
                results[(M, use_bias)] = (np_(torch.stack(outs)), np_(ref))
        # the fused call inside a CUDA graph, replayed (the epoch lives on the device)
        M = 1
        X, Wd = case(M, K, N, G, sigma=0.05, seed=99, device=dev)
        qd = quant(Wd, G)
        row = Row.from_quantized(*qd, G)
        k = K // world
        xl = X[:, rank * k:(rank + 1) * k].contiguous()
        eager = row(xl)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            row(xl)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                yg = row(xl)
            for _ in range(4):
                g.replay()
        torch.cuda.synchronize(dev)
        graph_ok = bool(torch.equal(yg, eager))
        flags = _lib.check_device_errors(dev)
        del g
        close_peer_channels()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, graph_ok, flags, None))
    except Exception as e:
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_fused_row_parallel_gemm_allreduce(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_row_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, results, graph_ok, flags, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert flags == 0, f"rank {rank}: device error flags {flags}"
        assert graph_ok, f"rank {rank}: graph replays differ from the eager fused call"
        for (M, use_bias), (outs, ref) in results.items():
            for i in range(outs.shape[0]):
                if world == 2:
                    # same partials, same fp32 sum (two terms commute), one fp16 rounding
                    assert np.array_equal(outs[i], ref), f"rank {rank} M={M} bias={use_bias} call {i}"
                else:
                    # rank-order sum vs NCCL's reduction order: equal up to fp32 reassociation
                    assert_gemm_close(outs[i], ref, f"rank {rank} M={M} bias={use_bias} call {i}")
    # the ranks agree with each other (every rank sums the same words in rank order)
    for key in res[0][1]:
        for r in range(1, world):
            assert np.array_equal(res[0][1][key][0], res[r][1][key][0])
    # and with the oracle of the unsharded layer (rebuilt here from the same seeds)
    K, N, G = 2048, 1024, 128
    for (M, use_bias), (outs, _) in res[0][1].items():
        X, Wd = gpu_case(M, K, N, G, sigma=0.05, seed=11 + M)
        qd = quantize_weight(Wd, G)
        ref = oracle.reference_w4a16(np_(X), *(np_(t) for t in qd), G)
        if use_bias:
            bias = (torch.randn(N, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
                    * 0.1).half()
            ref = (ref + np_(bias)).astype(np.float16)
        for i in range(outs.shape[0]):
            assert_gemm_close(outs[i], ref, f"fused all-reduce vs oracle M={M} bias={use_bias} call {i}")


def _fused_col_rank(rank: int, world: int, port: int, q) -> None:
    try:
        for p in (os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200"), ROOT,
                  os.path.join(ROOT, "tests")):
            sys.path.insert(0, p)
        import datetime
        import torch.distributed as dist
        from helpers import gpu_case as case
        from w4a16 import _lib, quantize_weight as quant
        from w4a16.parallel import ColumnParallelW4A16Linear as Col, RowParallelW4A16Linear as Row
        from w4a16.parallel import close_peer_channels

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        K, N, G = 2048, 1024, 128        # N columns in all, N / world per rank
        results = {}
        for M in (1, 5, 32):
            X, Wd = case(M, K, N, G, sigma=0.05, seed=21 + M, device=dev)
            qd = quant(Wd, G)
            bias = (torch.randn(N, generator=torch.Generator(device=dev).manual_seed(4), device=dev)
                    * 0.1).half()
            for use_bias in (False, True):
                fused = Col.from_quantized(*qd, G, bias=bias if use_bias else None)
                nccl = Col.from_quantized(*qd, G, bias=bias if use_bias else None)
                nccl.fused_gather = False
                outs = [fused(X, gather=True) for _ in range(3)]   # several epochs: both halves
                ref = nccl(X, gather=True)
                results[(M, use_bias)] = (np_(torch.stack(outs)), np_(ref))
        # gathers and all-reduces interleaved on one channel (row output = N / world columns)
        M = 3
        X, Wd = case(M, K, N, G, sigma=0.05, seed=7, device=dev)
        col = Col.from_quantized(*quant(Wd, G), G)
        Xr, Wr = case(M, K, N // world, G, sigma=0.05, seed=8, device=dev)
        row = Row.from_quantized(*quant(Wr, G), G)
        row_ref = Row.from_quantized(*quant(Wr, G), G)
        row_ref.fused_allreduce = False
        k = K // world
        xl = Xr[:, rank * k:(rank + 1) * k].contiguous()
        mixed_ok = True
        for _ in range(3):
            yg = col(X, gather=True)
            yr = row(xl)
            yr_ref = row_ref(xl)
            mixed_ok &= bool(torch.equal(yr, yr_ref)) if world == 2 else \
                bool(((yr.float() - yr_ref.float()).abs() <= 1e-2 + 1e-3 * yr_ref.float().abs()).all())
            mixed_ok &= bool(torch.equal(yg[:, rank * (N // world):(rank + 1) * (N // world)], col(X)))
        # the fused gather inside a CUDA graph, replayed
        eager = col(X, gather=True)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            col(X, gather=True)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                yg = col(X, gather=True)
            for _ in range(4):
                g.replay()
        torch.cuda.synchronize(dev)
        graph_ok = bool(torch.equal(yg, eager))
        flags = _lib.check_device_errors(dev)
        del g
        close_peer_channels()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, mixed_ok and graph_ok, flags, None))
    except Exception as e:
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_fused_column_parallel_gemm_allgather(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_col_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, results, ok, flags, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert flags == 0, f"rank {rank}: device error flags {flags}"
        assert ok, f"rank {rank}: interleaved or graph-replayed calls differ"
        for (M, use_bias), (outs, ref) in results.items():
            for i in range(outs.shape[0]):
                # every column is one rank's fp16 GEMM result: the same bits as NCCL's gather
                assert np.array_equal(outs[i], ref), f"rank {rank} M={M} bias={use_bias} call {i}"
    for key in res[0][1]:
        for r in range(1, world):
            assert np.array_equal(res[0][1][key][0], res[r][1][key][0])
    # and with the oracle of the unsharded layer (rebuilt here from the same seeds)
    K, N, G = 2048, 1024, 128
    for (M, use_bias), (outs, _) in res[0][1].items():
        X, Wd = gpu_case(M, K, N, G, sigma=0.05, seed=21 + M)
        qd = quantize_weight(Wd, G)
        ref = oracle.reference_w4a16(np_(X), *(np_(t) for t in qd), G)
        if use_bias:
            bias = (torch.randn(N, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda")
                    * 0.1).half()
            ref = (ref + np_(bias)).astype(np.float16)
        for i in range(outs.shape[0]):
            assert_gemm_close(outs[i], ref, f"fused all-gather vs oracle M={M} bias={use_bias} call {i}")
