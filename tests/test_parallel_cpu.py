"""Tensor-parallel algebra on CPU: two gloo ranks shard a quantised weight the
way ``w4a16.parallel`` does, each computes its part with the numpy oracle, and
the gathered / reduced result must equal the unsharded oracle.

This exercises the host-side logic -- shard_columns, shard_rows,
gather_columns, all_reduce_sum -- and the collectives, without a GPU (the
per-rank GEMM on a GPU is covered by tests/test_gpu_parallel.py).
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_f32(X, qw, s, z, G):
    import oracle
    W = oracle.dequantize_weight(qw, s, z, G).astype(np.float32)
    return X.astype(np.float32) @ W


def _rank_main(rank: int, world: int, port: int, q) -> None:
    try:
        for p in (os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200"), ROOT):
            sys.path.insert(0, p)
        import torch.distributed as dist
        import oracle
        from w4a16.parallel import all_reduce_sum, gather_columns, shard_columns, shard_rows

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(5)
        M, K, N, G = 3, 512, 96, 64
        X = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
        W = (rng.standard_normal((K, N), dtype=np.float32) * 0.05).astype(np.float16)
        qw, s, z = oracle.quantize_weight(W, G)
        full = oracle.reference_w4a16(X, qw, s, z, G)

        # column-parallel: local slice, then all-gather
        tq, ts, tz = (torch.from_numpy(a) for a in (qw, s, z))
        cq, cs, cz, _ = shard_columns(tq, ts, tz, rank, world)
        y_loc = torch.from_numpy(oracle.reference_w4a16(X, cq.numpy(), cs.numpy(), cz.numpy(), G))
        y = gather_columns(y_loc)
        col_ok = bool(np.array_equal(y.numpy(), full))

        # row-parallel: K-slice of x and of the weight, fp32 partials, all-reduce
        rq, rs, rz = shard_rows(tq, ts, tz, G, rank, world)
        k = K // world
        part = torch.from_numpy(_oracle_f32(X[:, rank * k:(rank + 1) * k], rq.numpy(), rs.numpy(),
                                            rz.numpy(), G))
        y_row = all_reduce_sum(part).to(torch.float16).numpy().astype(np.float32)
        ref = full.astype(np.float32)
        row_ok = bool(np.all(np.abs(y_row - ref) <= 1e-2 + 1e-3 * np.abs(ref)))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, col_ok, row_ok, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, False, repr(e)))


def test_two_rank_column_and_row_parallel_algebra():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, col_ok, row_ok, err in sorted(results):
        assert err is None, f"rank {rank}: {err}"
        assert col_ok, f"rank {rank}: gathered column shards differ from the unsharded oracle"
        assert row_ok, f"rank {rank}: reduced row shards outside the tolerance"


def test_shard_shapes_and_errors():
    from w4a16.parallel import shard_columns, shard_rows
    qw = torch.arange(64 * 96, dtype=torch.int32).view(64, 96)
    s = torch.ones(8, 96, dtype=torch.float16)
    z = torch.zeros(8, 96, dtype=torch.float16)
    parts = [shard_columns(qw, s, z, r, 4) for r in range(4)]
    assert torch.equal(torch.cat([p[0] for p in parts], dim=1), qw)
    assert all(p[0].is_contiguous() and p[0].shape == (64, 24) for p in parts)
    rows = [shard_rows(qw, s, z, 64, r, 2) for r in range(2)]
    assert torch.equal(torch.cat([r[0] for r in rows], dim=0), qw)
    assert rows[0][1].shape == (4, 96)
    with pytest.raises(AssertionError):
        shard_rows(qw, s, z, 128, 0, 8)       # 512/8 = 64 rows per rank is not a multiple of 128
    with pytest.raises(AssertionError):
        shard_columns(qw, s, z, 0, 5)          # 96 columns do not split over 5 ranks
