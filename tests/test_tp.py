"""CPU: the tensor-parallel host logic with world_size 2 gloo ranks.

The per-rank matmul is the oracle (popcorn's k order, f32), injected into the
layers, so the test checks sharding, padding, all-gather reassembly and
all-reduce exactly as the GPU path runs them; the GPU path differs only in
the per-rank call (the library's C ABI) and the backend (NCCL).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from popcorn_b200.tp import ColumnParallelLinear, RowParallelLinear, shard_bounds


def oracle_matmul(x, q, s):
    return torch.from_numpy(oracle.dequant_matmul(x.numpy(), q.numpy(), s.numpy()))


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, case, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, N, K = case
        x = torch.from_numpy(oracle.fill_normal(M * K, 1, 1.0).reshape(M, K))
        w = oracle.fill_normal(N * K, 2, 0.02).reshape(N, K)
        qn, sn = oracle.quantize(w)
        q, s = torch.from_numpy(qn), torch.from_numpy(sn)
        col = ColumnParallelLinear(q, s, local_matmul=oracle_matmul)
        y_col = col(x)
        row = RowParallelLinear(q, s, local_matmul=oracle_matmul)
        y_row = row(x)
        ret[rank] = (y_col.numpy().copy(), y_row.numpy().copy())
    finally:
        dist.destroy_process_group()


def run_ranks(world, case):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    ret = mgr.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return dict(ret)


def test_shard_bounds_cover_exactly():
    for n in (1, 7, 4096, 11008):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


@pytest.mark.parametrize("case", [(1, 64, 96), (3, 37, 50)])
def test_column_and_row_parallel_gloo_world2(case):
    M, N, K = case
    ret = run_ranks(2, case)
    x = oracle.fill_normal(M * K, 1, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, 2, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)
    ref = oracle.dequant_matmul(x, q, s)
    for r in range(2):
        y_col, y_row = ret[r]
        # Column-parallel: each output channel is computed whole on one rank,
        # so the gathered result is bit-identical to the single-device one.
        np.testing.assert_array_equal(y_col, ref)
        # Row-parallel: two partial k-sums added; f32 rounding only.
        assert oracle.normwise_rel_err(y_row, ref) <= 1e-5
    np.testing.assert_array_equal(ret[0][1], ret[1][1])  # all ranks agree
