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
from popcorn_b200.tp import (STACK_PARTS, ColumnParallelLinear, LinearStack, RowParallelLinear, shard_bounds,
                             shard_stack_layer, stack_part_shape)


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


SMALL_STACK = {"hidden": 64, "qkv": 192, "ffn": 176}


def small_stack_weights(layers):
    full = []
    for i in range(layers):
        layer = {}
        for j, part in enumerate(STACK_PARTS):
            N, K = stack_part_shape(SMALL_STACK, part)
            w = oracle.fill_normal(N * K, 100 + 10 * i + j, 0.02).reshape(N, K)
            q, s = oracle.quantize(w)
            layer[part] = (torch.from_numpy(q), torch.from_numpy(s))
        full.append(layer)
    return full


def stack_reference(full, x, world):
    """The stack computed whole on one device, with the o projection reading
    the same qkv columns that the ranks' shards feed it."""
    h = x
    hid = SMALL_STACK["hidden"]
    for layer in full:
        a = oracle.dequant_matmul(h, layer["qkv"][0].numpy(), layer["qkv"][1].numpy())
        cols = []
        for r in range(world):
            lo, _ = shard_bounds(SMALL_STACK["qkv"], world, r)
            klo, khi = shard_bounds(hid, world, r)
            cols.append(a[:, lo:lo + (khi - klo)])
        xo = np.ascontiguousarray(np.concatenate(cols, axis=1))
        h1 = oracle.dequant_matmul(xo, layer["o"][0].numpy(), layer["o"][1].numpy())
        g = oracle.dequant_matmul(h1, layer["gate"][0].numpy(), layer["gate"][1].numpy())
        h = oracle.dequant_matmul(g, layer["down"][0].numpy(), layer["down"][1].numpy())
    return h


def _stack_worker(rank, world, port, M, layers, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = small_stack_weights(layers)
        shards = [shard_stack_layer(layer, rank, world) for layer in full]
        stack = LinearStack(shards, M, SMALL_STACK, torch.device("cpu"), local_matmul=oracle_matmul)
        x = torch.from_numpy(oracle.fill_normal(M * SMALL_STACK["hidden"], 7, 1.0).reshape(M, -1))
        ret[rank] = stack(x).numpy().copy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 3, 6])
def test_linear_stack_gloo_world2(M):
    world, layers = 2, 2
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = free_port()
    procs = [ctx.Process(target=_stack_worker, args=(r, world, port, M, layers, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x = oracle.fill_normal(M * SMALL_STACK["hidden"], 7, 1.0).reshape(M, -1)
    ref = stack_reference(small_stack_weights(layers), x, world)
    np.testing.assert_array_equal(ret[0], ret[1])  # all ranks agree
    assert oracle.normwise_rel_err(ret[0], ref) <= 1e-5


def test_linear_stack_single_rank_is_the_plain_chain():
    # world 1 (no process group): every projection is one plain call.
    M = 2
    full = small_stack_weights(1)
    stack = LinearStack([shard_stack_layer(full[0], 0, 1)], M, SMALL_STACK, torch.device("cpu"),
                        local_matmul=oracle_matmul)
    x = oracle.fill_normal(M * SMALL_STACK["hidden"], 7, 1.0).reshape(M, -1)
    np.testing.assert_array_equal(stack(torch.from_numpy(x)).numpy(), stack_reference(full, x, 1))
