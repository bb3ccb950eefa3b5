"""GPU (2+ devices): the decode GEMVs with their collective fused over NVLink.

Two ranks (spawned processes, one GPU each; NCCL only to set up the group and
to compare results) share one PeerGroup and run, in the same order on both:

* popcornDequantizeMatmulAllGather_i8f32 on their shards of one weight
  matrix -- every rank's gathered [M, N] output must equal a single-GPU
  popcornDequantizeMatmul_i8f32 of the whole matrix bit for bit (each output
  channel is computed whole on one rank with the same arithmetic);
* popcornDequantizeMatmulAllReduce_i8f32 on their slices of the input
  channels -- every rank must hold the same bits, within f32 rounding
  (1e-5 normwise) of the single-GPU call over the whole K.

Shapes and the two kinds of call are interleaved on one group, several calls
in a row, with N and K that do not split evenly, so consecutive calls of
different sizes share the receive areas.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, port, cases, ret):
    import datetime

    import torch.distributed as dist

    import oracle
    import popcorn_b200 as pc
    from popcorn_b200.tp import FusedColumnParallelLinear, FusedRowParallelLinear, PeerGroup

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        peer = PeerGroup(4, 12288, dev)
        layers = []
        for (kind, M, N, K) in cases:
            x = torch.from_numpy(oracle.fill_normal(M * K, 1, 1.0).reshape(M, K)).to(dev)
            w = oracle.fill_normal(N * K, 2, 0.02).reshape(N, K)
            qn, sn = oracle.quantize(w)
            q, s = torch.from_numpy(qn).to(dev), torch.from_numpy(sn).to(dev)
            layer = (FusedColumnParallelLinear if kind == "gather" else FusedRowParallelLinear)(q, s, peer)
            layers.append((kind, x, q, s, layer))
        results = []
        for rep in range(3):
            for (kind, x, q, s, layer) in layers:
                xi = x * (rep + 1)
                y = layer(xi)
                ref = pc.dequantize_matmul(xi, q, s, path=pc.PATH_SIMT_F32)
                torch.cuda.synchronize()
                if kind == "gather":
                    good = bool(torch.equal(y, ref))
                    err = 0.0
                else:
                    err = float(((y - ref).abs().max() / ref.abs().max()).item())
                    good = err <= 1e-5
                    # every rank must hold identical bits
                    ys = [torch.empty_like(y) for _ in range(WORLD)]
                    dist.all_gather(ys, y)
                    good = good and all(torch.equal(ys[0], t) for t in ys)
                results.append((kind, tuple(y.shape), good, err))
        errs = pc.device_errors()
        dist.barrier()
        ret[rank] = (results, errs)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
def test_fused_collectives_match_single_gpu():
    import torch.multiprocessing as mp

    cases = [
        ("gather", 1, 4096, 4096),
        ("reduce", 1, 4096, 4096),
        ("gather", 2, 1000, 4096),
        ("reduce", 1, 4096, 11008),
        ("gather", 1, 777, 8192),
        ("reduce", 3, 4096, 1376),
        ("gather", 4, 12288, 4096),
        ("reduce", 2, 999, 4096),
    ]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    ret = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, cases, ret)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(WORLD):
        results, errs = ret[r]
        assert errs == 0, r
        assert len(results) == 3 * len(cases)
        for (kind, shape, good, err) in results:
            assert good, (r, kind, shape, err)
