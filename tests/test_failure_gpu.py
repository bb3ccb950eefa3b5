"""GPU (one device): a fused collective whose peer never answers gives up.

The decode GEMVs with a fused all-gather or all-reduce wait for other ranks'
values in device memory. Each wait is bounded (1 s of %globaltimer); when it
runs out the kernel records bit 0x100 in its error word, leaves the missing
outputs unwritten and returns, so the context stays usable and the host learns
of the failure through popcornB200DeviceErrors (where the decode kernels'
bits sit 16 places up).

Here rank 0 of a two-rank group runs alone: rank 1's "receive area" is a
second buffer on this GPU that nothing ever writes into, so every value rank
0 waits for is missing. Nothing faults or hangs: the wait is made to run out,
which is the failure the bound exists for. Afterwards an ordinary call on the
same device must still be right.
"""
import ctypes
import time

import numpy as np
import pytest

import oracle
import popcorn_b200 as pc

pytestmark = pytest.mark.gpu

PEER_TIMEOUT_BIT = 0x100 << 16   # decode-kernel bit 0x100, as popcornB200DeviceErrors reports it


def _lonely_group(torch, cuda, M, N):
    """Rank 0 of world 2 whose rank-1 area is a local buffer nobody fills."""
    words = 2 * 2 * M * N  # two halves, each an all-reduce of [M, N] over 2 ranks
    recv = [torch.zeros((words,), dtype=torch.int64, device=cuda) for _ in range(2)]
    state = torch.zeros((2,), dtype=torch.int32, device=cuda)
    g = pc.TpGroup()
    g.recv[0], g.recv[1] = recv[0].data_ptr(), recv[1].data_ptr()
    g.recv_bytes = 8 * words
    g.state = state.data_ptr()
    g.rank, g.world = 0, 2
    return g, recv, state


def _case(M, N, K, seed):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    q, s = oracle.quantize(oracle.fill_normal(N * K, seed + 1, 0.02).reshape(N, K))
    return x, q, s


@pytest.mark.parametrize("kind", ["all_reduce", "all_gather"])
def test_missing_peer_times_out_and_is_reported(cuda, kind):
    import torch

    lib = pc.load_library()
    assert pc.device_errors() == 0
    M, N, K = 1, 1024, 2048
    x, q, s = _case(M, N, K, 5)
    xd, qd, sd = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (x, q, s))
    g, recv, state = _lonely_group(torch, cuda, M, N)
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if kind == "all_reduce":
        st = lib.popcornDequantizeMatmulAllReduce_i8f32(ctypes.byref(g), out.data_ptr(), xd.data_ptr(),
                                                        qd.data_ptr(), sd.data_ptr(), M, N, K, None)
    else:
        # rank 0 owns the first half of the output channels
        st = lib.popcornDequantizeMatmulAllGather_i8f32(ctypes.byref(g), out.data_ptr(), xd.data_ptr(),
                                                        qd.data_ptr(), sd.data_ptr(), M, 0, N // 2, N, K, None)
    assert st == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 0.9 <= waited <= 10.0, waited
    flags = pc.device_errors()
    assert flags & PEER_TIMEOUT_BIT, hex(flags)
    assert pc.device_errors() == 0  # reading clears the bits
    got = out.cpu().numpy()
    if kind == "all_gather":
        # this rank's own channels were written; the other rank's never arrived
        ref = oracle.dequant_matmul(x, q[: N // 2], s[: N // 2], fused=True, threads=8)
        assert oracle.normwise_rel_err(got[:, : N // 2], ref) <= 1e-5
        assert np.isnan(got[:, N // 2:]).all()
    # the call count still advanced (the kernel ran to its end)
    assert int(state[0].item()) == 1

    # The context is still usable: an ordinary call right after is correct.
    y = pc.dequantize_matmul(xd, qd, sd)
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    assert oracle.normwise_rel_err(y.cpu().numpy(), ref) <= 1e-5
