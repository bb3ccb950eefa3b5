"""GPU: the allocation-free tensor-path entry point, through the C ABI.

popcornDequantizeMatmulNoAlloc_i8f32 exists for callers that cannot let a
library allocate device memory (they hand out all GPU memory through their own
allocator, or forbid allocation after start-up). It keeps its scratch in one
fixed device array inside the library, so it must give the same answers as the
allocating tensor path -- including on a second call, which reuses the array
the first call left behind. This file is collected last so that a run which
stops at the first failure has already run every other test; it also passes
when run alone in a fresh process.
"""
import numpy as np
import pytest

import oracle
import popcorn_b200 as pc

pytestmark = pytest.mark.gpu

TOL_TENSOR = 2e-3  # normwise, the tensor path's tolerance


def _dev(torch, cuda, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _inputs(M, N, K, seed):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, seed + 1, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)
    return x, q, s


def _run_both(torch, cuda, x, q, s):
    M, K = x.shape
    N = q.shape[0]
    xd, qd, sd = _dev(torch, cuda, x), _dev(torch, cuda, q), _dev(torch, cuda, s)
    got = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    ref = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    st = pc.popcornDequantizeMatmulNoAlloc_i8f32(got.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                                 M, N, K, None)
    assert st == pc.POPCORN_SUCCESS, pc.load_library().popcornGetLastCudaErrorString()
    st = pc.popcornDequantizeMatmulPath_i8f32(ref.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                              M, N, K, pc.PATH_TENSOR_F16, None)
    assert st == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    return got.cpu().numpy(), ref.cpu().numpy()


def test_no_alloc_matches_allocating_path_twice_in_a_row(cuda):
    import torch

    # Two calls back to back with different shapes and data: the second
    # reuses the array the first one filled.
    for (M, N, K, seed) in [(300, 384, 2048, 11), (64, 200, 4096, 12)]:
        x, q, s = _inputs(M, N, K, seed)
        got, ref = _run_both(torch, cuda, x, q, s)
        assert np.isfinite(got).all()
        assert oracle.normwise_rel_err(got, ref) <= TOL_TENSOR
        np.testing.assert_array_equal(got, ref)  # same kernels, same inputs
        assert oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s, fused=True, threads=8)) <= TOL_TENSOR


def test_no_alloc_rejects_sizes_beyond_its_array(cuda):
    import torch

    lib = pc.load_library()
    q = torch.zeros((128, 4096), dtype=torch.int8, device=cuda)
    s = torch.ones((128,), dtype=torch.float32, device=cuda)
    x = torch.zeros((1, 16), dtype=torch.float32, device=cuda)
    out = torch.zeros((1, 16), dtype=torch.float32, device=cuda)
    # M*K*2 = 2049*4096*2 > 16 MiB, and M > 16384: rejected before any launch.
    assert lib.popcornDequantizeMatmulNoAlloc_i8f32(out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(),
                                                    2049, 128, 4096, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert lib.popcornDequantizeMatmulNoAlloc_i8f32(out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(),
                                                    16385, 128, 16, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # K % 16 != 0 is a shape the tensor path cannot run.
    assert lib.popcornDequantizeMatmulNoAlloc_i8f32(out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(),
                                                    1, 128, 40, None) == pc.POPCORN_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
