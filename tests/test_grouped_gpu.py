"""GPU: per-group int8 dequant-matmul and quantize (popcorn src/quantize.cu:114-218, :567-697).

* popcorn's own grouped fixtures (tests/golden, made by its CPU loops) within
  its test tolerance (test/test_quantize.cu:5, TOL_PERGROUP = 1e-4 absolute),
  and bit for bit against the oracle's fused restatement;
* bit for bit against popcorn's own grouped kernel rebuilt for sm_100a, on
  small problems (the path that follows popcorn's operation order) where
  popcorn's kernel is correct (K % 32 == 0: its weight tile load reads the
  wrong elements on a K tail);
* random shapes on every kernel variant (decode M <= 4, M > 4 in chunks of
  four rows, group sizes that are not a multiple of 16, unaligned operands)
  against the oracle at the f32 path's tolerance;
* codes and scales of the quantizer bit for bit against popcorn's kernels and
  the oracle, special values included.
"""
import numpy as np
import pytest

import oracle
import popcorn_b200 as pc

pytestmark = pytest.mark.gpu

TOL_PERGROUP = 1e-4   # popcorn test/test_quantize.cu:5 (absolute)
TOL_F32 = 1e-5        # normwise, f32 path


def _dev(torch, cuda, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _grouped(torch, cuda, x, q, s, gs, x_offset=0):
    M, K = x.shape
    N = q.shape[0]
    xs = torch.zeros(M * K + x_offset + 4, dtype=torch.float32, device=cuda)
    xs[x_offset:x_offset + M * K] = _dev(torch, cuda, x.reshape(-1))
    qd, sd = _dev(torch, cuda, q), _dev(torch, cuda, s)
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    st = pc.popcornDequantizeMatmulGrouped_i8f32(out.data_ptr(), xs.data_ptr() + 4 * x_offset, qd.data_ptr(),
                                                 sd.data_ptr(), M, N, K, gs, None)
    assert st == pc.POPCORN_SUCCESS, pc.load_library().popcornGetLastCudaErrorString()
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    return out.cpu().numpy()


def _case(M, N, K, gs, seed):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, seed + 1, 0.02).reshape(N, K)
    q, s = oracle.quantize_grouped(w, gs)
    return x, q, s


@pytest.mark.parametrize("case", ["g_basic", "g_large"])
def test_reference_fixtures(cuda, golden, case):
    import torch

    x, q, s = golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"]
    gs = int(golden[f"{case}/group_size"])
    got = _grouped(torch, cuda, x, q, s, gs)
    assert np.max(np.abs(got - golden[f"{case}/out"])) <= TOL_PERGROUP
    np.testing.assert_array_equal(got, oracle.dequant_matmul_grouped(x, q, s, gs, fused=True))


@pytest.mark.skipif(not oracle.have_popcorn_ref_gpu(), reason="popcorn's kernels not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(2, 3, 32, 8), (32, 64, 128, 32), (5, 40, 256, 64), (3, 17, 96, 96)])
def test_matches_popcorn_kernel_bitwise(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s = _case(M, N, K, gs, 3 * M + N)
    got = _grouped(torch, cuda, x, q, s, gs)
    ref = pc_ref_grouped(torch, cuda, x, q, s, gs)
    np.testing.assert_array_equal(got, ref)


def pc_ref_grouped(torch, cuda, x, q, s, gs):
    lib = oracle.popcorn_ref_gpu()
    M, K = x.shape
    N = q.shape[0]
    xd, qd, sd = _dev(torch, cuda, x), _dev(torch, cuda, q), _dev(torch, cuda, s)
    out = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    assert lib.popcornDequantizeMatmulGrouped_i8f32(out.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                                    M, N, K, gs, None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("shape", [
    (1, 4096, 4096, 128), (1, 4096, 11008, 128), (1, 777, 8192, 64), (1, 300, 16384, 2048),
    (2, 4096, 4096, 64), (2, 999, 8192, 256), (3, 1000, 4096, 32), (4, 4097, 4096, 16),
    (16, 2048, 1024, 128), (33, 512, 2048, 512), (8, 300, 96, 24), (5, 1000, 4112, 16), (1, 5000, 4096, 4096),
])
def test_random_shapes_match_oracle(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s = _case(M, N, K, gs, M + N + K)
    got = _grouped(torch, cuda, x, q, s, gs)
    ref = oracle.dequant_matmul_grouped(x, q, s, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


@pytest.mark.parametrize("N,K,gs", [
    (4096, 4096, 128), (4000, 4096, 256), (2000, 4096, 1024),
    (8192, 1024, 32), (8192, 1024, 64), (6000, 2048, 64), (6000, 2048, 128), (3000, 2048, 2048),
])
def test_staged_decode_vs_oracle_and_row_split(cuda, N, K, gs):
    # The staged M = 1 kernel (tensor path, group scales applied to exact
    # per-group sums): the oracle within the f32 tolerance, each row's bits
    # independent of how rows share a CTA, and popcorn's per-element form in
    # warps holding a non-finite or extreme activation.
    import torch

    x, q, s = _case(1, N, K, gs, N + K + gs)
    got = _grouped(torch, cuda, x, q, s, gs)
    ref = oracle.dequant_matmul_grouped(x, q, s, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32
    lo, n2 = 29, (1 << 22) // K + 51  # above the sequential kernel's 2^22 multiply-adds
    sub = _grouped(torch, cuda, x, np.ascontiguousarray(q[lo:lo + n2]), np.ascontiguousarray(s[lo:lo + n2]), gs)
    assert np.array_equal(sub.view(np.uint32), got[:, lo:lo + n2].view(np.uint32))
    xi = x.copy()
    xi[0, 5] = np.inf
    xi[0, K // 2:K // 2 + 64] *= 2.0 ** -120
    got = _grouped(torch, cuda, xi, q, s, gs)
    want = oracle.dequant_matmul_grouped(xi, q, s, gs, fused=True, threads=8)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])


def test_unaligned_activations_take_the_exact_path(cuda):
    import torch

    x, q, s = _case(2, 2000, 4096, 128, 9)
    got = _grouped(torch, cuda, x, q, s, 128, x_offset=1)
    ref = oracle.dequant_matmul_grouped(x, q, s, 128, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


def test_one_group_equals_the_per_channel_call(cuda):
    import torch

    x, q, s = _case(1, 4096, 4096, 4096, 21)
    got = _grouped(torch, cuda, x, q, s, 4096)
    ref = pc.dequantize_matmul(_dev(torch, cuda, x), _dev(torch, cuda, q), _dev(torch, cuda, s[:, 0].copy()),
                               path=pc.PATH_SIMT_F32).cpu().numpy()
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


def _special_rows(N, K):
    w = oracle.fill_normal(N * K, 77, 0.02).reshape(N, K).copy()
    w[0, 3] = np.nan
    w[1, 5] = np.inf
    w[2, :] = 0.0
    w[2, 7] = -0.0
    w[3] *= 1e-38  # denormals
    w[4, :8] = np.float32([127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5])  # exact ties in group 0
    w[5, 9] = -np.inf
    return w


@pytest.mark.parametrize("shape", [(6, 64, 16), (40, 1024, 128), (9, 4096, 4096), (6, 96, 24), (7, 40, 4)])
def test_quantize_bitwise(cuda, shape):
    import torch

    N, K, gs = shape
    w = _special_rows(N, K)
    wd = _dev(torch, cuda, w)
    q, s = pc.quantize_grouped(wd, gs)
    torch.cuda.synchronize()
    qo, so = oracle.quantize_grouped(w, gs)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    if oracle.have_popcorn_ref_gpu():
        lib = oracle.popcorn_ref_gpu()
        qr = torch.zeros((N, K), dtype=torch.int8, device=cuda)
        sr = torch.zeros((N, K // gs), dtype=torch.float32, device=cuda)
        assert lib.popcornQuantizeGrouped_f32i8(qr.data_ptr(), sr.data_ptr(), wd.data_ptr(), N, K, gs, None) == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(q.cpu().numpy(), qr.cpu().numpy())
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), sr.cpu().numpy().view(np.uint32))


def test_quantize_reference_fixture(cuda, golden):
    import torch

    w = golden["qg_basic/w"]
    gs = int(golden["qg_basic/group_size"])
    q, s = pc.quantize_grouped(_dev(torch, cuda, w), gs)
    torch.cuda.synchronize()
    assert np.max(np.abs(s.cpu().numpy() - golden["qg_basic/scale"])) <= TOL_PERGROUP
    # codes: popcorn's GPU rounds half to even, its test loop half away; they
    # can differ only on exact .5 quotients
    diff = q.cpu().numpy().astype(np.int32) - golden["qg_basic/codes_test_loop"].astype(np.int32)
    assert np.all(np.abs(diff) <= 1)


# ---------------------------------------------------------------------------
# Tensor-core path (M > 4, >= 2^27 multiply-adds, group size % 32 == 0): codes
# times group scale (normalised per row by a power of two) enter the tensor
# cores as f16, activations as f16 after a per-row power of two.
# ---------------------------------------------------------------------------
TC_SHAPES = [
    (8, 4096, 4096, 128),     # single-CTA kernel, cluster split-K
    (32, 11008, 4096, 128),   # CTA pairs, 16 activation rows per CTA
    (64, 4096, 4096, 32),     # four groups per k-block
    (100, 2000, 4096, 64),    # M and N tails
    (256, 4096, 4096, 128),   # CTA pairs, 128 activation rows per CTA
    (300, 1000, 2048, 256),
    (16, 4096, 4096, 4096),   # one group per row
    (5, 8192, 4096, 512),
]


@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tensor_path_matches_oracle(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s = _case(M, N, K, gs, 7 * M + N)
    got = _grouped(torch, cuda, x, q, s, gs)
    ref = oracle.dequant_matmul_grouped(x, q, s, gs, fused=True, threads=8)
    err = oracle.normwise_rel_err(got, ref)
    assert err <= 1e-3, err   # bar: 2e-3


@pytest.mark.parametrize("magnitude", [1e-30, 1e30])
def test_tensor_path_extreme_scales(cuda, magnitude):
    # Rows whose scales differ by many orders of magnitude: each row is
    # normalised by its own power of two before f16.
    import torch

    M, N, K, gs = 16, 2048, 4096, 128
    x, q, s = _case(M, N, K, gs, 99)
    s = s.copy()
    s[::2] *= np.float32(magnitude)
    s[1::4] *= np.float32(1e-6 if magnitude > 1 else 1e6)
    got = _grouped(torch, cuda, x, q, s, gs)
    ref = oracle.dequant_matmul_grouped(x, q, s, gs, fused=True, threads=8)
    for rows in (slice(0, None, 2), slice(1, None, 4), slice(3, None, 4)):
        assert oracle.normwise_rel_err(got[:, rows], ref[:, rows]) <= 1e-3
