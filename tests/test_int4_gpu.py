"""GPU: int4 packed asymmetric per-group dequant-matmul and quantize
(popcorn src/quantize.cu:329-446, :699-888).

* popcorn's own int4 fixtures (tests/golden, made by its CPU loops) within its
  test tolerance (test/test_quantize.cu:5, TOL_PERGROUP = 1e-4 absolute), and
  bit for bit against the oracle's fused restatement;
* bit for bit against popcorn's own int4 kernel rebuilt for sm_100a on the
  shapes that take the path following popcorn's operation order (small
  problems, odd group sizes, group sizes that are not a multiple of 16);
* random shapes on every decode variant (M <= 4, M > 4 in chunks of four
  rows) and the fallbacks (unaligned operands, K % 16 != 0) against the
  oracle at the f32 path's tolerance;
* packed codes, scales and zero points of the quantizer bit for bit against
  popcorn's kernels and the oracle: NaN, infinities, denormals, exact .5
  quotients, signed zeros, odd group sizes whose bytes straddle two groups.
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


def _matmul(torch, cuda, x, q, s, z, gs, x_offset=0, q_offset=0):
    M, K = x.shape
    N = q.shape[0]
    xs = torch.zeros(M * K + x_offset + 4, dtype=torch.float32, device=cuda)
    xs[x_offset:x_offset + M * K] = _dev(torch, cuda, x.reshape(-1))
    qs = torch.zeros(q.size + q_offset + 16, dtype=torch.uint8, device=cuda)
    qs[q_offset:q_offset + q.size] = _dev(torch, cuda, q.reshape(-1))
    sd, zd = _dev(torch, cuda, s), _dev(torch, cuda, z)
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    st = pc.popcornDequantizeMatmulGrouped_i4f32(out.data_ptr(), xs.data_ptr() + 4 * x_offset,
                                                 qs.data_ptr() + q_offset, sd.data_ptr(), zd.data_ptr(), M, N, K, gs,
                                                 None)
    assert st == pc.POPCORN_SUCCESS, pc.load_library().popcornGetLastCudaErrorString()
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    return out.cpu().numpy()


def _popcorn_matmul(torch, cuda, x, q, s, z, gs):
    lib = oracle.popcorn_ref_gpu()
    M, K = x.shape
    N = q.shape[0]
    xd, qd, sd, zd = (_dev(torch, cuda, a) for a in (x, q, s, z))
    out = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    assert lib.popcornDequantizeMatmulGrouped_i4f32(out.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                                    zd.data_ptr(), M, N, K, gs, None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _case(M, N, K, gs, seed):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, seed + 1, 0.02).reshape(N, K)
    q, s, z = oracle.quantize_grouped_i4(w, gs)
    return x, q, s, z


@pytest.mark.parametrize("case", ["i4_basic", "i4_large"])
def test_reference_fixtures(cuda, golden, case):
    import torch

    x, q = golden[f"{case}/x"], golden[f"{case}/q"]
    s, z = golden[f"{case}/scale"], golden[f"{case}/zero"]
    gs = int(golden[f"{case}/group_size"])
    got = _matmul(torch, cuda, x, q, s, z, gs)
    assert np.max(np.abs(got - golden[f"{case}/out"])) <= TOL_PERGROUP
    np.testing.assert_array_equal(got, oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True))


@pytest.mark.skipif(not oracle.have_popcorn_ref_gpu(), reason="popcorn's kernels not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(2, 3, 32, 8), (16, 32, 64, 32), (5, 40, 256, 64), (3, 17, 96, 96), (4, 7, 30, 3),
                                   (2, 5, 36, 6), (1, 64, 100, 50)])
def test_matches_popcorn_kernel_bitwise(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s, z = _case(M, N, K, gs, 3 * M + N)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    np.testing.assert_array_equal(got, _popcorn_matmul(torch, cuda, x, q, s, z, gs))
    np.testing.assert_array_equal(got, oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True))


@pytest.mark.parametrize("shape", [
    (1, 4096, 4096, 128), (1, 4096, 11008, 128), (1, 777, 8192, 64), (1, 300, 16384, 2048),
    (2, 4096, 4096, 64), (2, 999, 8192, 256), (3, 1000, 4096, 32), (4, 4097, 4096, 16),
    (16, 2048, 1024, 128), (33, 512, 2048, 512), (8, 300, 96, 24), (5, 1000, 4112, 16), (1, 5000, 4096, 4096),
    (2, 3000, 1030, 10), (1, 2000, 4098, 2),
    # staged decode (M = 1, K <= 4096, rows in shared memory): ragged row
    # counts per SM, one row per CTA, 41 rows per CTA
    (1, 1000, 4096, 32), (1, 100, 2048, 64), (1, 6000, 4096, 128),
])
def test_random_shapes_match_oracle(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s, z = _case(M, N, K, gs, M + N + K)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


@pytest.mark.parametrize("N,K,gs", [(8192, 1024, 64), (6000, 2048, 128), (6000, 1024, 256), (3000, 2048, 512),
                                    (4096, 4096, 128), (3000, 4096, 512), (2000, 4096, 1024)])
def test_tensor_path_decode_vs_oracle_and_row_split(cuda, N, K, gs):
    # The M = 1 tensor-path kernel (codes unpacked to bytes, mma.sync against
    # fixed-point digits, zero points through exact group sums of x): the
    # oracle within the f32 tolerance, and each row's bits independent of
    # how rows share a CTA.
    import torch

    x, q, s, z = _case(1, N, K, gs, N + K + gs)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32
    lo, n2 = 29, (1 << 22) // K + 51  # above the sequential kernel's 2^22 multiply-adds
    sub = _matmul(torch, cuda, x, np.ascontiguousarray(q[lo:lo + n2]), np.ascontiguousarray(s[lo:lo + n2]),
                  np.ascontiguousarray(z[lo:lo + n2]), gs)
    assert np.array_equal(sub.view(np.uint32), got[:, lo:lo + n2].view(np.uint32))


@pytest.mark.parametrize("kind", ["nan", "inf", "tiny"])
def test_decode_nonfinite_and_tiny_activations(cuda, kind):
    # M = 1 with a NaN, an infinity or a slice of denormals in x: those warps
    # leave the fixed-point layout; every output must match the oracle's
    # (non-finite exactly where popcorn's sum is).
    import torch

    M, N, K, gs = 1, 2000, 4096, 128
    x, q, s, z = _case(M, N, K, gs, 31)
    x = x.copy()
    if kind == "nan":
        x[0, 37] = np.nan
    elif kind == "inf":
        x[0, 1000] = np.inf
    else:
        x[0, 2048:2064] = np.float32(1e-40)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    if fin.any():
        assert oracle.normwise_rel_err(got[fin], ref[fin]) <= TOL_F32
        assert np.array_equal(np.sign(got[~fin & ~np.isnan(ref)]), np.sign(ref[~fin & ~np.isnan(ref)]))


@pytest.mark.parametrize("offsets", [(1, 0), (0, 1), (0, 4)])
def test_unaligned_operands_take_the_exact_path(cuda, offsets):
    import torch

    x, q, s, z = _case(2, 2000, 4096, 128, 9)
    got = _matmul(torch, cuda, x, q, s, z, 128, x_offset=offsets[0], q_offset=offsets[1])
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, 128, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


def test_off_centre_zero_points(cuda):
    # Groups of one sign only: zero points far from 8 (all-positive groups
    # have zero < 0), the case where the decode layout's centred codes cancel
    # least.
    import torch

    M, N, K, gs = 1, 2048, 4096, 64
    x = oracle.fill_normal(M * K, 5, 1.0).reshape(M, K)
    w = np.abs(oracle.fill_normal(N * K, 6, 0.02)).reshape(N, K) + np.float32(0.05)
    w[::2] *= -1.0
    q, s, z = oracle.quantize_grouped_i4(w, gs)
    assert z.min() < -10 and z.max() > 20
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


def _bits(a):
    """Bit patterns with every NaN made one pattern: the GPU's canonical NaN
    (0x7fffffff) and the host's (0xffc00000) are the same value."""
    a = np.asarray(a, dtype=np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FFFFFFF), a.view(np.uint32))


def _special_rows(N, K):
    w = oracle.fill_normal(N * K, 77, 0.02).reshape(N, K).copy()
    w[0, 3] = np.nan
    w[1, 5] = np.inf
    w[2, :] = 0.0
    w[2, 7] = -0.0
    w[3] *= 1e-38  # denormals
    # groups holding both 0 and 15 get scale 1, zero 0: every .5 is a tie
    w[4, :] = np.resize(np.float32([15, 0, 0.5, 1.5, 2.5, 3.5, 14.5, 7.5]), K)
    w[5, 9] = -np.inf
    if N > 6:
        w[6, :] = -0.0   # all zeros, mixed signs: the sign of zero follows the block order
        w[6, 1::3] = 0.0
    if N > 7:
        w[7, :] = np.nan
    return w


@pytest.mark.parametrize("shape", [(6, 64, 16), (40, 1024, 128), (9, 4096, 4096), (8, 96, 24), (8, 42, 3), (8, 30, 5),
                                   (8, 1024, 512), (9, 4096, 2048), (7, 300, 300)])
def test_quantize_bitwise(cuda, shape):
    import torch

    N, K, gs = shape
    w = _special_rows(N, K)
    wd = _dev(torch, cuda, w)
    q, s, z = pc.quantize_grouped_i4(wd, gs)
    torch.cuda.synchronize()
    qo, so, zo = oracle.quantize_grouped_i4(w, gs)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))
    np.testing.assert_array_equal(_bits(z.cpu().numpy()), _bits(zo))
    if oracle.have_popcorn_ref_gpu():
        lib = oracle.popcorn_ref_gpu()
        qr = torch.zeros((N, K // 2), dtype=torch.uint8, device=cuda)
        sr = torch.zeros((N, K // gs), dtype=torch.float32, device=cuda)
        zr = torch.zeros((N, K // gs), dtype=torch.float32, device=cuda)
        assert lib.popcornQuantizeGrouped_f32i4(qr.data_ptr(), sr.data_ptr(), zr.data_ptr(), wd.data_ptr(), N, K, gs,
                                                None) == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(q.cpu().numpy(), qr.cpu().numpy())
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), sr.cpu().numpy().view(np.uint32))
        np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), zr.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("gs", [256, 512, 1024])
def test_quantize_signed_zero_groups(cuda, gs):
    import torch

    rng = np.random.default_rng(gs)
    N = 64
    w = np.zeros((N, gs), dtype=np.float32)
    for r in range(N):
        w[r, rng.choice(gs, size=int(rng.integers(1, 6)), replace=False)] = -0.0
    q, s, z = pc.quantize_grouped_i4(_dev(torch, cuda, w), gs)
    torch.cuda.synchronize()
    _, so, zo = oracle.quantize_grouped_i4(w, gs)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), zo.view(np.uint32))
    assert np.all(q.cpu().numpy() == 0)


def test_quantize_reference_fixture(cuda, golden):
    import torch

    w = golden["qi4_basic/w"]
    gs = int(golden["qi4_basic/group_size"])
    q, s, z = pc.quantize_grouped_i4(_dev(torch, cuda, w), gs)
    torch.cuda.synchronize()
    assert np.max(np.abs(s.cpu().numpy() - golden["qi4_basic/scale"])) <= TOL_PERGROUP
    assert np.max(np.abs(z.cpu().numpy() - golden["qi4_basic/zero"])) <= TOL_PERGROUP
    # codes: popcorn's GPU rounds half to even, its test loop half away; they
    # can differ only on exact .5 quotients
    got = q.cpu().numpy()
    ref = golden["qi4_basic/packed_test_loop"]
    for shift in (0, 4):
        d = ((got >> shift) & 15).astype(np.int32) - ((ref >> shift) & 15).astype(np.int32)
        assert np.all(np.abs(d) <= 1)


def test_quantize_then_matmul(cuda):
    import torch

    M, N, K, gs = 1, 4096, 4096, 128
    x = oracle.fill_normal(M * K, 11, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, 12, 0.02).reshape(N, K)
    q, s, z = pc.quantize_grouped_i4(_dev(torch, cuda, w), gs)
    out = pc.dequantize_matmul_grouped_i4(_dev(torch, cuda, x), q, s, z, gs)
    torch.cuda.synchronize()
    qo, so, zo = oracle.quantize_grouped_i4(w, gs)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    ref = oracle.dequant_matmul_grouped_i4(x, qo, so, zo, gs, fused=True, threads=8)
    assert oracle.normwise_rel_err(out.cpu().numpy(), ref) <= TOL_F32
    # 4-bit codes: the product is within the quantization error of x @ w.T
    # (0.085 normwise for these inputs on the oracle)
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    assert oracle.normwise_rel_err(out.cpu().numpy(), exact) <= 0.15


# ---------------------------------------------------------------------------
# Tensor-core path (M > 4, >= 2^27 multiply-adds, group size % 32 == 0): the
# converters unpack the nibbles and write (code - zero) * scale, normalised per
# row by a power of two, to tensor memory as f16.
# ---------------------------------------------------------------------------
TC_SHAPES = [
    (8, 4096, 4096, 128),
    (32, 11008, 4096, 128),
    (64, 4096, 4096, 32),
    (100, 2000, 4096, 64),
    (256, 4096, 4096, 128),
    (300, 1000, 2048, 256),
    (16, 4096, 4096, 4096),
    (5, 8192, 4096, 512),
]


@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tensor_path_matches_oracle(cuda, shape):
    import torch

    M, N, K, gs = shape
    x, q, s, z = _case(M, N, K, gs, 7 * M + N)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    err = oracle.normwise_rel_err(got, ref)
    assert err <= 1e-3, err   # bar: 2e-3


def test_tensor_path_off_centre_and_extreme(cuda):
    import torch

    M, N, K, gs = 24, 2048, 4096, 64
    x = oracle.fill_normal(M * K, 5, 1.0).reshape(M, K)
    w = np.abs(oracle.fill_normal(N * K, 6, 0.02)).reshape(N, K) + np.float32(0.05)
    w[::2] *= -1.0
    q, s, z = oracle.quantize_grouped_i4(w, gs)
    s = s.copy()
    s[::3] *= np.float32(1e-25)
    s[1::3] *= np.float32(1e25)
    got = _matmul(torch, cuda, x, q, s, z, gs)
    ref = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, fused=True, threads=8)
    for rows in (slice(0, None, 3), slice(1, None, 3), slice(2, None, 3)):
        assert oracle.normwise_rel_err(got[:, rows], ref[:, rows]) <= 1e-3
