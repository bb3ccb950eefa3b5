"""GPU: the fused neighbours of the dequant-matmul (include/popcorn_b200.h):
RMSNorm -> DequantizeMatmul and DequantizeMatmul(gate), DequantizeMatmul(up)
-> Silu -> Mul, each in one call.

* popcorn's own RMSNorm and SiLU fixtures (test/test_reduction.cu:511-583,
  test/test_unary.cu:356-381, tolerance 1e-5) through the fused calls with
  identity weights;
* every path (decode layout M <= 4, tensor cores M > 4, the unfused sequence
  for small or unaligned problems) against the oracle's composition of
  popcorn's RMSNorm, matmul and SiLU, and against popcorn's own GPU kernels
  run as the sequence (RMSNorm_f32, DequantizeMatmul_i8f32, Silu_f32, Mul_f32).
"""
import numpy as np
import pytest

import oracle
import popcorn_b200 as pc

pytestmark = pytest.mark.gpu

TOL = 1e-5            # popcorn test/test_reduction.cu:4, test/test_unary.cu:4 (absolute)
TOL_F32 = 1e-5        # normwise, f32 path
TOL_TC = 1e-3         # normwise asserted for the tensor path (bar 2e-3)
EPS = 1e-5


def _dev(torch, cuda, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _ref(x, nw, q, s, qu=None, su=None, norm=True):
    xin = oracle.rmsnorm(x, nw, EPS) if norm else x
    g = oracle.dequant_matmul(xin, q, s, fused=True, threads=8)
    if qu is None:
        return g
    u = oracle.dequant_matmul(xin, qu, su, fused=True, threads=8)
    return oracle.silu(g) * u


def _run(torch, cuda, x, nw, q, s, qu=None, su=None, norm=True, x_offset=0):
    M, K = x.shape
    xs = torch.zeros(M * K + x_offset + 4, dtype=torch.float32, device=cuda)
    xs[x_offset:x_offset + M * K] = _dev(torch, cuda, x.reshape(-1))
    xd = xs[x_offset:x_offset + M * K].view(M, K)
    nwd = None if nw is None else _dev(torch, cuda, nw)
    args = [_dev(torch, cuda, a) for a in (q, s)]
    if qu is None:
        out = pc.rmsnorm_dequantize_matmul(xd, nwd, EPS, *args)
    else:
        out = pc.dequantize_matmul_silu_mul(xd, *args, _dev(torch, cuda, qu), _dev(torch, cuda, su),
                                            norm_weight=nwd, eps=EPS if norm else None)
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    return out.cpu().numpy()


def _case(M, N, K, seed, glu):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    nw = (np.float32(1.0) + oracle.fill_normal(K, seed + 7, 0.1)).astype(np.float32)
    q, s = oracle.quantize(oracle.fill_normal(N * K, seed + 1, 0.02).reshape(N, K))
    qu = su = None
    if glu:
        qu, su = oracle.quantize(oracle.fill_normal(N * K, seed + 2, 0.02).reshape(N, K))
    return x, nw, q, s, qu, su


def test_popcorn_rmsnorm_fixtures_through_identity_weights(cuda):
    import torch

    eye_q = np.eye(4, dtype=np.int8)
    ones = np.ones(4, dtype=np.float32)
    # rmsnorm_basic (test_reduction.cu:511-545): 2 rows, no weight
    x = np.float32([[1, 2, 3, 4], [2, 2, 2, 2]])
    rms0 = np.sqrt(np.float32((1 + 4 + 9 + 16) / 4.0) + np.float32(EPS), dtype=np.float32)
    rms1 = np.sqrt(np.float32(4.0) + np.float32(EPS), dtype=np.float32)
    expected = np.vstack([x[0] / rms0, x[1] / rms1]).astype(np.float32)
    got = _run(torch, cuda, x, None, eye_q, ones)
    assert np.max(np.abs(got - expected)) <= TOL
    # rmsnorm_with_weight (:547-583)
    x = np.float32([[1, 2, 3, 4]])
    w = np.float32([0.5, 1.0, 1.5, 2.0])
    expected = ((x / rms0) * w).astype(np.float32)
    got = _run(torch, cuda, x, w, eye_q, ones)
    assert np.max(np.abs(got - expected)) <= TOL


def test_popcorn_silu_fixture_through_identity_weights(cuda):
    # silu_basic (test_unary.cu:356-381): gate = up = identity gives silu(x) * x.
    import torch

    x = np.float32([[0.0, 1.0, -1.0, 2.0, -2.0]])
    eye_q = np.eye(5, dtype=np.int8)
    ones = np.ones(5, dtype=np.float32)
    expected = (x / (np.float32(1) + np.exp(-x, dtype=np.float32))) * x
    got = _run(torch, cuda, x, None, eye_q, ones, eye_q, ones, norm=False)
    assert np.max(np.abs(got - expected)) <= TOL


# (M, N, K): decode layout with one, two and four K slices per thread, 2 and 3
# activation rows, tensor cores (single CTA with split-K, CTA pairs), the
# unfused sequence (K % 16 != 0).
SHAPES = [(1, 4096, 4096), (1, 11008, 4096), (1, 4096, 11008), (1, 1000, 16384), (2, 4096, 4096), (2, 999, 8192),
          (3, 2048, 4096), (4, 4097, 4096), (8, 4096, 4096), (64, 2048, 4096), (100, 9600, 1024), (256, 4096, 4096),
          (3, 500, 1000)]


def _tol(M, N, K):
    return TOL_TC if (M > 4 and M * N * K >= (1 << 27)) else TOL_F32


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("kind", ["norm", "glu", "norm_glu"])
def test_fused_matches_oracle(cuda, shape, kind):
    import torch

    M, N, K = shape
    glu = kind != "norm"
    norm = kind != "glu"
    x, nw, q, s, qu, su = _case(M, N, K, 5 * M + N + K, glu)
    got = _run(torch, cuda, x, nw, q, s, qu, su, norm=norm)
    ref = _ref(x, nw, q, s, qu, su, norm=norm)
    assert oracle.normwise_rel_err(got, ref) <= _tol(M, N, K)


@pytest.mark.parametrize("shape", [(1, 4096, 4096), (2, 2048, 4096), (64, 2048, 4096)])
def test_norm_without_weight_and_unaligned_x(cuda, shape):
    import torch

    M, N, K = shape
    x, _, q, s, qu, su = _case(M, N, K, 3, True)
    for off in (0, 1):
        got = _run(torch, cuda, x, None, q, s, qu, su, x_offset=off)
        ref = _ref(x, None, q, s, qu, su)
        assert oracle.normwise_rel_err(got, ref) <= _tol(M, N, K)


@pytest.mark.skipif(not oracle.have_popcorn_ref_gpu(), reason="popcorn's kernels not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(1, 4096, 4096), (3, 1024, 2048), (16, 512, 1024)])
def test_matches_popcorn_kernel_sequence(cuda, shape):
    import torch

    M, N, K = shape
    x, nw, q, s, qu, su = _case(M, N, K, 11, True)
    lib = oracle.popcorn_ref_gpu()
    xd, nwd = _dev(torch, cuda, x), _dev(torch, cuda, nw)
    qd, sd, qud, sud = (_dev(torch, cuda, a) for a in (q, s, qu, su))
    xn = torch.empty_like(xd)
    g = torch.empty((M, N), dtype=torch.float32, device=cuda)
    u = torch.empty_like(g)
    a = torch.empty_like(g)
    ref = torch.empty_like(g)
    assert lib.popcornRMSNorm_f32(xn.data_ptr(), xd.data_ptr(), nwd.data_ptr(), M, K, EPS, None) == 0
    assert lib.popcornDequantizeMatmul_i8f32(g.data_ptr(), xn.data_ptr(), qd.data_ptr(), sd.data_ptr(), M, N, K,
                                             None) == 0
    assert lib.popcornDequantizeMatmul_i8f32(u.data_ptr(), xn.data_ptr(), qud.data_ptr(), sud.data_ptr(), M, N, K,
                                             None) == 0
    assert lib.popcornSilu_f32(a.data_ptr(), g.data_ptr(), M * N, None) == 0
    assert lib.popcornMul_f32(ref.data_ptr(), a.data_ptr(), u.data_ptr(), M * N, None) == 0
    torch.cuda.synchronize()
    got = _run(torch, cuda, x, nw, q, s, qu, su)
    assert oracle.normwise_rel_err(got, ref.cpu().numpy()) <= _tol(M, N, K)
    # the oracle composition agrees with popcorn's sequence too
    assert oracle.normwise_rel_err(_ref(x, nw, q, s, qu, su), ref.cpu().numpy()) <= 1e-5
