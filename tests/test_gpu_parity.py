"""GPU parity of the sm_100a library, called through its C ABI.

Checks, in the spirit of popcorn's own suite (test/test_quantize.cu):
* the reference suite's fixtures through popcornDequantizeMatmul_i8f32 /
  ...Batched_i8f32 / popcornQuantize_f32i8 against golden vectors made by the
  reference's CPU loops (absolute tolerance 1e-5 as in TOL_PERCHANNEL, :4);
* quantize codes and scales bit-exact against the oracle (rint) and against
  popcorn's own quantize kernels rebuilt for sm_100a, special values included;
* the oracle itself bit-exact against popcorn's own matmul kernel (pin);
* the f32 path within 1e-5 normwise and the tensor path within 2e-3 normwise
  (max|got - ref| / max|ref|) on shapes with tails and unaligned pointers;
* no writes outside the output (guard bytes around every output).
"""
import ctypes

import os

import numpy as np
import pytest

import oracle
import popcorn_b200 as pc

pytestmark = pytest.mark.gpu

TOL_ABS = 1e-5          # popcorn test/test_quantize.cu:4
TOL_F32 = 1e-5          # normwise, f32 CUDA-core path
TOL_TENSOR = 2e-3       # normwise, f16 tensor-core path
GUARD = 4096            # guard elements on each side of an output


def dev(a, torch, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


class Guarded:
    """Device output with canary-filled guard regions on both sides."""

    def __init__(self, torch, cuda, n, dtype, fill):
        self.torch = torch
        self.n = n
        self.buf = torch.full((n + 2 * GUARD,), fill, dtype=dtype, device=cuda)
        self.fill = fill
        self.view = self.buf[GUARD:GUARD + n]

    def ptr(self):
        return self.view.data_ptr()

    def check(self):
        b = self.buf.cpu()
        lo, hi = b[:GUARD], b[GUARD + self.n:]
        if b.dtype.is_floating_point and self.fill != self.fill:
            assert bool(self.torch.isnan(lo).all()) and bool(self.torch.isnan(hi).all()), "guard overwritten"
        else:
            assert bool((lo == self.fill).all()) and bool((hi == self.fill).all()), "guard overwritten"
        return self.view.cpu().numpy()


def abi_matmul(torch, cuda, x, q, s, path=pc.PATH_AUTO, x_offset=0, q_offset=0):
    """Run the dequant-matmul through the C ABI; x/q may sit at odd byte offsets."""
    M, K = x.shape
    N = q.shape[0]
    xs = torch.zeros(M * K + x_offset + 4, dtype=torch.float32, device=cuda)
    xs[x_offset:x_offset + M * K] = dev(x.reshape(-1), torch, cuda)
    qs = torch.zeros(N * K + q_offset + 16, dtype=torch.int8, device=cuda)
    qs[q_offset:q_offset + N * K] = dev(q.reshape(-1), torch, cuda)
    sd = dev(s, torch, cuda)
    out = Guarded(torch, cuda, M * N, torch.float32, float("nan"))
    xp = xs.data_ptr() + 4 * x_offset
    qp = qs.data_ptr() + q_offset
    if path == pc.PATH_AUTO:
        st = pc.popcornDequantizeMatmul_i8f32(out.ptr(), xp, qp, sd.data_ptr(), M, N, K, None)
    else:
        st = pc.popcornDequantizeMatmulPath_i8f32(out.ptr(), xp, qp, sd.data_ptr(), M, N, K, path, None)
    assert st == pc.POPCORN_SUCCESS, pc.load_library().popcornGetLastCudaErrorString()
    torch.cuda.synchronize()
    return out.check().reshape(M, N)


def random_case(M, N, K, seed):
    x = oracle.fill_normal(M * K, seed, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, seed + 1000, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)
    return x, q, s


# ---------------------------------------------------------------------------
# The reference suite's fixtures (golden vectors from its own CPU loops).
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["basic", "identity", "large", "single_row"])
def test_reference_matmul_fixtures(golden, cuda, case):
    import torch

    x, q, s = golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"]
    got = abi_matmul(torch, cuda, x, q, s)
    np.testing.assert_allclose(got, golden[f"{case}/out"], rtol=0, atol=TOL_ABS)


@pytest.mark.parametrize("case", ["batched_basic", "batched_large"])
def test_reference_batched_fixtures(golden, cuda, case):
    import torch

    x, q, s = golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"]
    B, M, K = x.shape
    N = q.shape[0]
    out = Guarded(torch, cuda, B * M * N, torch.float32, float("nan"))
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    st = pc.popcornDequantizeMatmulBatched_i8f32(out.ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                                 B, M, N, K, None)
    assert st == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    got = out.check().reshape(B, M, N)
    np.testing.assert_allclose(got, golden[f"{case}/out"], rtol=0, atol=TOL_ABS)


@pytest.mark.parametrize("case", ["q_basic", "q_large", "q_roundtrip", "q_ties"])
def test_reference_quantize_fixtures(golden, cuda, case):
    import torch

    w = golden[f"{case}/w"]
    N, K = w.shape
    q_out = Guarded(torch, cuda, N * K, torch.int8, 77)
    s_out = Guarded(torch, cuda, N, torch.float32, -3.0)
    wd = dev(w, torch, cuda)
    assert pc.popcornQuantize_f32i8(q_out.ptr(), s_out.ptr(), wd.data_ptr(), N, K, None) == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    q = q_out.check().reshape(N, K)
    s = s_out.check()
    qo, so = oracle.quantize(w)  # rint, popcorn's GPU semantics
    np.testing.assert_array_equal(q, qo)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(s, golden[f"{case}/scale"])
    # Where the test loop's roundf differs, the input is an exact tie.
    ref = golden[f"{case}/codes_test_loop"]
    quot = w / s[:, None]
    assert np.all(np.abs(quot[q != ref] - np.trunc(quot[q != ref])) == 0.5)


def test_config1_host_parity(golden, cuda):
    import torch
    from tests.golden.make_golden import config1_inputs

    x, w = config1_inputs()
    wd = dev(w, torch, cuda)
    q, s = pc.quantize(wd)
    torch.cuda.synchronize()
    qo, so = oracle.quantize(w)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), golden["config1/scale"])
    # The golden output was made from the test loop's roundf codes; feed the
    # same codes (they differ from rintf only on exact .5 quotients).
    q_ref, s_ref = oracle.quantize(w, ties_away=True)
    got = abi_matmul(torch, cuda, x, q_ref, s_ref)
    ref = golden["config1/out"]
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32
    np.testing.assert_allclose(got, ref, rtol=0, atol=5e-5)


# ---------------------------------------------------------------------------
# popcorn's own kernels rebuilt for sm_100a.
# ---------------------------------------------------------------------------
needs_ref_gpu = pytest.mark.skipif(not oracle.have_popcorn_ref_gpu(), reason="oracle/_ref not built")


def special_rows(K):
    rng = np.random.default_rng(3)
    rows = [
        rng.standard_normal(K).astype(np.float32),
        np.zeros(K, np.float32),
        np.full(K, -0.0, np.float32),
        np.full(K, 1e-42, np.float32),                       # denormals
        (rng.standard_normal(K) * 1e30).astype(np.float32),
        np.where(np.arange(K) % 5 == 0, np.nan, 1.0).astype(np.float32),
        np.full(K, np.nan, np.float32),
        np.where(np.arange(K) == 3, np.inf, 2.0).astype(np.float32),
        np.where(np.arange(K) == 1, -np.inf, np.arange(K, dtype=np.float32)).astype(np.float32),
        (np.arange(K, dtype=np.float32) - K / 2) * np.float32(0.5),  # many .5 ties
        np.full(K, 3.4e38, np.float32),
    ]
    return np.stack(rows)


@needs_ref_gpu
@pytest.mark.parametrize("K", [1, 4, 37, 256, 4096, 4100])
def test_quantize_bitexact_vs_popcorn_kernel(cuda, K):
    import torch

    w = special_rows(K)
    w = np.concatenate([w, oracle.fill_normal(40 * K, K, 0.02).reshape(40, K)])
    N = w.shape[0]
    wd = dev(w, torch, cuda)
    q1, s1 = pc.quantize(wd)
    q2 = torch.empty_like(q1)
    s2 = torch.empty_like(s1)
    ref = oracle.popcorn_ref_gpu()
    assert ref.popcornQuantize_f32i8(q2.data_ptr(), s2.data_ptr(), wd.data_ptr(), N, K, None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q1.cpu().numpy(), q2.cpu().numpy())
    np.testing.assert_array_equal(s1.cpu().numpy().view(np.uint32), s2.cpu().numpy().view(np.uint32))
    qo, so = oracle.quantize(w)
    np.testing.assert_array_equal(q1.cpu().numpy(), qo)
    np.testing.assert_array_equal(s1.cpu().numpy().view(np.uint32), so.view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(5, 1000, 4096), (6, 4096, 4096), (7, 513, 2048), (8, 300, 4000)])
def test_f32_path_five_to_eight_rows(cuda, M, N, K):
    # Five to eight activation rows on the CUDA-core path: two row groups of
    # the x-stationary kernel (K <= 4096), or the generic kernel (K % 16 != 0).
    import torch

    x, q, s = random_case(M, N, K, 3 * M + N + K)
    got = abi_matmul(torch, cuda, x, q, s, path=pc.PATH_SIMT_F32)
    err = oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s))
    assert err <= TOL_F32, err


def near_tie_rows(K, rows=8):
    """Rows whose values sit on and within a few ulps of every half-integer
    multiple of the row's scale (the boundaries where rint(v / scale) changes),
    with the row maximum pinned so that scale = max / 127 is known."""
    out = []
    for r in range(rows):
        mx = np.float32(0.37 * (r + 1))
        sc = np.float32(mx / np.float32(127.0))
        vals = []
        for j in range(-128, 127):
            v = np.float32(np.float32(j + 0.5) * sc)
            for d in range(-3, 4):
                vals.append(v)
                v = np.nextafter(v, np.float32(np.inf) if d >= 0 else np.float32(-np.inf))
        row = np.resize(np.array(vals, np.float32), K)
        row = np.clip(row, -mx, mx)
        row[0] = mx
        out.append(row.astype(np.float32))
    return np.stack(out)


@needs_ref_gpu
@pytest.mark.parametrize("K", [1000, 4096, 8192, 12288, 20000])
def test_quantize_near_ties_bitexact(cuda, K):
    # The quantizer multiplies by the reciprocal scale and falls back to the
    # division near rounding boundaries; codes must still equal popcorn's
    # rint(v / scale) bit for bit (row-block kernels for K <= 16384, the
    # per-warp kernel beyond and for K % 16 != 0).
    import torch

    w = near_tie_rows(K)
    N = w.shape[0]
    wd = dev(w, torch, cuda)
    q1, s1 = pc.quantize(wd)
    q2 = torch.empty_like(q1)
    s2 = torch.empty_like(s1)
    ref = oracle.popcorn_ref_gpu()
    assert ref.popcornQuantize_f32i8(q2.data_ptr(), s2.data_ptr(), wd.data_ptr(), N, K, None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q1.cpu().numpy(), q2.cpu().numpy())
    np.testing.assert_array_equal(s1.cpu().numpy().view(np.uint32), s2.cpu().numpy().view(np.uint32))
    qo, so = oracle.quantize(w)
    np.testing.assert_array_equal(q1.cpu().numpy(), qo)


@needs_ref_gpu
@pytest.mark.parametrize("shape", [(1, 64, 64), (3, 40, 96), (16, 256, 1024), (33, 100, 512)])
def test_oracle_pinned_to_popcorn_matmul_kernel(cuda, shape):
    # popcorn's kernel accumulates sequentially in k with a fused multiply-add;
    # the oracle's fused variant must reproduce it bit for bit (K % 32 == 0, the
    # shapes where popcorn's kernel has no tail bug, src/quantize.cu:57-58).
    import torch

    M, N, K = shape
    x, q, s = random_case(M, N, K, 21)
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    out = torch.empty((M, N), dtype=torch.float32, device=cuda)
    ref = oracle.popcorn_ref_gpu()
    assert ref.popcornDequantizeMatmul_i8f32(out.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                             M, N, K, None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.dequant_matmul(x, q, s, fused=True))


@needs_ref_gpu
@pytest.mark.parametrize("shape", [(1, 4096, 4096), (4, 1024, 4096), (32, 512, 2048)])
def test_matmul_vs_popcorn_kernel(cuda, shape):
    import torch

    M, N, K = shape
    x, q, s = random_case(M, N, K, 31)
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    ref_out = torch.empty((M, N), dtype=torch.float32, device=cuda)
    assert oracle.popcorn_ref_gpu().popcornDequantizeMatmul_i8f32(
        ref_out.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), M, N, K, None) == 0
    got = pc.dequantize_matmul(xd, qd, sd)
    torch.cuda.synchronize()
    path = pc.select_path(xd.data_ptr(), qd.data_ptr(), M, N, K)
    tol = TOL_TENSOR if path == pc.PATH_TENSOR_F16 else TOL_F32
    assert oracle.normwise_rel_err(got.cpu().numpy(), ref_out.cpu().numpy()) <= tol


# ---------------------------------------------------------------------------
# Shapes with tails, odd K, unaligned pointers, every path.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 7, 33])
@pytest.mark.parametrize("N,K", [(1, 16), (7, 48), (129, 512), (64, 1000), (17, 4112), (300, 8192)])
def test_simt_path_shapes(cuda, M, N, K):
    import torch

    x, q, s = random_case(M, N, K, M * 7 + N)
    got = abi_matmul(torch, cuda, x, q, s, path=pc.PATH_SIMT_F32)
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32


@pytest.mark.parametrize("x_off,q_off", [(1, 0), (0, 3), (2, 5)])
def test_unaligned_pointers(cuda, x_off, q_off):
    import torch

    M, N, K = 5, 70, 256
    x, q, s = random_case(M, N, K, 41)
    got = abi_matmul(torch, cuda, x, q, s, x_offset=x_off, q_offset=q_off)
    assert oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s)) <= TOL_F32


def test_tensor_path_rejects_what_it_cannot_run(cuda):
    import torch

    x, q, s = random_case(8, 64, 40, 5)  # K % 16 != 0
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    out = torch.empty((8, 64), dtype=torch.float32, device=cuda)
    st = pc.popcornDequantizeMatmulPath_i8f32(out.data_ptr(), xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                              8, 64, 40, pc.PATH_TENSOR_F16, None)
    assert st == pc.POPCORN_ERROR_INVALID_VALUE


@pytest.mark.parametrize("N,K", [(1, 1), (3, 5), (64, 4096), (130, 4112), (7, 100), (5, 48), (2000, 1040),
                                 (3, 8192)])
def test_dequantize_bitexact(cuda, N, K):
    import torch

    w = oracle.fill_normal(N * K, N + K, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)
    out = Guarded(torch, cuda, N * K, torch.float32, float("nan"))
    qd, sd = dev(q, torch, cuda), dev(s, torch, cuda)
    assert pc.popcornDequantize_i8f32(out.ptr(), qd.data_ptr(), sd.data_ptr(), N, K, None) == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    got = out.check().reshape(N, K)
    np.testing.assert_array_equal(got.view(np.uint32), oracle.dequantize(q, s).view(np.uint32))


@pytest.mark.parametrize("N,K", [(1, 1), (3, 5), (64, 4096), (130, 4112), (7, 100), (4096, 4096), (5, 48),
                                 (2000, 1040), (3, 8192)])
def test_dequantize_bf16_bitexact(cuda, N, K):
    # bf16 output: the f32 product rounded once to nearest even, bit for bit;
    # scales spanning many binades (ties and bf16 subnormals included).
    import torch

    w = oracle.fill_normal(N * K, N + 2 * K, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)
    s = (s * np.exp2(np.arange(N) % 200 - 100).astype(np.float32)).astype(np.float32)
    s[0] = 0.0
    out = Guarded(torch, cuda, N * K, torch.int16, -12345)
    qd, sd = dev(q, torch, cuda), dev(s, torch, cuda)
    assert pc.popcornDequantize_i8bf16(out.ptr(), qd.data_ptr(), sd.data_ptr(), N, K, None) == pc.POPCORN_SUCCESS
    torch.cuda.synchronize()
    got = out.check().reshape(N, K).view(np.uint16)
    np.testing.assert_array_equal(got, oracle.dequantize_bf16(q, s))
    y = pc.dequantize(qd, sd, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy().view(np.uint16), oracle.dequantize_bf16(q, s))


def test_runs_on_caller_stream(cuda):
    import torch

    x, q, s = random_case(2, 512, 1024, 9)
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        out = pc.dequantize_matmul(xd, qd, sd, stream=st)
    st.synchronize()
    assert oracle.normwise_rel_err(out.cpu().numpy(), oracle.dequant_matmul(x, q, s)) <= TOL_F32


def test_quantize_full_size_roundtrip_property(cuda):
    # 4096 x 4096 ~ N(0, 0.02): codes from the GPU equal the oracle's, and the
    # dequantized weights are within half a step of the input.
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(0)
    w = torch.randn((4096, 4096), generator=g, device=cuda) * 0.02
    q, s = pc.quantize(w)
    d = pc.dequantize(q, s)
    torch.cuda.synchronize()
    # |w/s - q| <= 1/2, plus the f32 roundings of w/s and q*s (|q| <= 127).
    assert bool(((d - w).abs() <= (0.5 + 2.0 ** -15) * s[:, None]).all())
    assert int(q.abs().max()) == 127
    qo, so = oracle.quantize(w.cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy(), so)


def test_error_record_is_per_thread(lib):
    import threading

    # A fresh thread starts with no recorded CUDA error.
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.popcornGetLastCudaError()))
    t.start()
    t.join()
    assert seen == [0]
    assert isinstance(ctypes.c_int(lib.popcornGetLastCudaError()).value, int)


# ---------------------------------------------------------------------------
# tcgen05 tensor-core path.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("M", [1, 5, 16, 32, 33, 64, 65, 100, 128, 129, 256, 300])
@pytest.mark.parametrize("N,K", [(128, 64), (100, 16), (300, 80), (256, 1024), (129, 4096)])
def test_tensor_path_shapes(cuda, M, N, K):
    import torch

    x, q, s = random_case(M, N, K, 100 + M + N + K)
    got = abi_matmul(torch, cuda, x, q, s, path=pc.PATH_TENSOR_F16)
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    err = oracle.normwise_rel_err(got, ref)
    assert err <= TOL_TENSOR, err
    # int8 digit activations (M <= 128) ~4e-5, f16 activations (M > 128)
    # ~1e-4: both far inside the tolerance.
    assert err <= 5e-4, err


@pytest.mark.parametrize("M,N,K", [(5, 9600, 512), (16, 9601, 256), (33, 9500, 1024), (64, 9728, 2048),
                                   (100, 10000, 1024), (128, 12288, 4096), (130, 9600, 512)])
def test_tensor_path_pairs_for_many_weight_tiles(cuda, M, N, K):
    # More 128-row weight tiles than half the SMs: one CTA per tile on the
    # int8 path (M <= 128), CTA pairs (cta_group::2) above; odd M and N tails.
    import torch

    x, q, s = random_case(M, N, K, 7 + M + N + K)
    got = abi_matmul(torch, cuda, x, q, s, path=pc.PATH_TENSOR_F16)
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    err = oracle.normwise_rel_err(got, ref)
    assert err <= 5e-4, err


# ---------------------------------------------------------------------------
# The int8 tensor path (per-channel weights, 4 < M <= 128): activations as two
# signed 8-bit digits of a 16-bit fixed-point row, tcgen05.mma.kind::i8 on the
# raw weight codes, split-K partials summed through L2 when tiles are few.
# ---------------------------------------------------------------------------
TOL_I8 = 2e-4  # normwise; the 16-bit rows give ~4e-5


@pytest.mark.parametrize("M,N,K", [
    (5, 4096, 4096),      # 32 tiles: cluster split-K, BM = 32
    (32, 4096, 4096),
    (64, 4096, 11008),    # split-K with ragged k-block shares, K tail
    (128, 4096, 4096),    # BM = 128
    (100, 2000, 8192),    # 16 tiles: 8-way split, N tail
    (17, 11008, 4096),    # 86 tiles, no split
    (128, 12288, 4096),
    (65, 300, 16),        # a single, mostly zero-filled k-block
])
def test_int8_tensor_path_shapes(cuda, M, N, K):
    import torch

    x, q, s = random_case(M, N, K, 11 * M + N + K)
    got = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_I8


@pytest.mark.parametrize("M,K,x_off", [(48, 20480, 0), (33, 4096, 1), (9, 2064, 3)])
def test_int8_tensor_path_prologue_forms(cuda, M, K, x_off):
    # K beyond the row-in-registers prologue and unaligned activations: the
    # warp-per-row digit prologue.
    import torch

    N = 1024
    x, q, s = random_case(M, N, K, 5 + M + K)
    got = abi_matmul(torch, cuda, x, q, s, x_offset=x_off)
    assert pc.device_errors() == 0
    assert oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s, fused=True, threads=8)) <= TOL_I8


def test_int8_tensor_path_special_rows(cuda):
    # Magnitudes from 1e-33 (pre-scaled by 2^100) to 1e35, an all-zero row, a
    # NaN row, rows with one or two infinities of the same sign.
    import torch

    M, N, K = 12, 4096, 4096
    x, q, s = random_case(M, N, K, 91)
    x = x.copy()
    x[0] *= 1e-33
    x[1] *= 1e35
    x[2] = 0.0
    x[3, 5] = np.nan
    x[4, 7] = np.inf
    x[5, 9] = -np.inf
    x[6, 11] = np.inf
    x[6, 4000] = np.inf
    x[7] *= 2.0 ** -100
    got = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    for m in (0, 1, 7, 8, 9, 10, 11):
        assert oracle.normwise_rel_err(got[m], ref[m]) <= TOL_I8, m
    assert np.all(got[2] == 0.0)
    assert np.all(np.isnan(got[3]))
    for m in (4, 5):
        # one infinity: +-inf with popcorn's sign, NaN exactly where popcorn's
        # sum is NaN (the code at the infinite entry is 0)
        assert np.array_equal(np.isnan(got[m]), np.isnan(ref[m])), m
        inf = np.isinf(ref[m])
        assert np.array_equal(got[m][inf], ref[m][inf]), m
    # two infinities: every output non-finite, as popcorn's (which is NaN
    # wherever the two terms' signs differ)
    assert np.all(~np.isfinite(got[6])) and np.all(~np.isfinite(ref[6]))


def test_int8_tensor_path_is_deterministic(cuda):
    # Split-K partials are summed in rank order: repeated calls agree bitwise.
    import torch

    x, q, s = random_case(96, 4096, 11008, 17)
    a = abi_matmul(torch, cuda, x, q, s)
    b = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_f32_path_fixed_point_edges(cuda):
    # The M = 1 decode kernel computes in fixed point per thread slice; warps
    # whose slice holds a non-finite or extreme |x| take the float path.
    # Check both, and rows mixing them, against the oracle.
    import torch

    N, K = 2048, 4096  # above the sequential kernel's 2^22 multiply-adds
    x, q, s = random_case(1, N, K, 31)
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    for scale in (1.0, 2.0 ** -80, 2.0 ** -95, 2.0 ** 95, 2.0 ** 105):
        got = abi_matmul(torch, cuda, (x * scale).astype(np.float32), q, s)
        want = oracle.dequant_matmul((x * scale).astype(np.float32), q, s, fused=True, threads=8)
        assert oracle.normwise_rel_err(got, want) <= TOL_F32, scale
    # one slice far below the others (its warp falls back), zero slices
    xm = x.copy()
    xm[0, :64] *= 2.0 ** -120
    xm[0, 2048:2560] = 0.0
    got = abi_matmul(torch, cuda, xm, q, s)
    assert oracle.normwise_rel_err(got, oracle.dequant_matmul(xm, q, s, fused=True, threads=8)) <= TOL_F32
    # a single inf: every output is +-inf (or NaN where the code is 0)
    xi = x.copy()
    xi[0, 100] = np.inf
    got = abi_matmul(torch, cuda, xi, q, s)
    want = oracle.dequant_matmul(xi, q, s, fused=True, threads=8)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])
    # a NaN poisons every output
    xn = x.copy()
    xn[0, 4000] = np.nan
    assert np.all(np.isnan(abi_matmul(torch, cuda, xn, q, s)))
    assert pc.device_errors() == 0
    assert oracle.normwise_rel_err(abi_matmul(torch, cuda, x, q, s), ref) <= TOL_F32


def test_tensor_path_row_scaling_handles_extreme_rows(cuda):
    # Rows of wildly different magnitude, an all-zero row, a NaN row and an
    # infinite entry: every finite row keeps f16 relative precision.
    import torch

    M, N, K = 8, 256, 512
    x, q, s = random_case(M, N, K, 77)
    x = x.copy()
    x[0] *= 1e-30
    x[1] *= 1e30
    x[2] = 0.0
    x[3, 5] = np.nan
    x[4, 7] = np.inf
    x[5] *= 3e-42 / np.abs(x[5]).max()  # denormal row
    got = abi_matmul(torch, cuda, x, q, s, path=pc.PATH_TENSOR_F16)
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True)
    for m in (0, 1, 6, 7):
        assert oracle.normwise_rel_err(got[m], ref[m]) <= 5e-4, m
    assert np.all(got[2] == 0.0)
    assert np.all(np.isnan(got[3]))
    assert np.all(~np.isfinite(got[4]))


def test_tensor_path_prefill_full_size(cuda):
    # M=2048, K=4096, N=4096 against a float64 torch reference on the GPU.
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(7)
    x = torch.randn((2048, 4096), generator=g, device=cuda)
    w = torch.randn((4096, 4096), generator=g, device=cuda) * 0.02
    q, s = pc.quantize(w)
    y = pc.dequantize_matmul(x, q, s)
    assert pc.select_path(x.data_ptr(), q.data_ptr(), 2048, 4096, 4096) == pc.PATH_TENSOR_F16
    ref = x.double() @ (q.double() * s.double()[:, None]).T
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err <= TOL_TENSOR, err


@pytest.mark.parametrize("fmt", ["channel", "group8", "int4"])
def test_tensor_path_ragged_prefill_all_formats(cuda, fmt):
    # M=2000, N=4096: persistent CTA pairs over 128 tiles whose last tile row
    # holds 208 of 256 activation rows, every weight format, against a
    # float64 product of the dequantized weights.
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(21)
    M, N, K, gs = 2000, 4096, 1024, 128
    x = torch.randn((M, K), generator=g, device=cuda)
    w = torch.randn((N, K), generator=g, device=cuda) * 0.02
    if fmt == "channel":
        q, s = pc.quantize(w)
        y = pc.dequantize_matmul(x, q, s)
        wd = q.double() * s.double()[:, None]
    elif fmt == "group8":
        q, s = pc.quantize_grouped(w, gs)
        y = pc.dequantize_matmul_grouped(x, q, s, gs)
        wd = q.double() * s.double().repeat_interleave(gs, dim=1)
    else:
        q, s, z = pc.quantize_grouped_i4(w, gs)
        y = pc.dequantize_matmul_grouped_i4(x, q, s, z, gs)
        codes = torch.stack(((q & 15), (q >> 4)), dim=-1).reshape(N, K).double()
        wd = (codes - z.double().repeat_interleave(gs, dim=1)) * s.double().repeat_interleave(gs, dim=1)
    ref = x.double() @ wd.T
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err <= TOL_TENSOR, err


def test_tensor_path_skinny_full_size(cuda):
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(8)
    x = torch.randn((32, 4096), generator=g, device=cuda)
    w = torch.randn((11008, 4096), generator=g, device=cuda) * 0.02
    q, s = pc.quantize(w)
    y = pc.dequantize_matmul(x, q, s)
    ref = x.double() @ (q.double() * s.double()[:, None]).T
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err <= TOL_TENSOR, err


@pytest.mark.parametrize("N,K", [
    (1000, 288),    # 9 k-steps: warps 9..15 own none
    (5000, 544),    # 34 rows per CTA, 17 k-steps
    (4096, 1376),   # down projection slice of an 8-way split
    (4096, 2752),   # ... of a 4-way split
    (3000, 5120),   # 10 or 11 k-steps per warp
    (2000, 8192),   # the largest staged K, 14 rows per CTA
    (8192, 2048),   # 56 rows per CTA in four row groups
    (8000, 2080),   # 65 k-steps (uneven warps), 55 rows per CTA
    (3000, 1536),   # 3 k-steps per warp
])
def test_staged_decode_any_k_and_row_split(cuda, N, K):
    # The staged M = 1 kernel (K % 32 == 0, rows within shared memory): the
    # oracle's result within the f32 tolerance, and each row's bits
    # independent of how many rows share a CTA (a sub-range of rows as its
    # own call returns the same values).
    import torch

    x, q, s = random_case(1, N, K, 91 + K)
    got = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    assert oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s, fused=True, threads=8)) <= TOL_F32
    lo, n2 = 37, 151
    sub = abi_matmul(torch, cuda, x, np.ascontiguousarray(q[lo:lo + n2]), np.ascontiguousarray(s[lo:lo + n2]))
    assert np.array_equal(sub.view(np.uint32), got[:, lo:lo + n2].view(np.uint32))


def test_decode_full_size_vs_oracle(cuda):
    import torch

    x, q, s = random_case(1, 4096, 4096, 55)
    got = abi_matmul(torch, cuda, x, q, s)
    assert oracle.normwise_rel_err(got, oracle.dequant_matmul(x, q, s, fused=True, threads=8)) <= TOL_F32


@needs_ref_gpu
@pytest.mark.parametrize("M,N,K", [
    (32, 11008, 4096),    # skinny decode batch (MLP up-projection)
    (128, 12288, 4096),   # stack qkv at 128 rows: CTA pairs
    (2048, 4096, 4096),   # prefill: persistent CTA pairs, f16 activations
])
def test_workload_sizes_vs_oracle_and_popcorn_kernel(cuda, M, N, K):
    # The matmul workloads at their full sizes on the seeded generator's data
    # (X ~ N(0,1), W ~ N(0,0.02), per-row int8): the library against the
    # oracle (popcorn's loop order, fused multiply-add, all host threads) and
    # against popcorn's own kernel rebuilt for sm_100a, same inputs.
    import torch

    x, q, s = random_case(M, N, K, 77 + M)
    got = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    threads = max(1, min(32, os.cpu_count() or 1))
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=threads)
    err = oracle.normwise_rel_err(got, ref)
    assert err <= 5e-4, err
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    theirs = torch.empty((M, N), dtype=torch.float32, device=cuda)
    assert oracle.popcorn_ref_gpu().popcornDequantizeMatmul_i8f32(theirs.data_ptr(), xd.data_ptr(), qd.data_ptr(),
                                                                  sd.data_ptr(), M, N, K, None) == 0
    torch.cuda.synchronize()
    theirs = theirs.cpu().numpy()
    assert np.array_equal(theirs, ref), "popcorn's kernel and the oracle disagree"
    assert oracle.normwise_rel_err(got, theirs) <= 5e-4


def test_tensor_path_back_to_back_calls_reuse_scratch(cuda):
    # Stream-ordered scratch: many calls in flight on one stream stay correct.
    import torch

    M, N, K = 256, 512, 1024
    x, q, s = random_case(M, N, K, 3)
    xd, qd, sd = dev(x, torch, cuda), dev(q, torch, cuda), dev(s, torch, cuda)
    outs = [pc.dequantize_matmul(xd * (i + 1), qd, sd, path=pc.PATH_TENSOR_F16) for i in range(8)]
    torch.cuda.synchronize()
    assert pc.device_errors() == 0
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    for i, o in enumerate(outs):
        assert oracle.normwise_rel_err(o.cpu().numpy() / (i + 1), ref) <= 5e-4


@pytest.mark.parametrize("M,N,K", [
    (1, 4096, 4096), (1, 1100, 4096), (1, 1000, 8192), (1, 777, 16384), (1, 1031, 11008),
    (1, 5000, 1024), (2, 4096, 4096), (2, 999, 8192), (3, 2000, 4096), (4, 4097, 4096), (4, 300, 4096),
    # M = 1 shapes of the bulk-copy decode kernel: more rows than one CTA per
    # SM can own (extra CTAs), fewer rows than SMs, every rows-per-stage and
    # slices-per-thread variant, K with partial 4 KB slices.
    (1, 40000, 1024), (1, 300, 16384), (1, 2100, 2048), (1, 9000, 512), (1, 4000, 1376), (1, 1000, 5504),
    (1, 400, 12288), (1, 2000, 16384), (1, 3, 1 << 21),
])
def test_bulk_gemv_variants(cuda, M, N, K):
    # Every template variant of the decode GEMVs (f32 path, M <= 4).
    import torch

    assert M * N * K > (1 << 22)
    x, q, s = random_case(M, N, K, 7 * M + N)
    got = abi_matmul(torch, cuda, x, q, s)
    assert pc.device_errors() == 0
    if K > 65536:
        # A sequential f32 sum over millions of terms carries its own rounding
        # error well above 1e-5; compare such rows with a float64 product.
        ref = x.astype(np.float64) @ (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    else:
        ref = oracle.dequant_matmul(x, q, s, fused=True, threads=8)
    assert oracle.normwise_rel_err(got, ref) <= TOL_F32
