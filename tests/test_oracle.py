"""CPU: the oracle restatement against the golden vectors and the reference loops.

The golden vectors were made by popcorn's own test-side CPU loops
(test/test_quantize.cu:24-41, :677-706) on the reference suite's own inputs
(tests/golden/make_golden.py). The restatement must reproduce them bit for
bit; the rintf/roundf difference is confined to exact .5 quotients.
"""
import hashlib

import numpy as np
import pytest

import oracle

MATMUL_CASES = ["basic", "identity", "large", "single_row"]
QUANT_CASES = ["q_basic", "q_large", "q_roundtrip", "q_ties"]


@pytest.mark.parametrize("case", MATMUL_CASES)
def test_matmul_matches_reference_loop_bitwise(golden, case):
    out = oracle.dequant_matmul(golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"])
    np.testing.assert_array_equal(out, golden[f"{case}/out"])


def test_identity_literal(golden):
    out = oracle.dequant_matmul(golden["identity/x"], golden["identity/q"], golden["identity/scale"])
    np.testing.assert_array_equal(out, golden["identity/expected_literal"])


@pytest.mark.parametrize("case", ["batched_basic", "batched_large"])
def test_batched_matches_reference_loop_bitwise(golden, case):
    x, q, s = golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"]
    B, M, K = x.shape
    # Batched == one matmul over B*M rows (x, out contiguous).
    out = oracle.dequant_matmul(x.reshape(B * M, K), q, s).reshape(B, M, -1)
    np.testing.assert_array_equal(out, golden[f"{case}/out"])


@pytest.mark.parametrize("case", QUANT_CASES)
def test_quantize_roundf_matches_reference_loop(golden, case):
    q, s = oracle.quantize(golden[f"{case}/w"], ties_away=True)
    np.testing.assert_array_equal(q, golden[f"{case}/codes_test_loop"])
    np.testing.assert_array_equal(s, golden[f"{case}/scale"])


@pytest.mark.parametrize("case", QUANT_CASES)
def test_quantize_rint_differs_only_on_ties(golden, case):
    w = golden[f"{case}/w"]
    q, s = oracle.quantize(w)
    np.testing.assert_array_equal(s, golden[f"{case}/scale"])
    ref = golden[f"{case}/codes_test_loop"]
    quot = w / s[:, None]
    tie = np.abs(quot - np.trunc(quot)) == 0.5
    assert np.array_equal(q[~tie], ref[~tie])
    # Every disagreement is a tie, and rint is half-to-even there.
    assert np.all(q[q != ref].astype(np.int64) % 2 == 0)


def test_quantize_ties_half_to_even(golden):
    q, _ = oracle.quantize(golden["q_ties/w"])
    assert q.tolist() == [[127, 0, 2, 2, 0, -2, -2, 126]]


def test_roundtrip_bound(golden):
    # popcorn test/test_quantize.cu:996-1016: |dequant - orig| <= 0.6 * scale.
    w = golden["q_roundtrip/w"]
    q, s = oracle.quantize(w)
    d = oracle.dequantize(q, s)
    assert np.all(np.abs(d - w) <= 0.6 * s[:, None])
    assert s[3] == 1.0  # all-zero row


def test_config1_generator_and_outputs(golden):
    from tests.golden.make_golden import CONFIG1, config1_inputs

    x, w = config1_inputs()
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(golden["config1/x_sha256"])
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(golden["config1/w_sha256"])
    q, s = oracle.quantize(w, ties_away=True)
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(golden["config1/codes_test_loop_sha256"])
    np.testing.assert_array_equal(s, golden["config1/scale"])
    out = oracle.dequant_matmul(x, q, s)
    np.testing.assert_array_equal(out, golden["config1/out"])
    assert list(golden["config1/shape"]) == [CONFIG1["M"], CONFIG1["K"], CONFIG1["N"]]
    # Generator statistics: mean ~0, std ~sigma, |x| < 6 sigma by construction.
    assert abs(float(x.mean())) < 0.05 and abs(float(x.std()) - 1.0) < 0.05
    assert abs(float(w.std()) - 0.02) < 0.001 and float(np.abs(w).max()) < 0.12


def test_threaded_oracle_bitwise():
    x = oracle.fill_normal(3 * 200, 5, 1.0).reshape(3, 200)
    w = oracle.fill_normal(37 * 200, 6, 0.02).reshape(37, 200)
    q, s = oracle.quantize(w)
    for fused in (False, True):
        a = oracle.dequant_matmul(x, q, s, fused=fused)
        b = oracle.dequant_matmul(x, q, s, fused=fused, threads=5)
        np.testing.assert_array_equal(a, b)


def test_fused_and_unfused_agree_to_f32_rounding():
    x = oracle.fill_normal(4 * 4096, 7, 1.0).reshape(4, 4096)
    w = oracle.fill_normal(64 * 4096, 8, 0.02).reshape(64, 4096)
    q, s = oracle.quantize(w)
    a = oracle.dequant_matmul(x, q, s, fused=False)
    b = oracle.dequant_matmul(x, q, s, fused=True)
    assert oracle.normwise_rel_err(b, a) < 1e-5


def test_normwise_metric_detects_a_planted_error():
    ref = np.array([[1.0, -2.0, 4.0]], dtype=np.float32)
    bad = ref.copy()
    bad[0, 1] += 0.01
    assert oracle.normwise_rel_err(ref, ref) == 0.0
    assert abs(oracle.normwise_rel_err(bad, ref) - 0.0025) < 1e-7


@pytest.mark.skipif(not oracle.have_ref_loops(), reason="reference loops not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 7, 33), (5, 64, 1000), (16, 129, 512)])
def test_oracle_equals_reference_loops_random(shape):
    M, N, K = shape
    x = oracle.fill_normal(M * K, 11 + M, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, 12 + N, 0.02).reshape(N, K)
    qr, sr = oracle.ref_quantize(w)
    qo, so = oracle.quantize(w, ties_away=True)
    np.testing.assert_array_equal(qr, qo)
    np.testing.assert_array_equal(sr, so)
    np.testing.assert_array_equal(oracle.ref_dequant_matmul(x, qr, sr), oracle.dequant_matmul(x, qr, sr))
    np.testing.assert_array_equal(oracle.ref_dequant_matmul(x, qr, sr, threads=3), oracle.dequant_matmul(x, qr, sr))


@pytest.mark.skipif(not oracle.have_ref_loops(), reason="reference loops not built (oracle/_ref)")
def test_planted_oracle_mistake_is_caught():
    # A wrong restatement (scale applied twice) must not pass the pin.
    x = oracle.fill_normal(2 * 64, 1, 1.0).reshape(2, 64)
    w = oracle.fill_normal(8 * 64, 2, 0.02).reshape(8, 64)
    q, s = oracle.ref_quantize(w)
    wrong = oracle.dequant_matmul(x, q, s * s)
    assert not np.array_equal(wrong, oracle.ref_dequant_matmul(x, q, s))


# ---------------------------------------------------------------------------
# Per-group int8 (popcorn src/quantize.cu:114-218, :571-640; its CPU loops
# test/test_quantize.cu:42-61, :709-742).
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["g_basic", "g_large"])
def test_grouped_matmul_matches_reference_loop_bitwise(golden, case):
    gs = int(golden[f"{case}/group_size"])
    out = oracle.dequant_matmul_grouped(golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"], gs)
    np.testing.assert_array_equal(out, golden[f"{case}/out"])
    out3 = oracle.dequant_matmul_grouped(golden[f"{case}/x"], golden[f"{case}/q"], golden[f"{case}/scale"], gs,
                                         threads=3)
    np.testing.assert_array_equal(out3, golden[f"{case}/out"])


def test_grouped_quantize_roundf_matches_reference_loop(golden):
    q, s = oracle.quantize_grouped(golden["qg_basic/w"], int(golden["qg_basic/group_size"]), ties_away=True)
    np.testing.assert_array_equal(q, golden["qg_basic/codes_test_loop"])
    np.testing.assert_array_equal(s, golden["qg_basic/scale"])


def test_grouped_with_one_group_is_the_per_channel_path():
    x = oracle.fill_normal(3 * 64, 5, 1.0).reshape(3, 64)
    w = oracle.fill_normal(9 * 64, 6, 0.02).reshape(9, 64)
    q, s = oracle.quantize(w)
    qg, sg = oracle.quantize_grouped(w, 64)
    np.testing.assert_array_equal(q, qg)
    np.testing.assert_array_equal(s, sg[:, 0])
    np.testing.assert_array_equal(oracle.dequant_matmul(x, q, s), oracle.dequant_matmul_grouped(x, qg, sg, 64))


@pytest.mark.skipif(not oracle.have_ref_loops(), reason="reference loops not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(1, 7, 8, 4), (3, 17, 64, 16), (5, 33, 96, 32), (4, 40, 256, 128), (2, 9, 48, 48)])
def test_grouped_oracle_equals_reference_loops_random(shape):
    M, N, K, gs = shape
    x = oracle.fill_normal(M * K, M + N, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, K, 0.02).reshape(N, K)
    qr, sr = oracle.ref_quantize_grouped(w, gs)
    qo, so = oracle.quantize_grouped(w, gs, ties_away=True)
    np.testing.assert_array_equal(qr, qo)
    np.testing.assert_array_equal(sr, so)
    np.testing.assert_array_equal(oracle.ref_dequant_matmul_grouped(x, qr, sr, gs),
                                  oracle.dequant_matmul_grouped(x, qr, sr, gs, threads=2))


# ---------------------------------------------------------------------------
# Int4 packed asymmetric per-group (popcorn src/quantize.cu:329-446, :699-888;
# its CPU loops test/test_quantize.cu:67-99, :746-789).
# ---------------------------------------------------------------------------
def _unpack_i4(q):
    """[N, K/2] bytes -> [N, K] codes, low nibble first (numpy, independent of the oracle)."""
    q = np.asarray(q, dtype=np.uint8)
    codes = np.empty((q.shape[0], 2 * q.shape[1]), dtype=np.int64)
    codes[:, 0::2] = q & 0x0F
    codes[:, 1::2] = q >> 4
    return codes


@pytest.mark.parametrize("case", ["i4_basic", "i4_large"])
def test_int4_matmul_matches_reference_loop_bitwise(golden, case):
    x, q = golden[f"{case}/x"], golden[f"{case}/q"]
    s, z = golden[f"{case}/scale"], golden[f"{case}/zero"]
    gs = int(golden[f"{case}/group_size"])
    for threads in (1, 3):
        out = oracle.dequant_matmul_grouped_i4(x, q, s, z, gs, threads=threads)
        np.testing.assert_array_equal(out, golden[f"{case}/out"])
    # The same product from the unpacked codes in float64.
    codes = _unpack_i4(q)
    g = np.arange(codes.shape[1]) // gs
    w = (codes - z[:, g].astype(np.float64)) * s[:, g].astype(np.float64)
    ref = x.astype(np.float64) @ w.T
    assert oracle.normwise_rel_err(golden[f"{case}/out"], ref) <= 1e-6


def test_int4_basic_layout_is_low_nibble_first(golden):
    # The test's comment spells out the codes of row 0 (1..8) and row 1 (0..7).
    np.testing.assert_array_equal(_unpack_i4(golden["i4_basic/q"]), [[1, 2, 3, 4, 5, 6, 7, 8],
                                                                      [0, 1, 2, 3, 4, 5, 6, 7]])


def test_int4_swapped_nibbles_are_caught(golden):
    q = golden["i4_large/q"]
    swapped = ((q >> 4) | (q << 4)).astype(np.uint8)
    out = oracle.dequant_matmul_grouped_i4(golden["i4_large/x"], swapped, golden["i4_large/scale"],
                                           golden["i4_large/zero"], int(golden["i4_large/group_size"]))
    assert oracle.normwise_rel_err(out, golden["i4_large/out"]) > 1e-3


def test_int4_quantize_test_loop_matches_reference(golden):
    q, s, z = oracle.quantize_grouped_i4(golden["qi4_basic/w"], int(golden["qi4_basic/group_size"]), test_loop=True)
    np.testing.assert_array_equal(q, golden["qi4_basic/packed_test_loop"])
    np.testing.assert_array_equal(s.view(np.uint32), golden["qi4_basic/scale"].view(np.uint32))
    np.testing.assert_array_equal(z.view(np.uint32), golden["qi4_basic/zero"].view(np.uint32))
    # Group (0..3): scale 3/15, zero 0, codes round(v * 5) -> 0, 5, 10, 15.
    np.testing.assert_array_equal(_unpack_i4(q)[0, :4], [0, 5, 10, 15])


def test_int4_quantize_variants_differ_only_on_ties():
    w = oracle.fill_normal(16 * 512, 41, 0.02).reshape(16, 512)
    qk, sk, zk = oracle.quantize_grouped_i4(w, 64)
    qt, st, zt = oracle.quantize_grouped_i4(w, 64, test_loop=True)
    np.testing.assert_array_equal(sk, st)
    np.testing.assert_array_equal(zk, zt)
    ck, ct = _unpack_i4(qk), _unpack_i4(qt)
    g = np.arange(512) // 64
    d = w / sk[:, g] + zk[:, g]
    ties = (d - np.floor(d)) == 0.5
    assert np.all(ck[~ties] == ct[~ties])
    assert np.all(np.abs(ck - ct) <= 1)


def _kernel_order_key(i):
    """Rank of element i of a group in popcorn's 256-thread min/max block:
    thread i % 256 (its tree keeps the lower partner, so threads rank by their
    bit-reversed index), then the thread's own scan order i // 256."""
    t = i % 256
    rev = int(f"{t:08b}"[::-1], 2)
    return (rev, i // 256)


@pytest.mark.parametrize("gs", [256, 512, 96, 2048])
def test_int4_quantize_zero_sign_follows_the_kernel_block_order(gs):
    rng = np.random.default_rng(gs)
    for trial in range(20):
        w = np.zeros((1, gs), dtype=np.float32)
        neg = rng.choice(gs, size=int(rng.integers(1, 4)), replace=False)
        w[0, neg] = -0.0
        q, s, z = oracle.quantize_grouped_i4(w, gs)
        # All values compare equal, so min is the element the block keeps:
        # the smallest key; zero = -min / 1.
        first = min(range(gs), key=_kernel_order_key)
        min_is_neg = np.signbit(w[0, first])
        assert s[0, 0] == 1.0
        assert np.signbit(z[0, 0]) == (not min_is_neg)
        assert np.all(q == 0)


def test_int4_quantize_nan_and_inf():
    w = oracle.fill_normal(4 * 32, 3, 1.0).reshape(4, 32).copy()
    w[0, 5] = np.nan                 # skipped by min/max; its own code packs as 0
    w[1, :16] = np.nan               # a group of NaN only: min +inf, max -inf
    w[2, 3] = np.inf
    q, s, z = oracle.quantize_grouped_i4(w, 16)
    finite = np.delete(w[0, :16], 5)
    assert s[0, 0] == np.float32(np.float32(finite.max() - finite.min()) / np.float32(15))
    assert _unpack_i4(q)[0, 5] == 0
    assert s[1, 0] == -np.inf and np.isnan(z[1, 0]) and np.all(_unpack_i4(q)[1, :16] == 0)
    assert s[2, 0] == np.inf


@pytest.mark.skipif(not oracle.have_ref_loops(), reason="reference loops not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(1, 7, 8, 4), (3, 17, 64, 16), (5, 33, 96, 32), (4, 40, 256, 128), (2, 9, 36, 6),
                                   (2, 5, 30, 3)])
def test_int4_oracle_equals_reference_loops_random(shape):
    M, N, K, gs = shape
    x = oracle.fill_normal(M * K, M + N, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, K, 0.02).reshape(N, K)
    if gs % 2 == 0:
        qr, sr, zr = oracle.ref_quantize_grouped_i4(w, gs)
        qo, so, zo = oracle.quantize_grouped_i4(w, gs, test_loop=True)
        np.testing.assert_array_equal(qr, qo)
        np.testing.assert_array_equal(sr, so)
        np.testing.assert_array_equal(zr, zo)
    else:
        qr, sr, zr = oracle.quantize_grouped_i4(w, gs)
    np.testing.assert_array_equal(oracle.ref_dequant_matmul_grouped_i4(x, qr, sr, zr, gs),
                                  oracle.dequant_matmul_grouped_i4(x, qr, sr, zr, gs, threads=2))


def test_bf16_dequantize_rounds_to_nearest_even():
    # The oracle's bf16 expansion equals torch's own f32 -> bf16 conversion
    # (round to nearest, ties to even) of the f32 product, including exact
    # ties, values that round up into the next binade, subnormals and zeros.
    import torch

    N, K = 64, 256
    q, s = oracle.quantize(oracle.fill_normal(N * K, 3, 0.02).reshape(N, K))
    s = (s * np.exp2(np.arange(N) % 64 * 4 - 130).astype(np.float32)).astype(np.float32)
    s[1] = 1.0 + 2.0 ** -8   # q * s lands on bf16 ties for many q
    s[2] = 1.0 - 2.0 ** -9
    s[3] = 0.0
    got = oracle.dequantize_bf16(q, s)
    f32 = oracle.dequantize(q, s)
    want = torch.from_numpy(f32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, want)
