"""Generate the golden vectors in tests/golden from popcorn's own CPU loops.

Run from the repository root after ``make -C oracle ref`` (needs the reference
checkout to build oracle/_ref/libref_loops.so):

    python tests/golden/make_golden.py

Inputs are the reference test suite's own in-test fixtures, rebuilt here with
the same formulas (each case cites popcorn test/test_quantize.cu), plus the
seeded host-parity configuration (M=16, K=1024, N=1024; X ~ N(0,1), W ~
N(0,0.02), per-row int8). Expected outputs come from the reference loops
``ref_dequant_matmul_i8`` (:24-41), ``ref_quantize_i8`` (:677-706) and their
per-group forms ``ref_dequant_matmul_grouped_i8`` (:42-61) and
``ref_quantize_grouped_i8`` (:709-742) and the int4 loops
``ref_dequant_matmul_grouped_i4`` (:67-99) and ``ref_quantize_grouped_i4``
(:746-789), compiled from the reference sources,
never from this repository's code. Cases whose
values the test spells out (the identity test) also store those values.
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden")

CONFIG1 = dict(M=16, K=1024, N=1024, x_seed=0, w_seed=1, x_sigma=1.0, w_sigma=0.02)


def f32(a):
    return np.asarray(a, dtype=np.float32)


def matmul_cases():
    cases = {}
    # dequant_matmul_i8_basic, test_quantize.cu:107-145
    x = f32([[1, 2, 3, 4], [5, 6, 7, 8]])
    q = np.array([[1, 2, 3, 4], [-1, -2, -3, -4], [2, 0, 2, 0]], dtype=np.int8)
    s = f32([0.5, 0.25, 1.0])
    cases["basic"] = (x, q, s)
    # dequant_matmul_i8_identity, :147-191
    x = np.diag(f32([1, 2, 3, 4]))
    q = np.eye(4, dtype=np.int8)
    s = f32([1, 1, 1, 1])
    cases["identity"] = (x, q, s)
    # dequant_matmul_i8_large, :193-238 (M64 N256 K128, patterned data)
    M, N, K = 64, 256, 128
    x = ((np.arange(M * K) % 100).astype(np.float32) - np.float32(50.0)) * np.float32(0.01)
    q = ((np.arange(N * K) % 256) - 128).astype(np.int8)
    s = np.float32(0.01) + (np.arange(N) % 10).astype(np.float32) * np.float32(0.001)
    cases["large"] = (x.reshape(M, K), q.reshape(N, K), s)
    # dequant_matmul_i8_single_row, :240-276
    x = f32([[1, 2, 3, 4, 5, 6, 7, 8]])
    q = np.array([[1] * 8, [2] * 8, [-1] * 8, [0] * 8], dtype=np.int8)
    s = f32([0.1, 0.2, 0.5, 1.0])
    cases["single_row"] = (x, q, s)
    return cases


def batched_cases():
    cases = {}
    # dequant_matmul_batched_i8_basic, :414-465 (B2 M2 N3 K4)
    x = f32([[1, 2, 3, 4], [5, 6, 7, 8], [-1, -2, -3, -4], [-5, -6, -7, -8]]).reshape(2, 2, 4)
    q = np.array([[1, 2, 3, 4], [-1, -2, -3, -4], [2, 0, 2, 0]], dtype=np.int8)
    s = f32([0.5, 0.25, 1.0])
    cases["batched_basic"] = (x, q, s)
    # dequant_matmul_batched_i8_large, :467-519 (B8 M16 N32 K64)
    B, M, N, K = 8, 16, 32, 64
    x = ((np.arange(B * M * K) % 100).astype(np.float32) - np.float32(50.0)) * np.float32(0.01)
    q = ((np.arange(N * K) % 200) - 100).astype(np.int8)
    s = np.float32(0.01) + (np.arange(N) % 10).astype(np.float32) * np.float32(0.002)
    cases["batched_large"] = (x.reshape(B, M, K), q.reshape(N, K), s)
    return cases


def quantize_cases():
    cases = {}
    # quantize_i8_basic, :793-832
    cases["q_basic"] = f32([[1, -2, 3, -4], [0.5, 0.5, 0.5, 0.5], [127, 0, -127, 0]])
    # quantize_i8_large, :834-873 (N64 K256)
    cases["q_large"] = (((np.arange(64 * 256) % 200).astype(np.float32) - np.float32(100.0))
                        * np.float32(0.5)).reshape(64, 256)
    # quantize_roundtrip_i8, :970-1024 (includes an all-zero row -> scale 1)
    cases["q_roundtrip"] = f32([
        [1, 2, 3, 4, 5, 6, 7, 8],
        [-1, -2, -3, -4, -5, -6, -7, -8],
        [0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5, 7.5],
        [0, 0, 0, 0, 0, 0, 0, 0],
    ])
    # Exact .5 quotients: max 127 -> scale exactly 1, so v/scale = v and
    # popcorn's GPU rintf (half to even) and its test loop's roundf (half away)
    # disagree on every element.
    cases["q_ties"] = f32([[127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5]])
    return cases


def grouped_cases():
    cases = {}
    # dequant_matmul_grouped_i8_basic, test_quantize.cu:283-327 (M2 N3 K8, group 4)
    x = f32([[1, 2, 3, 4, 5, 6, 7, 8], [-1, -2, -3, -4, -5, -6, -7, -8]])
    q = np.array([[1, 2, 3, 4, 5, 6, 7, 8], [-1, -2, -3, -4, -5, -6, -7, -8], [1, 1, 1, 1, 2, 2, 2, 2]],
                 dtype=np.int8)
    s = f32([[0.5, 0.25], [1.0, 0.5], [0.1, 0.2]])
    cases["g_basic"] = (x, q, s, 4)
    # dequant_matmul_grouped_i8_large, :329-379 (M32 N64 K128, group 32, patterned data)
    M, N, K, gs = 32, 64, 128, 32
    x = ((np.arange(M * K) % 50).astype(np.float32) - np.float32(25.0)) * np.float32(0.02)
    q = ((np.arange(N * K) % 200) - 100).astype(np.int8)
    s = np.float32(0.005) + (np.arange(N * (K // gs)) % 20).astype(np.float32) * np.float32(0.001)
    cases["g_large"] = (x.reshape(M, K), q.reshape(N, K), s.reshape(N, K // gs), gs)
    return cases


def int4_cases():
    cases = {}
    # dequant_matmul_grouped_i4_basic, test_quantize.cu:525-572 (M2 N2 K8, group 4)
    x = f32([[1, 2, 3, 4, 5, 6, 7, 8], [0.5, 1, 1.5, 2, 2.5, 3, 3.5, 4]])
    q = np.array([[0x21, 0x43, 0x65, 0x87], [0x10, 0x32, 0x54, 0x76]], dtype=np.uint8)
    s = f32([[0.5, 0.25], [1.0, 0.5]])
    z = f32([[8, 8], [7, 7]])
    cases["i4_basic"] = (x, q, s, z, 4)
    # dequant_matmul_grouped_i4_large, :574-626 (M16 N32 K64, group 32, patterned data)
    M, N, K, gs = 16, 32, 64, 32
    x = ((np.arange(M * K) % 50).astype(np.float32) - np.float32(25.0)) * np.float32(0.02)
    q = ((np.arange(N * (K // 2)) * 7 + 3) % 256).astype(np.uint8)
    g = np.arange(N * (K // gs))
    s = np.float32(0.01) + (g % 10).astype(np.float32) * np.float32(0.002)
    z = np.float32(7.5) + (g % 3).astype(np.float32) * np.float32(0.5)
    cases["i4_large"] = (x.reshape(M, K), q.reshape(N, K // 2), s.reshape(N, K // gs), z.reshape(N, K // gs), gs)
    return cases


def config1_inputs():
    c = CONFIG1
    x = oracle.fill_normal(c["M"] * c["K"], c["x_seed"], c["x_sigma"]).reshape(c["M"], c["K"])
    w = oracle.fill_normal(c["N"] * c["K"], c["w_seed"], c["w_sigma"]).reshape(c["N"], c["K"])
    return x, w


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    if not oracle.have_ref_loops():
        raise SystemExit("oracle/_ref/libref_loops.so missing: run `make -C oracle ref` first")
    data = {}
    for name, (x, q, s) in matmul_cases().items():
        data[f"{name}/x"], data[f"{name}/q"], data[f"{name}/scale"] = x, q, s
        data[f"{name}/out"] = oracle.ref_dequant_matmul(x, q, s)
    data["identity/expected_literal"] = np.diag(f32([1, 2, 3, 4]))
    for name, (x, q, s) in batched_cases().items():
        B, M, K = x.shape
        out = np.stack([oracle.ref_dequant_matmul(x[b], q, s) for b in range(B)])
        data[f"{name}/x"], data[f"{name}/q"], data[f"{name}/scale"], data[f"{name}/out"] = x, q, s, out
    for name, w in quantize_cases().items():
        qr, sr = oracle.ref_quantize(w)
        data[f"{name}/w"], data[f"{name}/codes_test_loop"], data[f"{name}/scale"] = w, qr, sr

    for name, (x, q, s, gs) in grouped_cases().items():
        data[f"{name}/x"], data[f"{name}/q"], data[f"{name}/scale"] = x, q, s
        data[f"{name}/group_size"] = np.array(gs, dtype=np.int64)
        data[f"{name}/out"] = oracle.ref_dequant_matmul_grouped(x, q, s, gs)
    # quantize_grouped_i8_basic, :875-917 (N2 K8, group 4)
    w = f32([[1, 2, 3, 4, -8, -6, -4, -2], [0.1, 0.2, 0.3, 0.4, 12.7, 0, -12.7, 6.35]])
    qr, sr = oracle.ref_quantize_grouped(w, 4)
    data["qg_basic/w"], data["qg_basic/codes_test_loop"], data["qg_basic/scale"] = w, qr, sr
    data["qg_basic/group_size"] = np.array(4, dtype=np.int64)

    for name, (x, q, s, z, gs) in int4_cases().items():
        data[f"{name}/x"], data[f"{name}/q"], data[f"{name}/scale"], data[f"{name}/zero"] = x, q, s, z
        data[f"{name}/group_size"] = np.array(gs, dtype=np.int64)
        data[f"{name}/out"] = oracle.ref_dequant_matmul_grouped_i4(x, q, s, z, gs)
    # quantize_grouped_i4_basic, :919-968 (N2 K8, group 4)
    w = f32([[0, 1, 2, 3, 4, 5, 6, 7], [-1, 0, 1, 2, 10, 11, 12, 13]])
    qr, sr, zr = oracle.ref_quantize_grouped_i4(w, 4)
    data["qi4_basic/w"], data["qi4_basic/packed_test_loop"] = w, qr
    data["qi4_basic/scale"], data["qi4_basic/zero"] = sr, zr
    data["qi4_basic/group_size"] = np.array(4, dtype=np.int64)

    x, w = config1_inputs()
    q, s = oracle.ref_quantize(w)
    data["config1/x_sha256"] = np.array(sha256(x))
    data["config1/w_sha256"] = np.array(sha256(w))
    data["config1/codes_test_loop_sha256"] = np.array(sha256(q))
    data["config1/scale"] = s
    data["config1/out"] = oracle.ref_dequant_matmul(x, q, s)
    data["config1/shape"] = np.array([CONFIG1["M"], CONFIG1["K"], CONFIG1["N"]], dtype=np.int64)

    path = os.path.join(OUT, "popcorn_ref_vectors.npz")
    np.savez_compressed(path, **data)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
