"""CPU oracle of popcorn's int8 dequant-matmul path -- TEST INFRASTRUCTURE.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package, and only as the checker or the timed CPU
baseline. The product path (``popcorn_b200``) never imports it.

* :func:`dequant_matmul`, :func:`quantize`, their per-group int8 and int4
  forms, :func:`dequantize` and :func:`fill_normal` wrap ``liboracle.so``
  (oracle.c, the C restatement).
* :func:`ref_loops` loads ``_ref/libref_loops.so``: popcorn's own test-side
  CPU loops (test/test_quantize.cu:24-41, :677-706) compiled from the
  reference sources; it pins the restatement and is the "reference" CPU
  baseline.
* :func:`popcorn_ref_gpu` loads ``_ref/libpopcorn_ref.so``: popcorn's own
  quantize.cu rebuilt for sm_100a, the GPU parity baseline.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(_HERE, "liboracle.so")
REF_LOOPS_LIB = os.path.join(_HERE, "_ref", "libref_loops.so")
REF_GPU_LIB = os.path.join(_HERE, "_ref", "libpopcorn_ref.so")

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

_lib = None
_ref_loops = None
_ref_gpu = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_LIB):
            raise OSError(f"oracle not built: {ORACLE_LIB} (run `make -C oracle`)")
        lib = ctypes.CDLL(ORACLE_LIB)
        lib.oracle_dequant_matmul_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int]
        lib.oracle_dequant_matmul_i8_mt.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int]
        lib.oracle_quantize_i8.argtypes = [_vp, _vp, _vp, _i64, _i64, _int]
        lib.oracle_dequantize_i8.argtypes = [_vp, _vp, _vp, _i64, _i64]
        lib.oracle_dequantize_i8_bf16.argtypes = [_vp, _vp, _vp, _i64, _i64]
        lib.oracle_fill_normal.argtypes = [_vp, _i64, ctypes.c_uint64, ctypes.c_float]
        lib.oracle_dequant_matmul_grouped_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int]
        lib.oracle_quantize_grouped_i8.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _int]
        lib.oracle_dequant_matmul_grouped_i4.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int]
        lib.oracle_quantize_grouped_i4.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int]
        lib.oracle_rmsnorm.argtypes = [_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int]
        lib.oracle_silu.argtypes = [_vp, _vp, _i64]
        for f in (lib.oracle_rmsnorm, lib.oracle_silu, lib.oracle_dequant_matmul_i8, lib.oracle_dequant_matmul_i8_mt, lib.oracle_quantize_i8,
                  lib.oracle_dequantize_i8, lib.oracle_dequantize_i8_bf16, lib.oracle_fill_normal, lib.oracle_dequant_matmul_grouped_i8,
                  lib.oracle_quantize_grouped_i8, lib.oracle_dequant_matmul_grouped_i4,
                  lib.oracle_quantize_grouped_i4):
            f.restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def fill_normal(n: int, seed: int, sigma: float) -> np.ndarray:
    """Deterministic ~N(0, sigma^2) f32 vector (SplitMix64 + Irwin-Hall(12))."""
    out = np.empty(n, dtype=np.float32)
    _load().oracle_fill_normal(_ptr(out), n, seed & 0xFFFFFFFFFFFFFFFF, sigma)
    return out


def dequant_matmul(x, q, scale, fused: bool = False, threads: int = 1) -> np.ndarray:
    """out[M,N] = sum_k x[m,k] * (q[n,k] * scale[n]) with popcorn's k order."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    if threads > 1:
        _load().oracle_dequant_matmul_i8_mt(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K, int(fused), threads)
    else:
        _load().oracle_dequant_matmul_i8(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K, int(fused))
    return out


def quantize(w, ties_away: bool = False):
    """(codes int8 [N,K], scales f32 [N]); rintf unless ties_away (roundf)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N,), dtype=np.float32)
    _load().oracle_quantize_i8(_ptr(q), _ptr(s), _ptr(w), N, K, int(ties_away))
    return q, s


def dequant_matmul_grouped(x, q, scale, group_size: int, fused: bool = False, threads: int = 1) -> np.ndarray:
    """out[M,N] = sum_k x[m,k] * (q[n,k] * scale[n, k // group_size]) with popcorn's k order."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    assert K % group_size == 0 and scale.size == N * (K // group_size)
    out = np.empty((M, N), dtype=np.float32)
    _load().oracle_dequant_matmul_grouped_i8(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K, group_size,
                                             int(fused), threads)
    return out


def quantize_grouped(w, group_size: int, ties_away: bool = False):
    """(codes int8 [N,K], scales f32 [N, K/group_size]); rintf unless ties_away."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    assert K % group_size == 0
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N, K // group_size), dtype=np.float32)
    _load().oracle_quantize_grouped_i8(_ptr(q), _ptr(s), _ptr(w), N, K, group_size, int(ties_away))
    return q, s


def dequant_matmul_grouped_i4(x, q, scale, zero, group_size: int, fused: bool = False,
                              threads: int = 1) -> np.ndarray:
    """out[M,N] = sum_k x[m,k] * ((nibble(q, n, k) - zero[n,g]) * scale[n,g]), g = k // group_size,
    popcorn's k order; q is [N, K/2] uint8, low nibble first."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    zero = np.ascontiguousarray(zero, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    assert K % 2 == 0 and K % group_size == 0 and q.shape == (N, K // 2)
    assert scale.size == N * (K // group_size) and zero.size == scale.size
    out = np.empty((M, N), dtype=np.float32)
    _load().oracle_dequant_matmul_grouped_i4(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), _ptr(zero), M, N, K,
                                             group_size, int(fused), threads)
    return out


def quantize_grouped_i4(w, group_size: int, test_loop: bool = False):
    """(packed uint8 [N, K/2], scale f32 [N, K/gs], zero f32 [N, K/gs]).

    Default: popcorn's GPU kernels (rintf, NaN-skipping min/max in its block
    order); ``test_loop``: popcorn's CPU test loop (roundf, first-value start,
    even group sizes only)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    assert K % 2 == 0 and K % group_size == 0
    assert not test_loop or group_size % 2 == 0
    q = np.empty((N, K // 2), dtype=np.uint8)
    s = np.empty((N, K // group_size), dtype=np.float32)
    z = np.empty((N, K // group_size), dtype=np.float32)
    _load().oracle_quantize_grouped_i4(_ptr(q), _ptr(s), _ptr(z), _ptr(w), N, K, group_size, int(test_loop))
    return q, s, z


def rmsnorm(x, weight=None, eps: float = 1e-5, fused: bool = True) -> np.ndarray:
    """popcorn's RMSNorm of the rows of x (weight may be None); fused: its GPU kernel's fmaf sum."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    out = np.empty_like(x)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    _load().oracle_rmsnorm(_ptr(out), _ptr(x), None if w is None else _ptr(w), rows, K, eps, int(fused))
    return out


def silu(x) -> np.ndarray:
    """popcorn's SiLU, x / (1 + expf(-x)), with the host's expf."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _load().oracle_silu(_ptr(out), _ptr(x), x.size)
    return out


def dequantize(q, scale) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    N, K = q.shape
    out = np.empty((N, K), dtype=np.float32)
    _load().oracle_dequantize_i8(_ptr(out), _ptr(q), _ptr(scale), N, K)
    return out


def dequantize_bf16(q, scale) -> np.ndarray:
    """bf16 bit patterns (uint16) of (float)q[n,k] * scale[n], rounded to nearest even."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    N, K = q.shape
    out = np.empty((N, K), dtype=np.uint16)
    _load().oracle_dequantize_i8_bf16(_ptr(out), _ptr(q), _ptr(scale), N, K)
    return out


def normwise_rel_err(got, ref) -> float:
    """max|got - ref| / max|ref| (the matmul parity metric)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref)) if ref.size else 0.0
    num = np.max(np.abs(got - ref)) if ref.size else 0.0
    if denom == 0.0:
        return float(num)
    return float(num / denom)


# ---------------------------------------------------------------------------
# Reference builds (oracle/_ref), present where the reference was compiled.
# ---------------------------------------------------------------------------
def reference_checkout():
    """The popcorn checkout that _ref was built from (recorded by
    ``make -C oracle ref``), or None when it is not on this machine."""
    try:
        with open(os.path.join(_HERE, "_ref", "source_dir")) as f:
            path = f.read().strip()
    except OSError:
        return None
    return path if os.path.isdir(path) else None


def have_ref_loops() -> bool:
    return os.path.exists(REF_LOOPS_LIB)


def ref_loops():
    """popcorn's own test-side CPU loops (ctypes CDLL)."""
    global _ref_loops
    if _ref_loops is None:
        lib = ctypes.CDLL(REF_LOOPS_LIB)
        lib.ref_loops_dequant_matmul_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64]
        lib.ref_loops_dequant_matmul_i8_mt.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int]
        lib.ref_loops_quantize_i8.argtypes = [_vp, _vp, _vp, _i64, _i64]
        lib.ref_loops_dequant_matmul_grouped_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64]
        lib.ref_loops_quantize_grouped_i8.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64]
        lib.ref_loops_dequant_matmul_grouped_i4.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64]
        lib.ref_loops_quantize_grouped_i4.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64]
        for f in (lib.ref_loops_dequant_matmul_i8, lib.ref_loops_dequant_matmul_i8_mt, lib.ref_loops_quantize_i8,
                  lib.ref_loops_dequant_matmul_grouped_i8, lib.ref_loops_quantize_grouped_i8,
                  lib.ref_loops_dequant_matmul_grouped_i4, lib.ref_loops_quantize_grouped_i4):
            f.restype = None
        _ref_loops = lib
    return _ref_loops


def ref_dequant_matmul(x, q, scale, threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    if threads > 1:
        ref_loops().ref_loops_dequant_matmul_i8_mt(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K, threads)
    else:
        ref_loops().ref_loops_dequant_matmul_i8(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K)
    return out


def ref_quantize(w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N,), dtype=np.float32)
    ref_loops().ref_loops_quantize_i8(_ptr(q), _ptr(s), _ptr(w), N, K)
    return q, s


def ref_dequant_matmul_grouped(x, q, scale, group_size: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    ref_loops().ref_loops_dequant_matmul_grouped_i8(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), M, N, K, group_size)
    return out


def ref_quantize_grouped(w, group_size: int):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N, K // group_size), dtype=np.float32)
    ref_loops().ref_loops_quantize_grouped_i8(_ptr(q), _ptr(s), _ptr(w), N, K, group_size)
    return q, s


def ref_dequant_matmul_grouped_i4(x, q, scale, zero, group_size: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    zero = np.ascontiguousarray(zero, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    ref_loops().ref_loops_dequant_matmul_grouped_i4(_ptr(out), _ptr(x), _ptr(q), _ptr(scale), _ptr(zero), M, N, K,
                                                    group_size)
    return out


def ref_quantize_grouped_i4(w, group_size: int):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K // 2), dtype=np.uint8)
    s = np.empty((N, K // group_size), dtype=np.float32)
    z = np.empty((N, K // group_size), dtype=np.float32)
    ref_loops().ref_loops_quantize_grouped_i4(_ptr(q), _ptr(s), _ptr(z), _ptr(w), N, K, group_size)
    return q, s, z


def have_popcorn_ref_gpu() -> bool:
    return os.path.exists(REF_GPU_LIB)


def popcorn_ref_gpu():
    """popcorn's own CUDA kernels rebuilt for sm_100a (ctypes CDLL)."""
    global _ref_gpu
    if _ref_gpu is None:
        lib = ctypes.CDLL(REF_GPU_LIB)
        lib.popcornDequantizeMatmul_i8f32.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.popcornDequantizeMatmul_i8f32.restype = _int
        lib.popcornDequantizeMatmulBatched_i8f32.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
        lib.popcornDequantizeMatmulBatched_i8f32.restype = _int
        lib.popcornQuantize_f32i8.argtypes = [_vp, _vp, _vp, _i64, _i64, _vp]
        lib.popcornQuantize_f32i8.restype = _int
        lib.popcornDequantizeMatmulGrouped_i8f32.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
        lib.popcornDequantizeMatmulGrouped_i8f32.restype = _int
        lib.popcornQuantizeGrouped_f32i8.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.popcornQuantizeGrouped_f32i8.restype = _int
        lib.popcornDequantizeMatmulGrouped_i4f32.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
        lib.popcornDequantizeMatmulGrouped_i4f32.restype = _int
        lib.popcornQuantizeGrouped_f32i4.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.popcornQuantizeGrouped_f32i4.restype = _int
        lib.popcornRMSNorm_f32.argtypes = [_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]
        lib.popcornRMSNorm_f32.restype = _int
        lib.popcornSilu_f32.argtypes = [_vp, _vp, _i64, _vp]
        lib.popcornSilu_f32.restype = _int
        lib.popcornMul_f32.argtypes = [_vp, _vp, _vp, _i64, _vp]
        lib.popcornMul_f32.restype = _int
        _ref_gpu = lib
    return _ref_gpu
