"""popcorn_b200 -- host-side mirror of popcorn's int8 dequant-matmul C ABI.

The product is the sm_100a library ``popcorn_b200/libpopcorn.so`` (and the
static archive ``lib/libpopcorn.a`` for cgo callers), built from
``popcorn_b200/csrc`` by ``make -C popcorn_b200``. This module loads that
library in-tree through ctypes and exposes

* the raw entry points under popcorn's own names (``popcornDequantizeMatmul_i8f32``
  and friends), taking device pointers as integers and returning the
  ``popcornStatus_t`` value, exactly as a cgo caller sees them
  (popcorn include/popcorn.h:11-27, :464-534);
* tensor-level helpers (``dequantize_matmul``, ``quantize``, ``dequantize``)
  that take CUDA torch tensors, pass the current torch stream, and raise
  :class:`PopcornError` on a non-success status, the way tendo turns a status
  into a Go error (popcorn README.md:85-107).

There is no fallback: if the library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpopcorn.so")

POPCORN_SUCCESS = 0
POPCORN_ERROR_INVALID_VALUE = 1
POPCORN_ERROR_CUDA = 2

PATH_AUTO = 0
PATH_SIMT_F32 = 1
PATH_TENSOR_F16 = 2
PATH_NAMES = {PATH_AUTO: "auto", PATH_SIMT_F32: "simt_f32", PATH_TENSOR_F16: "tensor_f16"}

# Every symbol declared in include/popcorn.h and include/popcorn_b200.h.
ABI_SYMBOLS = (
    "popcornGetErrorString",
    "popcornGetLastCudaError",
    "popcornGetLastCudaErrorString",
    "popcornDequantizeMatmul_i8f32",
    "popcornDequantizeMatmulBatched_i8f32",
    "popcornQuantize_f32i8",
    "popcornDequantizeMatmulGrouped_i8f32",
    "popcornQuantizeGrouped_f32i8",
    "popcornDequantizeMatmulGrouped_i4f32",
    "popcornQuantizeGrouped_f32i4",
)
EXT_SYMBOLS = (
    "popcornDequantize_i8f32",
    "popcornDequantize_i8bf16",
    "popcornDequantizeMatmulPath_i8f32",
    "popcornDequantizeMatmulSelectPath",
    "popcornDequantizeMatmulLaunchCount",
    "popcornB200DeviceErrors",
    "popcornDequantizeMatmulNoAlloc_i8f32",
    "popcornDequantizeMatmulAllGather_i8f32",
    "popcornDequantizeMatmulAllReduce_i8f32",
    "popcornRMSNormDequantizeMatmul_i8f32",
    "popcornDequantizeMatmulSiluMul_i8f32",
    "popcornRMSNormDequantizeMatmulSiluMul_i8f32",
    "popcornDequantizeMatmulColumnParallel_i8f32",
    "popcornDequantizeMatmulRowParallel_i8f32",
    "popcornGetLastNcclError",
)

TP_MAX_RANKS = 8


class TpGroup(ctypes.Structure):
    """popcornTpGroup_t (include/popcorn_tp.h)."""

    _fields_ = [
        ("recv", ctypes.c_void_p * TP_MAX_RANKS),
        ("recv_bytes", ctypes.c_int64),
        ("state", ctypes.c_void_p),
        ("rank", ctypes.c_int),
        ("world", ctypes.c_int),
    ]

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

_SIGNATURES = {
    "popcornGetErrorString": (ctypes.c_char_p, [_int]),
    "popcornGetLastCudaError": (_int, []),
    "popcornGetLastCudaErrorString": (ctypes.c_char_p, []),
    "popcornDequantizeMatmul_i8f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulBatched_i8f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "popcornQuantize_f32i8": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "popcornDequantizeMatmulGrouped_i8f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "popcornQuantizeGrouped_f32i8": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulGrouped_i4f32": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "popcornQuantizeGrouped_f32i4": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantize_i8f32": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "popcornDequantize_i8bf16": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "popcornDequantizeMatmulPath_i8f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "popcornDequantizeMatmulSelectPath": (_int, [_vp, _vp, _i64, _i64, _i64]),
    "popcornDequantizeMatmulLaunchCount": (_int, [_vp, _vp, _i64, _i64, _i64, _int]),
    "popcornB200DeviceErrors": (_int, [ctypes.POINTER(ctypes.c_uint)]),
    "popcornDequantizeMatmulNoAlloc_i8f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulAllGather_i8f32": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulAllReduce_i8f32": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornRMSNormDequantizeMatmul_i8f32": (_int, [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulSiluMul_i8f32": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornRMSNormDequantizeMatmulSiluMul_i8f32": (_int, [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _i64,
                                                           _i64, _i64, _vp]),
    "popcornDequantizeMatmulColumnParallel_i8f32": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornDequantizeMatmulRowParallel_i8f32": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "popcornGetLastNcclError": (_int, []),
}

_lib = None


class PopcornError(RuntimeError):
    """A non-success popcornStatus_t, with the CUDA error behind it if any."""

    def __init__(self, status: int, where: str):
        lib = load_library()
        msg = lib.popcornGetErrorString(status).decode()
        self.status = status
        self.cuda_error = None
        if status == POPCORN_ERROR_CUDA:
            self.cuda_error = lib.popcornGetLastCudaError()
            msg += ": " + lib.popcornGetLastCudaErrorString().decode()
        super().__init__(f"{where}: {msg}")


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load the in-tree sm_100a library (raises OSError if it is not built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise OSError(f"popcorn_b200 library not built: {p} (run `make -C popcorn_b200`)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ---------------------------------------------------------------------------
# Raw entry points: device pointers as ints, popcornStatus_t returned.
# ---------------------------------------------------------------------------
def popcornDequantizeMatmul_i8f32(out, x, qweight, scale, M, N, K, stream=0) -> int:
    return load_library().popcornDequantizeMatmul_i8f32(out, x, qweight, scale, M, N, K, stream)


def popcornDequantizeMatmulBatched_i8f32(out, x, qweight, scale, B, M, N, K, stream=0) -> int:
    return load_library().popcornDequantizeMatmulBatched_i8f32(out, x, qweight, scale, B, M, N, K, stream)


def popcornQuantize_f32i8(out, scale, inp, N, K, stream=0) -> int:
    return load_library().popcornQuantize_f32i8(out, scale, inp, N, K, stream)


def popcornDequantizeMatmulGrouped_i8f32(out, x, qweight, scale, M, N, K, group_size, stream=0) -> int:
    return load_library().popcornDequantizeMatmulGrouped_i8f32(out, x, qweight, scale, M, N, K, group_size, stream)


def popcornQuantizeGrouped_f32i8(out, scale, inp, N, K, group_size, stream=0) -> int:
    return load_library().popcornQuantizeGrouped_f32i8(out, scale, inp, N, K, group_size, stream)


def popcornDequantizeMatmulGrouped_i4f32(out, x, qweight, scale, zero, M, N, K, group_size, stream=0) -> int:
    return load_library().popcornDequantizeMatmulGrouped_i4f32(out, x, qweight, scale, zero, M, N, K, group_size,
                                                               stream)


def popcornQuantizeGrouped_f32i4(out, scale, zero, inp, N, K, group_size, stream=0) -> int:
    return load_library().popcornQuantizeGrouped_f32i4(out, scale, zero, inp, N, K, group_size, stream)


def popcornDequantize_i8f32(out, qweight, scale, N, K, stream=0) -> int:
    return load_library().popcornDequantize_i8f32(out, qweight, scale, N, K, stream)


def popcornDequantize_i8bf16(out, qweight, scale, N, K, stream=0) -> int:
    return load_library().popcornDequantize_i8bf16(out, qweight, scale, N, K, stream)


def popcornDequantizeMatmulPath_i8f32(out, x, qweight, scale, M, N, K, path, stream=0) -> int:
    return load_library().popcornDequantizeMatmulPath_i8f32(out, x, qweight, scale, M, N, K, path, stream)


def popcornDequantizeMatmulNoAlloc_i8f32(out, x, qweight, scale, M, N, K, stream=0) -> int:
    return load_library().popcornDequantizeMatmulNoAlloc_i8f32(out, x, qweight, scale, M, N, K, stream)


def select_path(x_ptr: int, q_ptr: int, M: int, N: int, K: int) -> int:
    return load_library().popcornDequantizeMatmulSelectPath(x_ptr, q_ptr, M, N, K)


def launch_count(x_ptr: int, q_ptr: int, M: int, N: int, K: int, path: int = PATH_AUTO) -> int:
    return load_library().popcornDequantizeMatmulLaunchCount(x_ptr, q_ptr, M, N, K, path)


def device_errors() -> int:
    """Read and clear the current device's kernel error bits (0 = none)."""
    flags = ctypes.c_uint(0)
    st = load_library().popcornB200DeviceErrors(ctypes.byref(flags))
    if st != POPCORN_SUCCESS:
        raise PopcornError(st, "popcornB200DeviceErrors")
    return flags.value


def _check(status: int, where: str) -> None:
    if status != POPCORN_SUCCESS:
        raise PopcornError(status, where)


# ---------------------------------------------------------------------------
# Tensor helpers (CUDA torch tensors, contiguous).
# ---------------------------------------------------------------------------
def dequantize_matmul(x, qweight, scale, out=None, path: int = PATH_AUTO, stream=None):
    """out[M, N] = x[M, K] @ (qweight[N, K] * scale[N, None]).T in f32."""
    import torch

    M, K = x.shape
    N = qweight.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    _check(
        popcornDequantizeMatmulPath_i8f32(
            out.data_ptr(), x.data_ptr(), qweight.data_ptr(), scale.data_ptr(), M, N, K, path, st
        ),
        "popcornDequantizeMatmulPath_i8f32",
    )
    return out


def dequantize_matmul_batched(x, qweight, scale, out=None, stream=None):
    """out[B, M, N] = x[B, M, K] @ (qweight * scale[:, None]).T in f32."""
    import torch

    B, M, K = x.shape
    N = qweight.shape[0]
    if out is None:
        out = torch.empty((B, M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    _check(
        popcornDequantizeMatmulBatched_i8f32(
            out.data_ptr(), x.data_ptr(), qweight.data_ptr(), scale.data_ptr(), B, M, N, K, st
        ),
        "popcornDequantizeMatmulBatched_i8f32",
    )
    return out


def quantize(w, out=None, scale=None, stream=None):
    """Per-row symmetric int8 quantization of f32 [N, K] -> (codes, scales)."""
    import torch

    N, K = w.shape
    if out is None:
        out = torch.empty((N, K), dtype=torch.int8, device=w.device)
    if scale is None:
        scale = torch.empty((N,), dtype=torch.float32, device=w.device)
    st = _stream_handle(stream)
    _check(popcornQuantize_f32i8(out.data_ptr(), scale.data_ptr(), w.data_ptr(), N, K, st), "popcornQuantize_f32i8")
    return out, scale


def quantize_grouped(w, group_size: int, out=None, scale=None, stream=None):
    """Per-group symmetric int8 quantization of f32 [N, K] -> (codes [N, K], scales [N, K / group_size])."""
    import torch

    N, K = w.shape
    if out is None:
        out = torch.empty((N, K), dtype=torch.int8, device=w.device)
    if scale is None:
        scale = torch.empty((N, K // group_size), dtype=torch.float32, device=w.device)
    st = _stream_handle(stream)
    _check(popcornQuantizeGrouped_f32i8(out.data_ptr(), scale.data_ptr(), w.data_ptr(), N, K, group_size, st),
           "popcornQuantizeGrouped_f32i8")
    return out, scale


def dequantize_matmul_grouped(x, qweight, scale, group_size: int, out=None, stream=None):
    """out[M, N] = x[M, K] @ (qweight[N, K] * scale[N, k // group_size]).T on the device."""
    import torch

    M, K = x.shape
    N = qweight.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    _check(popcornDequantizeMatmulGrouped_i8f32(out.data_ptr(), x.data_ptr(), qweight.data_ptr(), scale.data_ptr(),
                                                M, N, K, group_size, st), "popcornDequantizeMatmulGrouped_i8f32")
    return out


def quantize_grouped_i4(w, group_size: int, out=None, scale=None, zero=None, stream=None):
    """Per-group asymmetric int4 quantization of f32 [N, K] ->
    (packed codes uint8 [N, K / 2] low nibble first, scales and zero points [N, K / group_size])."""
    import torch

    N, K = w.shape
    G = K // group_size if group_size > 0 else 0
    if out is None:
        out = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    if scale is None:
        scale = torch.empty((N, G), dtype=torch.float32, device=w.device)
    if zero is None:
        zero = torch.empty((N, G), dtype=torch.float32, device=w.device)
    st = _stream_handle(stream)
    _check(popcornQuantizeGrouped_f32i4(out.data_ptr(), scale.data_ptr(), zero.data_ptr(), w.data_ptr(), N, K,
                                        group_size, st), "popcornQuantizeGrouped_f32i4")
    return out, scale, zero


def dequantize_matmul_grouped_i4(x, qweight, scale, zero, group_size: int, out=None, stream=None):
    """out[M, N] = x[M, K] @ ((codes(qweight)[N, K] - zero[N, g]) * scale[N, g]).T, g = k // group_size."""
    import torch

    M, K = x.shape
    N = qweight.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    _check(popcornDequantizeMatmulGrouped_i4f32(out.data_ptr(), x.data_ptr(), qweight.data_ptr(), scale.data_ptr(),
                                                zero.data_ptr(), M, N, K, group_size, st),
           "popcornDequantizeMatmulGrouped_i4f32")
    return out


def _ptr_or_null(t):
    return None if t is None else t.data_ptr()


def rmsnorm_dequantize_matmul(x, norm_weight, eps: float, qweight, scale, out=None, stream=None):
    """out[M, N] = RMSNorm(x; norm_weight, eps) @ (qweight * scale[:, None]).T (norm_weight may be None)."""
    import torch

    M, K = x.shape
    N = qweight.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    _check(load_library().popcornRMSNormDequantizeMatmul_i8f32(out.data_ptr(), x.data_ptr(), _ptr_or_null(norm_weight),
                                                              eps, qweight.data_ptr(), scale.data_ptr(), M, N, K, st),
           "popcornRMSNormDequantizeMatmul_i8f32")
    return out


def dequantize_matmul_silu_mul(x, q_gate, s_gate, q_up, s_up, norm_weight=None, eps=None, out=None, stream=None):
    """out[M, N] = silu(x' @ W_gate.T) * (x' @ W_up.T) with x' = x, or RMSNorm(x; norm_weight, eps)
    when eps is given (norm_weight may then be None)."""
    import torch

    M, K = x.shape
    N = q_gate.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    st = _stream_handle(stream)
    lib = load_library()
    if eps is None:
        _check(lib.popcornDequantizeMatmulSiluMul_i8f32(out.data_ptr(), x.data_ptr(), q_gate.data_ptr(),
                                                        s_gate.data_ptr(), q_up.data_ptr(), s_up.data_ptr(), M, N, K,
                                                        st), "popcornDequantizeMatmulSiluMul_i8f32")
    else:
        _check(lib.popcornRMSNormDequantizeMatmulSiluMul_i8f32(out.data_ptr(), x.data_ptr(), _ptr_or_null(norm_weight),
                                                               eps, q_gate.data_ptr(), s_gate.data_ptr(),
                                                               q_up.data_ptr(), s_up.data_ptr(), M, N, K, st),
               "popcornRMSNormDequantizeMatmulSiluMul_i8f32")
    return out


def dequantize(qweight, scale, out=None, stream=None, dtype=None):
    """[N, K] = qweight[N, K] * scale[N, None] in f32, or rounded to bf16 with dtype=torch.bfloat16."""
    import torch

    N, K = qweight.shape
    dtype = dtype or (out.dtype if out is not None else torch.float32)
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("dequantize writes float32 or bfloat16")
    if out is None:
        out = torch.empty((N, K), dtype=dtype, device=qweight.device)
    st = _stream_handle(stream)
    if dtype == torch.bfloat16:
        _check(popcornDequantize_i8bf16(out.data_ptr(), qweight.data_ptr(), scale.data_ptr(), N, K, st),
               "popcornDequantize_i8bf16")
    else:
        _check(popcornDequantize_i8f32(out.data_ptr(), qweight.data_ptr(), scale.data_ptr(), N, K, st),
               "popcornDequantize_i8f32")
    return out
