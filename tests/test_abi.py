"""CPU: the C-ABI library loads, exports what include/*.h declares, and keeps
popcorn's argument conventions for calls that launch nothing.

popcorn's conventions (src/quantize.cu:96-102, :311-317, :538-544): a null
buffer returns POPCORN_ERROR_INVALID_VALUE before sizes are looked at; any
size <= 0 returns POPCORN_SUCCESS without work. These paths return before any
CUDA call, so they run without a GPU.
"""
import ctypes
import os
import re
import subprocess

import pytest

import popcorn_b200 as pc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h)
           for h in ("popcorn.h", "popcorn_b200.h", "popcorn_tp.h", "popcorn_tp_nccl.h")]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(popcorn\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declarations_are_the_python_symbol_list():
    assert declared_functions() == sorted(pc.ABI_SYMBOLS + pc.EXT_SYMBOLS)


def _normalised(path):
    text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return " ".join(text.split())


def _prototype(norm, name):
    m = re.search(r"(?:const\s+)?\w+\*? \*?" + name + r" ?\([^;]*\);", norm)
    return None if m is None else re.sub(r"\s*([(),;*])\s*", r"\1", m.group(0))


def test_popcorn_h_matches_the_reference_header():
    # Read popcorn's own include/popcorn.h where its checkout is on this
    # machine: every hot-path prototype and the status enum must be the same
    # declaration, token for token.
    import oracle

    ref_dir = oracle.reference_checkout()
    ref_h = os.path.join(ref_dir, "include", "popcorn.h") if ref_dir else None
    if ref_h is None or not os.path.isfile(ref_h):
        pytest.skip("reference checkout not on this machine")
    ours, theirs = _normalised(HEADERS[0]), _normalised(ref_h)
    for name in pc.ABI_SYMBOLS:
        want = _prototype(theirs, name)
        assert want is not None, name
        assert _prototype(ours, name) == want, name
    enum = re.compile(r"typedef enum \{[^}]*\} popcornStatus_t;")
    assert enum.search(ours).group(0) == enum.search(theirs).group(0)


def test_popcorn_h_keeps_the_reference_signatures():
    # The exact C prototypes popcorn declares for this path
    # (include/popcorn.h:11-27, :464-473, :491-501, :527-534), whitespace-normalised;
    # the test above checks them against the reference header itself.
    norm = _normalised(HEADERS[0])
    for proto in [
        "POPCORN_SUCCESS = 0, POPCORN_ERROR_INVALID_VALUE = 1, POPCORN_ERROR_CUDA = 2, } popcornStatus_t;",
        "const char* popcornGetErrorString(popcornStatus_t status);",
        "cudaError_t popcornGetLastCudaError(void);",
        "const char* popcornGetLastCudaErrorString(void);",
        "popcornStatus_t popcornDequantizeMatmul_i8f32( float* out, const float* x, const int8_t* qweight, "
        "const float* scale, int64_t M, int64_t N, int64_t K, cudaStream_t stream );",
        "popcornStatus_t popcornDequantizeMatmulBatched_i8f32( float* out, const float* x, const int8_t* qweight, "
        "const float* scale, int64_t B, int64_t M, int64_t N, int64_t K, cudaStream_t stream );",
        "popcornStatus_t popcornQuantize_f32i8( int8_t* out, float* scale, const float* input, int64_t N, "
        "int64_t K, cudaStream_t stream );",
        # include/popcorn.h:477-487, :538-546
        "popcornStatus_t popcornDequantizeMatmulGrouped_i8f32( float* out, const float* x, const int8_t* qweight, "
        "const float* scale, int64_t M, int64_t N, int64_t K, int64_t group_size, cudaStream_t stream );",
        "popcornStatus_t popcornQuantizeGrouped_f32i8( int8_t* out, float* scale, const float* input, int64_t N, "
        "int64_t K, int64_t group_size, cudaStream_t stream );",
        # include/popcorn.h:506-517, :552-561
        "popcornStatus_t popcornDequantizeMatmulGrouped_i4f32( float* out, const float* x, const uint8_t* qweight, "
        "const float* scale, const float* zero, int64_t M, int64_t N, int64_t K, int64_t group_size, "
        "cudaStream_t stream );",
        "popcornStatus_t popcornQuantizeGrouped_f32i4( uint8_t* out, float* scale, float* zero, const float* input, "
        "int64_t N, int64_t K, int64_t group_size, cudaStream_t stream );",
    ]:
        assert proto in norm, proto


def test_shared_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_static_archive_exports_every_declared_symbol():
    archive = os.path.join(ROOT, "lib", "libpopcorn.a")
    assert os.path.exists(archive), "lib/libpopcorn.a not built"
    out = subprocess.run(["nm", "-g", "--defined-only", archive], capture_output=True, text=True, check=True).stdout
    defined = set(re.findall(r" [TW] (\w+)$", out, flags=re.M))
    for name in declared_functions():
        assert name in defined, name


def test_library_builds_for_sm100a_only():
    # The library's Makefile compiles and links every object for one target,
    # sm_100a, and nothing else (no other -gencode, no -arch shortcut).
    text = open(os.path.join(ROOT, "popcorn_b200", "Makefile")).read()
    assert re.findall(r"-gencode\s+(\S+)", text) == ["arch=compute_100a,code=sm_100a"]
    assert "-arch" not in text
    for rule in ("$(NVCC) $(NVCCFLAGS) -c", "$(NVCC) $(ARCH) -shared"):
        assert rule in text, rule
    assert "ARCH      := -gencode" in text and "$(ARCH)" in text.split("NVCCFLAGS :=")[1].split("\n")[0]


def test_error_strings(lib):
    assert lib.popcornGetErrorString(0) == b"success"
    assert lib.popcornGetErrorString(1) == b"invalid value"
    assert lib.popcornGetErrorString(2) == b"CUDA error"
    assert lib.popcornGetErrorString(7) == b"unknown error"
    assert lib.popcornGetLastCudaError() == 0
    assert lib.popcornGetLastCudaErrorString() == b"no error"


FAKE = 0x1000  # never dereferenced: these calls return before any CUDA work


def test_null_pointers_are_invalid_before_sizes(lib):
    for args in [(0, FAKE, FAKE, FAKE), (FAKE, 0, FAKE, FAKE), (FAKE, FAKE, 0, FAKE), (FAKE, FAKE, FAKE, 0)]:
        assert lib.popcornDequantizeMatmul_i8f32(*args, 1, 1, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
        assert lib.popcornDequantizeMatmul_i8f32(*args, 0, 0, 0, None) == pc.POPCORN_ERROR_INVALID_VALUE
        assert lib.popcornDequantizeMatmulBatched_i8f32(*args, 1, 1, 1, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
        assert lib.popcornDequantizeMatmulPath_i8f32(*args, 1, 1, 4, 0, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for args in [(0, FAKE, FAKE), (FAKE, 0, FAKE), (FAKE, FAKE, 0)]:
        assert lib.popcornQuantize_f32i8(*args, 1, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
        assert lib.popcornDequantize_i8f32(*args, 1, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
        assert lib.popcornDequantize_i8bf16(*args, 1, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE


@pytest.mark.parametrize("sizes", [(0, 1, 1), (1, 0, 1), (1, 1, 0), (-1, 5, 5), (5, -3, 5), (5, 5, -9)])
def test_nonpositive_sizes_are_noops(lib, sizes):
    M, N, K = sizes
    assert lib.popcornDequantizeMatmul_i8f32(FAKE, FAKE, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS
    assert lib.popcornDequantizeMatmulBatched_i8f32(FAKE, FAKE, FAKE, FAKE, 1, M, N, K, None) == pc.POPCORN_SUCCESS
    assert lib.popcornDequantizeMatmulBatched_i8f32(FAKE, FAKE, FAKE, FAKE, 0, 1, 1, 1, None) == pc.POPCORN_SUCCESS
    if N <= 0 or K <= 0:
        assert lib.popcornQuantize_f32i8(FAKE, FAKE, FAKE, N, K, None) == pc.POPCORN_SUCCESS
        assert lib.popcornDequantize_i8f32(FAKE, FAKE, FAKE, N, K, None) == pc.POPCORN_SUCCESS
        assert lib.popcornDequantize_i8bf16(FAKE, FAKE, FAKE, N, K, None) == pc.POPCORN_SUCCESS
    assert pc.launch_count(FAKE, FAKE, M, N, K) == 0


def _group(world=2, rank=0, recv_bytes=1 << 20):
    g = pc.TpGroup()
    g.world, g.rank = world, rank
    g.recv_bytes = recv_bytes
    g.state = FAKE
    for p in range(world):
        g.recv[p] = FAKE
    return g


def test_tp_group_layout_matches_header():
    # popcornTpGroup_t: 8 pointers, int64, pointer, int, int (include/popcorn_tp.h).
    assert ctypes.sizeof(pc.TpGroup) == 8 * 8 + 8 + 8 + 4 + 4
    assert pc.TpGroup.recv_bytes.offset == 64 and pc.TpGroup.state.offset == 72
    assert pc.TpGroup.rank.offset == 80 and pc.TpGroup.world.offset == 84


def test_allgather_argument_checks(lib):
    fn = lib.popcornDequantizeMatmulAllGather_i8f32
    g = _group()
    ok = (FAKE, FAKE, FAKE, FAKE)  # out, x, qweight, scale
    # null group or buffer -> invalid before sizes
    assert fn(None, *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for i in range(4):
        bufs = list(ok)
        bufs[i] = 0
        assert fn(ctypes.byref(g), *bufs, 0, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # non-positive sizes -> no-op
    assert fn(ctypes.byref(g), *ok, 0, 0, 8, 16, 64, None) == pc.POPCORN_SUCCESS
    assert fn(ctypes.byref(g), *ok, 1, 0, 0, 16, 64, None) == pc.POPCORN_SUCCESS
    # shard outside [0, N), M beyond the decode limit
    assert fn(ctypes.byref(g), *ok, 1, 12, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert fn(ctypes.byref(g), *ok, 1, -1, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert fn(ctypes.byref(g), *ok, 5, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # K % 16 != 0 or an unaligned x cannot take the vector kernel
    assert fn(ctypes.byref(g), *ok, 1, 0, 8, 16, 72, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert fn(ctypes.byref(g), FAKE, FAKE + 4, FAKE, FAKE, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # rank / world out of range
    for world, rank in ((2, 2), (9, 0), (0, 0), (2, -1)):
        bad = _group(world=max(1, min(world, 8)), rank=rank)
        bad.world = world
        assert fn(ctypes.byref(bad), *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # missing or misaligned receive area, missing state, receive area too small
    bad = _group()
    bad.recv[1] = 0
    assert fn(ctypes.byref(bad), *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    bad = _group()
    bad.recv[1] = FAKE + 4
    assert fn(ctypes.byref(bad), *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    bad = _group()
    bad.state = 0
    assert fn(ctypes.byref(bad), *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    bad = _group(recv_bytes=16 * 16 - 1)  # all-gather of M=1, N=16 needs 16 * M * N bytes
    assert fn(ctypes.byref(bad), *ok, 1, 0, 8, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE


def test_allreduce_argument_checks(lib):
    fn = lib.popcornDequantizeMatmulAllReduce_i8f32
    g = _group()
    ok = (FAKE, FAKE, FAKE, FAKE)
    assert fn(None, *ok, 1, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for i in range(4):
        bufs = list(ok)
        bufs[i] = 0
        assert fn(ctypes.byref(g), *bufs, 1, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for sizes in ((0, 16, 64), (1, 0, 64), (1, 16, 0), (-2, 16, 64)):
        assert fn(ctypes.byref(g), *ok, *sizes, None) == pc.POPCORN_SUCCESS
    assert fn(ctypes.byref(g), *ok, 5, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert fn(ctypes.byref(g), *ok, 1, 16, 40, None) == pc.POPCORN_ERROR_INVALID_VALUE
    # an all-reduce of M=1, N=16 over 2 ranks needs 16 * 2 * M * N bytes
    small = _group(recv_bytes=16 * 2 * 16 - 16)
    assert fn(ctypes.byref(small), *ok, 1, 16, 64, None) == pc.POPCORN_ERROR_INVALID_VALUE


def test_grouped_conventions(lib):
    # popcorn src/quantize.cu:190-202, :652-663: null -> invalid, sizes <= 0 ->
    # success, then group_size <= 0 or not dividing K -> invalid.
    mm = lib.popcornDequantizeMatmulGrouped_i8f32
    qg = lib.popcornQuantizeGrouped_f32i8
    for args in [(0, FAKE, FAKE, FAKE), (FAKE, 0, FAKE, FAKE), (FAKE, FAKE, 0, FAKE), (FAKE, FAKE, FAKE, 0)]:
        assert mm(*args, 1, 1, 8, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for args in [(0, FAKE, FAKE), (FAKE, 0, FAKE), (FAKE, FAKE, 0)]:
        assert qg(*args, 1, 8, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE
    for (M, N, K) in [(0, 2, 8), (2, 0, 8), (2, 2, 0), (-1, 2, 8)]:
        assert mm(FAKE, FAKE, FAKE, FAKE, M, N, K, 3, None) == pc.POPCORN_SUCCESS  # sizes first, as popcorn
    assert qg(FAKE, FAKE, FAKE, 0, 8, 3, None) == pc.POPCORN_SUCCESS
    assert qg(FAKE, FAKE, FAKE, 2, 0, 3, None) == pc.POPCORN_SUCCESS
    for gs in (0, -4, 3, 16):  # K = 10: popcorn's invalid-group test uses K=10, group 4
        assert mm(FAKE, FAKE, FAKE, FAKE, 2, 2, 10, gs, None) == pc.POPCORN_ERROR_INVALID_VALUE, gs
        assert qg(FAKE, FAKE, FAKE, 2, 10, gs, None) == pc.POPCORN_ERROR_INVALID_VALUE, gs
    assert mm(FAKE, FAKE, FAKE, FAKE, 2, 2, 10, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE


def test_int4_conventions(lib):
    # popcorn src/quantize.cu:418-433, :846-860: null -> invalid, sizes <= 0 ->
    # success, then group_size <= 0 or not dividing K -> invalid, then odd K
    # -> invalid (test/test_quantize.cu:628-670: K=9, group 3).
    mm = lib.popcornDequantizeMatmulGrouped_i4f32
    qg = lib.popcornQuantizeGrouped_f32i4
    for i in range(5):
        args = [FAKE] * 5
        args[i] = 0
        assert mm(*args, 1, 1, 8, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
    for i in range(4):
        args = [FAKE] * 4
        args[i] = 0
        assert qg(*args, 1, 8, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
    for (M, N, K) in [(0, 2, 8), (2, 0, 8), (2, 2, 0), (-1, 2, 8), (2, 2, -9)]:
        assert mm(FAKE, FAKE, FAKE, FAKE, FAKE, M, N, K, 3, None) == pc.POPCORN_SUCCESS
    assert qg(FAKE, FAKE, FAKE, FAKE, 0, 9, 3, None) == pc.POPCORN_SUCCESS
    assert qg(FAKE, FAKE, FAKE, FAKE, 2, 0, 3, None) == pc.POPCORN_SUCCESS
    for gs in (0, -4, 3, 16):
        assert mm(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 2, 10, gs, None) == pc.POPCORN_ERROR_INVALID_VALUE, gs
        assert qg(FAKE, FAKE, FAKE, FAKE, 2, 10, gs, None) == pc.POPCORN_ERROR_INVALID_VALUE, gs
    assert mm(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 2, 9, 3, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert qg(FAKE, FAKE, FAKE, FAKE, 2, 9, 3, None) == pc.POPCORN_ERROR_INVALID_VALUE


def test_fused_conventions(lib):
    # Every buffer but the RMSNorm weight must be non-null; sizes <= 0 are no-ops.
    norm = lib.popcornRMSNormDequantizeMatmul_i8f32
    glu = lib.popcornDequantizeMatmulSiluMul_i8f32
    both = lib.popcornRMSNormDequantizeMatmulSiluMul_i8f32
    for i in (0, 1, 3, 4):
        args = [FAKE] * 5
        args[i] = 0
        assert norm(args[0], args[1], args[2], 1e-5, args[3], args[4], 1, 4, 4, None) == \
            pc.POPCORN_ERROR_INVALID_VALUE, i
    for i in range(6):
        args = [FAKE] * 6
        args[i] = 0
        assert glu(*args, 1, 4, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
        assert both(args[0], args[1], FAKE, 1e-5, *args[2:], 1, 4, 4, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
    for (M, N, K) in [(0, 4, 4), (1, 0, 4), (1, 4, 0), (-1, 4, 4)]:
        assert norm(FAKE, FAKE, 0, 1e-5, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS
        assert glu(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS
        assert both(FAKE, FAKE, 0, 1e-5, FAKE, FAKE, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS


def test_batched_size_overflow_is_rejected(lib):
    big = 1 << 62
    assert lib.popcornDequantizeMatmulBatched_i8f32(FAKE, FAKE, FAKE, FAKE, big, 4, 1, 1, None) == \
        pc.POPCORN_ERROR_INVALID_VALUE


def test_path_selection_rules():
    a16 = 0x10000  # 16-byte aligned stand-in pointers
    # Decode shapes stay on the f32 CUDA-core path.
    assert pc.select_path(a16, a16, 1, 4096, 4096) == pc.PATH_SIMT_F32
    assert pc.select_path(a16, a16, 4, 4096, 4096) == pc.PATH_SIMT_F32
    # popcorn's own small test shapes stay on the f32 path (1e-5 absolute tolerance there).
    assert pc.select_path(a16, a16, 64, 256, 128) == pc.PATH_SIMT_F32
    # Unaligned pointers or K % 16 != 0 can never take the tensor path.
    assert pc.select_path(a16 + 4, a16, 2048, 4096, 4096) == pc.PATH_SIMT_F32
    assert pc.select_path(a16, a16 + 8, 2048, 4096, 4096) == pc.PATH_SIMT_F32
    assert pc.select_path(a16, a16, 2048, 4096, 4100) == pc.PATH_SIMT_F32
    assert pc.launch_count(a16, a16, 1, 4096, 4096) == 1


def test_nccl_layer_argument_checks(lib):
    # Checks that return before the communicator is used: null buffers (or a
    # null communicator) -> invalid, sizes <= 0 -> no-op, and a column-parallel
    # call with M > 1 needs its work buffer.
    col = lib.popcornDequantizeMatmulColumnParallel_i8f32
    row = lib.popcornDequantizeMatmulRowParallel_i8f32
    for i in range(5):
        args = [FAKE] * 5  # comm, out, x, qweight, scale
        args[i] = 0
        assert col(args[0], args[1], FAKE, *args[2:], 1, 8, 16, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
        assert row(*args, 1, 8, 16, None) == pc.POPCORN_ERROR_INVALID_VALUE, i
    for (M, N, K) in [(0, 8, 16), (1, 0, 16), (1, 8, 0), (-1, 8, 16)]:
        assert col(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS
        assert row(FAKE, FAKE, FAKE, FAKE, FAKE, M, N, K, None) == pc.POPCORN_SUCCESS
    assert col(FAKE, FAKE, 0, FAKE, FAKE, FAKE, 2, 8, 16, None) == pc.POPCORN_ERROR_INVALID_VALUE
    assert lib.popcornGetLastNcclError() == 0
