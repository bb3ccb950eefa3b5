"""Tensor-parallel int8 linear layers over torch.distributed (NCCL on B200s).

popcorn itself is single-GPU; this module is the multi-GPU layer above its C
ABI. One process per GPU, weights sharded once at set-up, each step one call
of the library per rank plus one collective:

* :class:`ColumnParallelLinear` -- output channels (rows of qweight) split
  across ranks. Every rank computes y[:, rows of its shard] with
  popcornDequantizeMatmul_i8f32 on a replicated x, then an all-gather of the
  shards rebuilds the full y on every rank.
* :class:`RowParallelLinear` -- input channels (columns of qweight) split
  across ranks. Every rank multiplies its slice of x by its column slice of
  qweight (re-packed contiguous once at set-up) and an all-reduce(sum) adds
  the partial outputs. The summation order across ranks differs from a
  single-GPU call, so results agree to f32 rounding, not bit for bit.

Shard boundaries are balanced: rank r owns [floor(n*r/P), floor(n*(r+1)/P)).
Shards of unequal size are padded to the largest for the all-gather.

The per-rank matmul is a parameter (``local_matmul``) so the host-side logic
can be exercised on CPU ranks with any reference implementation; the default
is the library's C ABI on the current CUDA stream.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import TP_MAX_RANKS, TpGroup, dequantize_matmul, load_library, PopcornError, POPCORN_SUCCESS

LocalMatmul = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Balanced contiguous shard [lo, hi) of n items for `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return (n * rank) // world, (n * (rank + 1)) // world


def _default_matmul(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return dequantize_matmul(x, q, s)


class ColumnParallelLinear:
    """y[M, N] = x[M, K] @ (qweight[N, K] * scale[N]).T, N split across ranks."""

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                 local_matmul: Optional[LocalMatmul] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = qweight.shape
        lo, hi = shard_bounds(self.N, self.world, self.rank)
        self.lo, self.hi = lo, hi
        self.q = qweight[lo:hi].contiguous()
        self.s = scale[lo:hi].contiguous()
        self.width = max(shard_bounds(self.N, self.world, r)[1] - shard_bounds(self.N, self.world, r)[0]
                         for r in range(self.world))
        self.matmul = local_matmul or _default_matmul

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        M = x.shape[0]
        y_local = self.matmul(x, self.q, self.s)                      # [M, n_r]
        if self.world == 1:
            return y_local
        n_r = self.hi - self.lo
        send = y_local if n_r == self.width else torch.nn.functional.pad(y_local, (0, self.width - n_r))
        send = send.contiguous()
        flat = torch.empty((self.world * M, self.width), dtype=send.dtype, device=send.device)
        dist.all_gather_into_tensor(flat, send, group=self.group)
        gathered = flat.view(self.world, M, self.width)
        parts = []
        for r in range(self.world):
            a, b = shard_bounds(self.N, self.world, r)
            parts.append(gathered[r, :, : b - a])
        return torch.cat(parts, dim=1)                                  # [M, N]


class RowParallelLinear:
    """y[M, N] = x[M, K] @ (qweight[N, K] * scale[N]).T, K split across ranks.

    The caller passes the full x (replicated) or only its slice via
    ``x_is_sharded``; the weights' column slice is copied once at set-up.
    """

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                 local_matmul: Optional[LocalMatmul] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = qweight.shape
        lo, hi = shard_bounds(self.K, self.world, self.rank)
        self.lo, self.hi = lo, hi
        self.q = qweight[:, lo:hi].contiguous()
        self.s = scale.contiguous()
        self.matmul = local_matmul or _default_matmul

    def __call__(self, x: torch.Tensor, x_is_sharded: bool = False) -> torch.Tensor:
        xs = x if x_is_sharded else x[:, self.lo:self.hi]
        y = self.matmul(xs.contiguous(), self.q, self.s)               # partial [M, N]
        if self.world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y


class PeerGroup:
    """Receive areas and call state of the fused decode collectives.

    Allocates, on every rank of ``group``, a zero-filled receive area in torch
    symmetric memory (peer-mapped over NVLink) large enough for an all-reduce
    of [max_m, max_n] outputs (which also covers an all-gather of that size),
    plus the rank's two-word call state, and fills the popcornTpGroup_t the C
    entry points take. One group serves any number of layers; every rank must
    make the same calls in the same order, each rank on one stream.
    """

    def __init__(self, max_m: int, max_n: int, device: torch.device, group: Optional[dist.ProcessGroup] = None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > TP_MAX_RANKS:
            raise ValueError(f"at most {TP_MAX_RANKS} ranks")
        self.max_m, self.max_n = max_m, max_n
        recv_bytes = 16 * self.world * max_m * max_n
        self.recv = symm_mem.empty((recv_bytes // 8,), dtype=torch.int64, device=device)
        self.recv.zero_()
        self.state = torch.zeros((2,), dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        handle = symm_mem.rendezvous(self.recv, self.group.group_name)
        g = TpGroup()
        for p in range(self.world):
            g.recv[p] = handle.buffer_ptrs[p]
        g.recv_bytes = recv_bytes
        g.state = self.state.data_ptr()
        g.rank, g.world = self.rank, self.world
        self.tp_group = g
        self._handle = handle
        dist.barrier(group=self.group)  # every rank's receive area is zero before any call

    def all_gather(self, out: torch.Tensor, x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, n_offset: int,
                   stream_handle: int) -> int:
        """out [M, N] <- all ranks' shards; q [n_local, K] is this rank's. Returns popcornStatus_t."""
        M, N = out.shape
        return load_library().popcornDequantizeMatmulAllGather_i8f32(
            ctypes.byref(self.tp_group), out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(), M, n_offset,
            q.shape[0], N, q.shape[1], stream_handle)

    def all_reduce(self, out: torch.Tensor, x: torch.Tensor, q: torch.Tensor, s: torch.Tensor,
                   stream_handle: int) -> int:
        """out [M, N] <- sum over ranks of x_r @ (q_r * s).T; x [M, K_r], q [N, K_r]. Returns popcornStatus_t."""
        M, N = out.shape
        return load_library().popcornDequantizeMatmulAllReduce_i8f32(
            ctypes.byref(self.tp_group), out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(), M, N,
            q.shape[1], stream_handle)


class NcclComm:
    """An NCCL communicator of its own over the ranks of ``group``, for the C
    entry points of include/popcorn_tp_nccl.h (which take an ncclComm_t, as a
    cgo caller holding its own communicator would pass). Rank 0's unique id
    travels through torch.distributed; ncclCommInitRank runs on ``device``.
    Uses the libnccl.so.2 already loaded in the process (torch's)."""

    class _UniqueId(ctypes.Structure):
        _fields_ = [("internal", ctypes.c_ubyte * 128)]

    def __init__(self, device: torch.device, group: Optional[dist.ProcessGroup] = None):
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        nccl = ctypes.CDLL("libnccl.so.2")
        nccl.ncclGetUniqueId.argtypes = [ctypes.POINTER(self._UniqueId)]
        nccl.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, self._UniqueId,
                                          ctypes.c_int]
        nccl.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        uid = self._UniqueId()
        if self.rank == 0 and nccl.ncclGetUniqueId(ctypes.byref(uid)) != 0:
            raise RuntimeError("ncclGetUniqueId failed")
        # all 128 bytes (a c_char array would stop at the first zero byte)
        box = [ctypes.string_at(ctypes.addressof(uid), 128) if self.rank == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(self.group, 0), group=self.group)
        ctypes.memmove(ctypes.addressof(uid), box[0], 128)
        self.comm = ctypes.c_void_p()
        with torch.cuda.device(device):
            rc = nccl.ncclCommInitRank(ctypes.byref(self.comm), self.world, uid, self.rank)
        if rc != 0:
            raise RuntimeError(f"ncclCommInitRank failed: {rc}")
        self._nccl = nccl

    def destroy(self) -> None:
        if self.comm:
            self._nccl.ncclCommDestroy(self.comm)
            self.comm = ctypes.c_void_p()

    def column_parallel(self, out: torch.Tensor, work: Optional[torch.Tensor], x: torch.Tensor, q: torch.Tensor,
                        s: torch.Tensor) -> None:
        """out [M, N] <- the full column-parallel output; q [N / P, K] is this rank's shard."""
        M, N = out.shape
        st = load_library().popcornDequantizeMatmulColumnParallel_i8f32(
            self.comm, out.data_ptr(), None if work is None else work.data_ptr(), x.data_ptr(), q.data_ptr(),
            s.data_ptr(), M, N, q.shape[1], torch.cuda.current_stream().cuda_stream)
        if st != POPCORN_SUCCESS:
            raise PopcornError(st, "popcornDequantizeMatmulColumnParallel_i8f32")

    def row_parallel(self, out: torch.Tensor, x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
        """out [M, N] <- sum over ranks of x_r @ (q_r * s).T; x [M, K_r], q [N, K_r]."""
        M, N = out.shape
        st = load_library().popcornDequantizeMatmulRowParallel_i8f32(
            self.comm, out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(), M, N, q.shape[1],
            torch.cuda.current_stream().cuda_stream)
        if st != POPCORN_SUCCESS:
            raise PopcornError(st, "popcornDequantizeMatmulRowParallel_i8f32")


class FusedColumnParallelLinear:
    """Column-parallel decode layer whose all-gather is fused into the GEMV.

    Each rank's kernel (popcornDequantizeMatmulAllGather_i8f32) computes its
    output channels and sends them to every other rank over NVLink; it
    finishes only when the other ranks' channels have arrived, so no
    collective call follows. Decode shapes only (M <= 4). The gathered result
    equals a single-GPU call bit for bit.
    """

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, peer: PeerGroup):
        self.N, self.K = qweight.shape
        self.peer = peer
        lo, hi = shard_bounds(self.N, peer.world, peer.rank)
        self.lo, self.hi = lo, hi
        self.q = qweight[lo:hi].contiguous()
        self.s = scale[lo:hi].contiguous()

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty((x.shape[0], self.N), dtype=torch.float32, device=x.device)
        st = self.peer.all_gather(out, x, self.q, self.s, self.lo, torch.cuda.current_stream().cuda_stream)
        if st != POPCORN_SUCCESS:
            raise PopcornError(st, "popcornDequantizeMatmulAllGather_i8f32")
        return out


class FusedRowParallelLinear:
    """Row-parallel decode layer whose all-reduce is fused into the GEMV.

    Input channels are split across ranks as in :class:`RowParallelLinear`;
    each rank's kernel (popcornDequantizeMatmulAllReduce_i8f32) sends its
    partial outputs to every rank and sums all ranks' partials in rank order,
    so every rank holds the same bits. Decode shapes only (M <= 4).
    """

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, peer: PeerGroup):
        self.N, self.K = qweight.shape
        self.peer = peer
        lo, hi = shard_bounds(self.K, peer.world, peer.rank)
        self.lo, self.hi = lo, hi
        self.q = qweight[:, lo:hi].contiguous()
        self.s = scale.contiguous()

    def __call__(self, x: torch.Tensor, x_is_sharded: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        xs = (x if x_is_sharded else x[:, self.lo:self.hi]).contiguous()
        if out is None:
            out = torch.empty((x.shape[0], self.N), dtype=torch.float32, device=x.device)
        st = self.peer.all_reduce(out, xs, self.q, self.s, torch.cuda.current_stream().cuda_stream)
        if st != POPCORN_SUCCESS:
            raise PopcornError(st, "popcornDequantizeMatmulAllReduce_i8f32")
        return out


# ---------------------------------------------------------------------------
# 7B-shaped linear stack (tensor-parallel, Megatron-style placement)
# ---------------------------------------------------------------------------
STACK_7B = {"hidden": 4096, "qkv": 12288, "ffn": 11008}
STACK_PARTS = ("qkv", "o", "gate", "up", "down")


def stack_part_shape(dims: dict, part: str) -> tuple[int, int]:
    """[N, K] of the full weight of one projection of a layer."""
    h = dims["hidden"]
    return {"qkv": (dims["qkv"], h), "o": (h, h), "gate": (dims["ffn"], h), "up": (dims["ffn"], h),
            "down": (h, dims["ffn"])}[part]


def shard_stack_layer(full: dict, rank: int, world: int) -> dict:
    """This rank's shards of one layer given its full (qweight, scale) pairs.

    qkv, gate and up are column-parallel (rows of qweight split); o and down
    are row-parallel (columns of qweight split, re-packed contiguous, the
    whole per-channel scale kept).
    """
    out = {}
    for part, (q, s) in full.items():
        if part in ("o", "down"):
            lo, hi = shard_bounds(q.shape[1], world, rank)
            out[part] = (q[:, lo:hi].contiguous(), s.contiguous())
        else:
            lo, hi = shard_bounds(q.shape[0], world, rank)
            out[part] = (q[lo:hi].contiguous(), s[lo:hi].contiguous())
    return out


def peer_fusable(M: int, K: int) -> bool:
    """Whether the fused decode collectives take these sizes (popcorn_tp.h)."""
    limit = {1: 16384, 2: 8192, 3: 4096, 4: 4096}.get(M, 0)
    return K % 16 == 0 and 0 < K <= limit


class LinearStack:
    """The linear layers of a decoder stack, tensor-parallel over `group`.

    Per layer: h -> qkv (column-parallel) -> o (row-parallel, all-reduce) ->
    gate and up (column-parallel; at M <= 4 one call over the rank's gate
    rows stacked on its up rows) -> down (row-parallel, all-reduce) -> h.
    Attention and the SiLU(gate) * up product lie outside the dequant-matmul
    path; in their place the o projection reads the first columns of the
    rank's qkv output and the down projection reads the rank's gate output,
    so every weight byte of every layer is streamed once per pass and every
    collective of a Megatron-style stack happens, with nothing else between
    the calls. Column-parallel outputs stay sharded (no all-gather). (The
    fused popcornDequantizeMatmulSiluMul_i8f32 was measured slower than the
    two plain calls at both M = 1 and M = 128, so the stack keeps them apart.)

    Row-parallel sums use the fused popcornDequantizeMatmulAllReduce_i8f32
    when a PeerGroup is given and M <= 4, else the library call followed by an
    NCCL all-reduce. All buffers are allocated here, so a pass can be captured
    in a CUDA graph. ``local_matmul`` (x, q, s) -> y replaces the library call
    (for host-side tests on CPU ranks, with torch.distributed all-reduce).

    Each layer dict gains a "gate_up" entry (the rank's gate and up shards
    concatenated by rows) and its "gate" and "up" entries become views of
    it, so at decode sizes the two projections stream as one matrix in one
    launch (at M = 128 two launches measured faster: 3.33 against 3.40 ms
    per pass, the merged 22016-row GEMM taking a second wave of CTA pairs).
    """

    def __init__(self, layers: list, M: int, dims: dict, device, group: Optional[dist.ProcessGroup] = None,
                 peer: Optional[PeerGroup] = None, local_matmul: Optional[LocalMatmul] = None):
        self.layers = layers
        self.M = M
        self.dims = dims
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.local_matmul = local_matmul
        h = dims["hidden"]
        ko = shard_bounds(h, self.world, self.rank)
        self.k_o = ko[1] - ko[0]
        k_down = layers[0]["down"][0].shape[1]
        fusable = self.world > 1 and peer_fusable(M, self.k_o) and peer_fusable(M, k_down)
        self.peer = peer if (peer is not None and fusable) else None
        n_qkv = layers[0]["qkv"][0].shape[0]
        n_ffn = layers[0]["gate"][0].shape[0]
        for w in layers:
            if "gate_up" not in w:
                qg, sg = w["gate"]
                qu, su = w["up"]
                q = torch.cat([qg, qu])
                sc = torch.cat([sg, su])
                w["gate_up"] = (q, sc)
                w["gate"] = (q[:n_ffn], sc[:n_ffn])
                w["up"] = (q[n_ffn:], sc[n_ffn:])
        if n_qkv < self.k_o:
            raise ValueError("qkv shard narrower than the o projection's input slice")
        f32 = torch.float32
        self.a = torch.empty((M, n_qkv), dtype=f32, device=device)
        self.xo = torch.empty((M, self.k_o), dtype=f32, device=device)
        self.h1 = torch.empty((M, h), dtype=f32, device=device)
        self.n_ffn = n_ffn
        self.merged = M <= 4
        self.gu = torch.empty((M, 2 * n_ffn), dtype=f32, device=device) if self.merged else None
        self.g = torch.empty((M, n_ffn), dtype=f32, device=device)
        self.u = None if self.merged else torch.empty((M, n_ffn), dtype=f32, device=device)
        self.h2 = torch.empty((M, h), dtype=f32, device=device)
        self._lib = None if local_matmul is not None else load_library()

    def _mm(self, out: torch.Tensor, x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
        if self.local_matmul is not None:
            out.copy_(self.local_matmul(x, q, s))
            return
        st = self._lib.popcornDequantizeMatmul_i8f32(out.data_ptr(), x.data_ptr(), q.data_ptr(), s.data_ptr(),
                                                     out.shape[0], q.shape[0], q.shape[1],
                                                     torch.cuda.current_stream().cuda_stream)
        if st != POPCORN_SUCCESS:
            raise PopcornError(st, "popcornDequantizeMatmul_i8f32")

    def _row(self, out: torch.Tensor, x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
        if self.peer is not None:
            st = self.peer.all_reduce(out, x, q, s, torch.cuda.current_stream().cuda_stream)
            if st != POPCORN_SUCCESS:
                raise PopcornError(st, "popcornDequantizeMatmulAllReduce_i8f32")
            return
        self._mm(out, x, q, s)
        if self.world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """One pass over every layer; returns the last layer's output buffer."""
        h = x
        for i, w in enumerate(self.layers):
            self._mm(self.a, h, *w["qkv"])
            if self.M == 1:
                xo = self.a[:, : self.k_o]                 # contiguous for a single row
            else:
                self.xo.copy_(self.a[:, : self.k_o])
                xo = self.xo
            self._row(self.h1, xo, *w["o"])
            if self.merged:
                self._mm(self.gu, self.h1, *w["gate_up"])
                if self.M == 1:
                    g = self.gu[:, : self.n_ffn]           # contiguous for a single row
                else:
                    self.g.copy_(self.gu[:, : self.n_ffn])
                    g = self.g
            else:
                self._mm(self.g, self.h1, *w["gate"])
                self._mm(self.u, self.h1, *w["up"])
                g = self.g
            self._row(self.h2, g, *w["down"])
            h = self.h2
        return h

    __call__ = forward

    def weight_bytes(self) -> int:
        """int8 weight bytes this rank streams per pass."""
        return sum(w[part][0].numel() for w in self.layers for part in STACK_PARTS)

    def launches_per_pass(self) -> int:
        """Library kernel launches per pass (NCCL and copies not counted)."""
        if self._lib is None:
            return 0
        n = 0
        M = self.M
        parts = ("qkv", "o", "gate_up", "down") if self.merged else STACK_PARTS
        for w in self.layers:
            for part in parts:
                q = w[part][0]
                n += self._lib.popcornDequantizeMatmulLaunchCount(0x10000, q.data_ptr(), M, q.shape[0],
                                                                  q.shape[1], 0)
        return n
