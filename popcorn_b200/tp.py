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

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import dequantize_matmul

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
