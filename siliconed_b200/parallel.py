"""Multi-GPU execution of the quantized linear: one process per GPU, torch.distributed for plumbing.

Two ways to spread the work (the reference has no multi-device code; these are new):

* Batch sharding (``batch_range``): every rank holds the whole weight and multiplies its own rows
  (its own images / token batches).  No collective on the data path; this is how ``bench.py``
  scales and how the denoise of independent images scales.
* Column-parallel linear (``ColumnParallelLinear``): rank r holds the columns ``column_ranges(N, P)[r]``
  of the weight (``sc_weight_create_shard``), computes ``y[:, n0:n1]``, and one all-gather over
  NVLink (NCCL) assembles ``y[M, N]``.  The gathered blocks arrive rank-major ([P, M, w]) and one
  copy puts the columns in place.

The local product is any callable ``(x, bias_shard) -> y_shard``: the library's ``QuantizedWeight.linear``
on GPUs; the CPU tests pass a stand-in so that the sharding and assembly logic runs under ``gloo``.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def column_ranges(n: int, world: int, align: int = 8) -> list[tuple[int, int]]:
    """Balanced [n0, n1) column blocks, boundaries on multiples of ``align`` (16-byte bf16 rows)
    except the end; blocks may be empty when n is small."""
    if n <= 0 or world <= 0:
        raise ValueError("n and world must be positive")
    units = -(-n // align)
    out = []
    for r in range(world):
        a = min(n, (r * units // world) * align)
        b = min(n, ((r + 1) * units // world) * align)
        out.append((a, b))
    return out


def batch_range(m: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [m0, m1) of rank ``rank`` when a batch of m rows is split across ``world`` ranks."""
    return (rank * m // world, (rank + 1) * m // world)


def gather_columns(y_local: torch.Tensor, ranges: Sequence[tuple[int, int]], group=None) -> torch.Tensor:
    """All-gathers the column blocks ``y_local`` [M, w_r] of every rank into y [M, N]."""
    world = len(ranges)
    m = y_local.shape[0]
    width = max(b - a for a, b in ranges)
    if y_local.shape[1] != width:  # pad to the common width (NCCL gathers equal sizes)
        pad = torch.zeros((m, width), dtype=y_local.dtype, device=y_local.device)
        pad[:, : y_local.shape[1]] = y_local
        y_local = pad
    blocks = torch.empty((world * m, width), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(blocks, y_local.contiguous(), group=group)
    blocks = blocks.view(world, m, width)
    n = ranges[-1][1]
    y = torch.empty((m, n), dtype=y_local.dtype, device=y_local.device)
    for r, (a, b) in enumerate(ranges):
        if b > a:
            y[:, a:b] = blocks[r, :, : b - a]
    return y


class ColumnParallelLinear:
    """A linear whose output columns are split over the ranks of ``group``.

    ``make_local(n0, n1)`` returns this rank's local product for columns [n0, n1): a callable
    ``(x, bias_shard) -> y_shard``.  On GPUs it registers the shard with
    ``QuantizedWeight(..., columns=(n0, n1))``.
    """

    def __init__(self, n: int, make_local: Callable[[int, int], Callable], group=None, align: int = 8):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n = n
        self.ranges = column_ranges(n, self.world, align)
        self.n0, self.n1 = self.ranges[self.rank]
        self.local = make_local(self.n0, self.n1) if self.n1 > self.n0 else None

    def __call__(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        if self.local is not None:
            b = None if bias is None else bias[self.n0:self.n1].contiguous()
            y_local = self.local(x, b)
        else:
            y_local = torch.empty((x.shape[0], 0), dtype=torch.bfloat16, device=x.device)
        return gather_columns(y_local, self.ranges, self.group)


def quantized_column_parallel(ctx, codes, kind: int, scales, n: int, *, published_nk: bool = False, group=None,
                              stream=None) -> ColumnParallelLinear:
    """A ColumnParallelLinear whose local product is libsiliconed_cuda's (one shard per rank)."""
    from .products import QuantizedWeight

    def make_local(n0, n1):
        w = QuantizedWeight(ctx, codes, kind, scales, published_nk=published_nk, columns=(n0, n1), stream=stream)

        def local(x, b):
            return w.linear(x, bias=b, stream=stream)

        local.weight = w
        return local

    return ColumnParallelLinear(n, make_local, group=group)
