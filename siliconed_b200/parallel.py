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


class FusedColumnParallelLinear:
    """The column-parallel linear with the all-gather fused into the product (``sc_linear_allgather``).

    Rank r registers its columns [n0, n1) and, every call, multiplies the whole x by them; the product's
    epilogue stores each output tile into every rank's y over NVLink (peer pointers opened once with
    CUDA IPC) and raises an epoch flag on every rank; ``sc_allgather_wait`` holds the stream until all
    ranks' columns have landed.  y is double-buffered (a rank may start call e + 1 while another still
    reads call e's result): the returned tensor stays valid until the call after next.  Set-up is
    collective (every rank of ``group`` constructs it); so is every call, with the same x shape.
    """

    def __init__(self, ctx, codes, kind: int, scales, n: int, m_max: int, *, published_nk: bool = False,
                 bias=None, group=None, stream=None, multicast: bool = True):
        import ctypes
        from . import abi
        from .products import QuantizedWeight
        self.ctx, self.group = ctx, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.n = n
        self.ranges = column_ranges(n, self.world, 8)
        self.n0, self.n1 = self.ranges[self.rank]
        if self.n1 <= self.n0:
            raise ValueError("every rank needs columns")
        self.w = QuantizedWeight(ctx, codes, kind, scales, published_nk=published_nk, columns=(self.n0, self.n1),
                                 stream=stream)
        self.bias = None if bias is None else bias[self.n0:self.n1].contiguous()
        dev = torch.device("cuda", ctx.device)
        self.m_max = m_max
        # The outputs in symmetric memory bound to an NVLink multicast object when the system has one
        # (torch's symmetric memory; one multimem store reaches every rank), else in ordinary device memory
        # whose peers open it through CUDA IPC.
        self.mc = [0, 0]
        self._symm = None
        if multicast:
            self._try_multicast(dev, m_max, n)
        if self._symm is None:
            self.y = [torch.empty((m_max, n), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=dev)
        self.ws = torch.empty(max(self.w.workspace_bytes(max(m_max, 1536)), 256), dtype=torch.uint8, device=dev)
        lib = ctx.lib
        mine = []
        for i, t in enumerate((self.y[0], self.y[1], self.flags)):
            if i < 2 and self._symm is not None:     # symmetric memory: no IPC handle needed (nor possible)
                mine.append((b"", 0))
                continue
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_size_t()
            ctx.check(lib.sc_ipc_handle(ctx.ptr, ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off)))
            mine.append((bytes(h), int(off.value)))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = []  # (pointer, offset) to close
        self.peer_y = [[0] * self.world for _ in range(2)]
        self.peer_flags = [0] * self.world
        for r, handles in enumerate(everyone):
            ptrs = []
            for i, ((h, off), t) in enumerate(zip(handles, (self.y[0], self.y[1], self.flags))):
                if r == self.rank:
                    ptrs.append(t.data_ptr())
                    continue
                if i < 2 and self._symm is not None:   # symmetric memory: the peers' addresses are known
                    ptrs.append(int(self._symm[1].buffer_ptrs[r]) + i * self.y[0].numel() * 2)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                ctx.check(lib.sc_ipc_open(ctx.ptr, buf, off, ctypes.byref(p)))
                self._opened.append((p.value, off))
                ptrs.append(p.value)
            self.peer_y[0][r], self.peer_y[1][r], self.peer_flags[r] = ptrs
        self._y_arr = [(ctypes.c_void_p * self.world)(*self.peer_y[i]) for i in range(2)]
        self._f_arr = (ctypes.c_void_p * self.world)(*self.peer_flags)
        self.epoch = 0
        dist.barrier(group=group)

    def _try_multicast(self, dev, m_max: int, n: int) -> None:
        try:
            import torch.distributed._symmetric_memory as symm
            t = symm.empty((2, m_max, n), dtype=torch.bfloat16, device=dev)
            h = symm.rendezvous(t, self.group if self.group is not None else dist.group.WORLD)
            ok = bool(h.has_multicast_support(symm.DeviceType.CUDA, dev.index)) and int(h.multicast_ptr) != 0
        except Exception:  # no symmetric memory or no multicast here: the IPC path
            ok, t, h = False, None, None
        flags = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN, group=self.group)   # every rank takes the same path
        if int(flags.item()) == 1:
            self._symm = (t, h)
            self.y = [t[0], t[1]]
            self.mc = [int(h.multicast_ptr), int(h.multicast_ptr) + m_max * n * 2]

    @property
    def uses_multicast(self) -> bool:
        return self._symm is not None

    def __call__(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        import ctypes
        m = x.shape[0]
        if m > self.m_max or x.shape[1] != self.w.k:
            raise ValueError(f"x must be [<= {self.m_max}, {self.w.k}]")
        self.epoch += 1
        buf = self.epoch % 2
        lib, ctx = self.ctx.lib, self.ctx
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream if stream is None else stream.cuda_stream)
        b = None if self.bias is None else ctypes.c_void_p(self.bias.data_ptr())
        ctx.check(lib.sc_linear_allgather_mc(ctx.ptr, self.w.ptr, ctypes.c_void_p(x.data_ptr()), m, b,
                                             ctypes.c_void_p(self.mc[buf]), self._y_arr[buf], self._f_arr, self.world,
                                             self.rank, self.n0, self.n, self.epoch,
                                             ctypes.c_void_p(self.ws.data_ptr()), self.ws.numel(), st))
        ctx.check(lib.sc_allgather_wait(ctx.ptr, ctypes.c_void_p(self.flags.data_ptr()), self.world, self.epoch, st))
        return self.y[buf][:m]

    def close(self) -> None:
        import ctypes
        torch.cuda.synchronize()
        for p, off in self._opened:
            self.ctx.lib.sc_ipc_close(self.ctx.ptr, ctypes.c_void_p(p), off)
        self._opened = []
        self.y = None
        self._symm = None
        self.w.close()
