"""N-split (column-parallel) NVFP4 linears across the GPUs of one box.

For the largest layers each rank owns ``out_features / g`` output rows of the weight and computes
its slice of the output for the (replicated) input; the bf16 slices are all-gathered over NVLink,
by NCCL or by the GEMM's own epilogue (``fused_gather``).  Backward: the upstream gradient's local columns feed the rank's dgrad and wgrad; the
partial input gradients are summed with an all-reduce, and each rank keeps the gradient of its own
weight rows.

Every slice is quantized with the *full* weight's global scale (an all-reduce(MAX) of the per-slice
scales: ``max(amax_r) / 2688`` rounds the same as each rank's own division because RN is monotone),
so a rank's cached operands are exactly the matching rows/columns of the unsplit layer's, and the
forward output equals the unsplit ``FP4Linear``'s bit for bit.  Backward does the same for the
upstream gradient's scale, so each rank's dY operands are the matching columns of the unsplit
layer's; dgrad differs from the unsplit layer's only by the bf16 rounding of the partial sums.
The collective logic is written against any local module (``ColumnParallel``), which is how it is
tested on CPU with gloo.  Without an initialised process group everything runs as one rank.
"""

from __future__ import annotations

import ctypes
import weakref

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import _lib
from . import _trace
from .linear import FP4Linear, FP4Recipe
from .quantize import _stream_ptr


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def _rank(group) -> int:
    return dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0


class _CopyToSplit(torch.autograd.Function):
    """Identity forward; all-reduce (sum) of the input gradient backward: the replicated input of a
    column-parallel layer receives one partial dgrad per rank."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        if _world(ctx.group) > 1:
            dist.all_reduce(grad, group=ctx.group)
        return grad, None


class _GatherColumns(torch.autograd.Function):
    """``(M, n)`` per rank -> ``(M, g * n)`` on every rank, rank r's slice at columns ``r*n ...``:
    one all-gather into a ``(g, M, n)`` buffer and a column permute.  Backward takes the local
    columns of the gradient (no communication)."""

    @staticmethod
    def forward(ctx, y, group):
        g = _world(group)
        ctx.group, ctx.g = group, g
        ctx.rank = _rank(group)
        y = y.contiguous()
        if g == 1:
            return y
        m, n = y.shape
        buf = torch.empty(g * m, n, dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(buf, y, group=group)
        return buf.view(g, m, n).permute(1, 0, 2).reshape(m, g * n)

    @staticmethod
    def backward(ctx, grad):
        if ctx.g == 1:
            return grad, None
        m, full = grad.shape
        n = full // ctx.g
        # A row-strided view: the quantizers read it in place (16-byte aligned rows, n % 128 == 0).
        return grad.reshape(m, ctx.g, n)[:, ctx.rank, :], None


class _FusedGathered(torch.autograd.Function):
    """The fused path's gather: the slice's GEMM already wrote every rank's copy of the full
    output (``buf``), so forward just hands that buffer out; backward takes the local columns of
    the gradient, as ``_GatherColumns`` does."""

    @staticmethod
    def forward(ctx, y_local, buf, g, rank):
        ctx.g, ctx.rank = g, rank
        return buf.detach()

    @staticmethod
    def backward(ctx, grad):
        m, full = grad.shape
        n = full // ctx.g
        return grad.reshape(m, ctx.g, n)[:, ctx.rank, :], None, None, None


class _CudaArray:
    """``__cuda_array_interface__`` over a raw device allocation, so ``torch.as_tensor`` can wrap
    it without a copy (the tensor keeps this object, and with it the allocation, alive)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str, owner):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None, "stream": None}
        self._owner = owner


class PeerOutput:
    """One full-width output buffer per rank, mapped into every other rank of the group by CUDA IPC
    (``rb_peer_alloc`` / ``rb_peer_handle`` / ``rb_peer_open``): plain device memory, no NVLink
    multicast object.  ``tensor`` is this rank's copy; ``peer_ptrs[p]`` the address of rank p's copy
    in this process (None for this rank).  Creating one is collective over the group (the handles
    travel by ``all_gather_object``); it cannot happen during stream capture."""

    _TYPESTR = {torch.bfloat16: "<i2", torch.float32: "<f4"}

    def __init__(self, rows: int, cols: int, dtype: torch.dtype, device: torch.device, group, world: int, rank: int):
        lib = _lib.load()
        esize = torch.empty((), dtype=dtype).element_size()
        nbytes = rows * cols * esize
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            _lib.check(lib.rb_peer_alloc(nbytes, ctypes.byref(ptr)), "nsplit peer buffer")
            self.ptr = ptr.value
            handle = ctypes.create_string_buffer(_lib.RB_PEER_HANDLE_BYTES)
            _lib.check(lib.rb_peer_handle(self.ptr, handle), "nsplit peer buffer")
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
            self.peer_ptrs = []
            for p in range(world):
                if p == rank:
                    self.peer_ptrs.append(None)
                    continue
                q = ctypes.c_void_p()
                _lib.check(lib.rb_peer_open(handles[p], ctypes.byref(q)), "nsplit peer buffer")
                self.peer_ptrs.append(q.value)
        # bf16 has no array-interface type code: wrap as 16-bit integers, then view as bf16.
        raw = torch.as_tensor(_CudaArray(self.ptr, (rows, cols), self._TYPESTR[dtype], self), device=device)
        self.tensor = raw.view(dtype) if dtype == torch.bfloat16 else raw
        self.handed_out = None  # weak reference to the last output view given to a caller

    def close(self, group) -> None:
        """Collective: unmap the peers' buffers, wait for every rank to do the same, free this one."""
        lib = _lib.load()
        for q in self.peer_ptrs:
            if q is not None:
                lib.rb_peer_close(q)
        self.peer_ptrs = []
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.tensor = None
        lib.rb_peer_free(self.ptr)
        self.ptr = None


def copy_to_split(x: torch.Tensor, group=None) -> torch.Tensor:
    return _CopyToSplit.apply(x, group)


def gather_split_columns(y: torch.Tensor, group=None) -> torch.Tensor:
    return _GatherColumns.apply(y, group)


class ColumnParallel(nn.Module):
    """Wraps a local ``in -> out/g`` module as the rank's slice of an ``in -> out`` layer:
    ``forward(x) = all_gather_columns(local(x))`` with the input-gradient all-reduce."""

    def __init__(self, local: nn.Module, group=None):
        super().__init__()
        self.local = local
        self.group = group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y = self.local(copy_to_split(x.reshape(-1, x.shape[-1]), self.group))
        return gather_split_columns(y, self.group).view(*lead, -1)


class FP4ColumnParallelLinear(ColumnParallel):
    """``FP4Linear(in_features, out_features)`` split along ``out_features`` over the ranks of
    ``group``: rank r holds rows ``r * out/g : (r + 1) * out/g`` of the weight (``out/g`` a multiple
    of 128).  ``load_full_weight`` takes the unsplit ``(out, in)`` weight and keeps this rank's rows.

    ``fused_gather=True`` replaces the NCCL all-gather with the GEMM's own epilogue: the slice's
    GEMM (``rb_nvfp4_gemm_allgather``) stores every output tile into all ranks' copies of a
    full-width output buffer over NVLink, so the gather overlaps the multiplication and needs no
    staging buffer or column permute.  The buffers are plain device allocations shared by CUDA IPC
    (``PeerOutput``; no multicast object), and the ranks order their use with two one-element NCCL
    all-reduces on the stream (before the GEMM: every rank is done with the buffer's previous
    contents; after it: every rank's tiles are in every copy), so a lost rank ends in the process
    group's timeout, not in an unbounded device wait.

    The returned output *is* one of ``output_buffers`` such buffers, used in turn: it stays valid
    while the caller holds it.  A forward that would reuse a buffer whose earlier output is still
    referenced (gradient accumulation or recomputation with more live outputs than buffers) raises
    instead of overwriting it."""

    def __init__(self, in_features: int, out_features: int, group=None, recipe: FP4Recipe | None = None,
                 device=None, dtype=None, fused_gather: bool = False, output_buffers: int = 2):
        g = _world(group)
        if out_features % (128 * g):
            raise ValueError(f"FP4ColumnParallelLinear: out_features {out_features} must split into multiples of "
                             f"128 over {g} ranks")
        super().__init__(FP4Linear(in_features, out_features // g, bias=False, recipe=recipe, device=device,
                                   dtype=dtype), group)
        self.in_features, self.out_features, self.world = in_features, out_features, g
        self.rank = _rank(group)
        # The upstream gradient is the full dY on every rank (the gather's backward slices it), so
        # every slice quantizes its columns with the full gradient's scale too.
        self.local.reduce_grad_scale = self.full_weight_scale_
        self.fused_gather = fused_gather and self.world > 1
        self.output_buffers = max(1, int(output_buffers))
        self._peer: dict = {}
        self._turn: dict = {}
        self._current = None
        if self.fused_gather:
            self.local.output_gemm = self._gemm_into_all_ranks

    def _ranks_barrier(self, device: torch.device) -> None:
        """Stream-ordered barrier over the group: a one-element NCCL all-reduce on the current
        stream completes on a rank only after every rank's earlier stream work has completed."""
        t = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(t, group=self.group)

    def _next_output(self, rows: int, dtype: torch.dtype, device: torch.device) -> PeerOutput:
        key = (rows, dtype)
        pool = self._peer.setdefault(key, [])
        turn = self._turn.get(key, 0)
        self._turn[key] = (turn + 1) % self.output_buffers
        if turn == len(pool):
            pool.append(PeerOutput(rows, self.out_features, dtype, device, self.group, self.world, self.rank))
        buf = pool[turn]
        if buf.handed_out is not None and buf.handed_out() is not None:
            raise RuntimeError(
                "FP4ColumnParallelLinear(fused_gather=True): the output of an earlier forward that used this "
                f"layer's output buffer {turn} is still referenced; with {self.output_buffers} buffers at most "
                f"{self.output_buffers} outputs may be alive at once (raise output_buffers, release the earlier "
                "output, or use fused_gather=False)")
        return buf

    def _gemm_into_all_ranks(self, xq, wq, bias, out_dtype):
        """The slice's forward GEMM writing its columns into every rank's full-width buffer."""
        if out_dtype not in (torch.bfloat16, torch.float32) or bias is not None:
            raise ValueError("FP4ColumnParallelLinear(fused_gather=True) supports bf16/fp32 outputs without bias")
        m = xq.packed.shape[0]
        n, k = wq.packed.shape[0], xq.packed.shape[1] * 2
        dev = xq.packed.device
        out = self._next_output(m, out_dtype, dev)
        buf = out.tensor
        esize = buf.element_size()
        col0 = self.rank * n
        peers = [q + col0 * esize for q in out.peer_ptrs if q is not None]
        arr = (ctypes.c_void_p * len(peers))(*peers)
        lib = _lib.load()
        self._ranks_barrier(dev)  # every rank is done with the buffer's previous contents
        tok = _trace.begin("gemm", 2.0 * m * n * k)
        _lib.check(
            lib.rb_nvfp4_gemm_allgather(
                xq.packed.data_ptr(), xq.scale.data_ptr(), wq.packed.data_ptr(), wq.scale.data_ptr(), m, n, k,
                xq.global_scale.data_ptr(), wq.global_scale.data_ptr(), None, 0, buf[:, col0:].data_ptr(),
                _lib.RB_OUT_BF16 if out_dtype == torch.bfloat16 else _lib.RB_OUT_F32, self.out_features, arr,
                len(peers), _stream_ptr(dev),
            ),
            "nvfp4.gemm_allgather",
        )
        _trace.end(tok)
        self._ranks_barrier(dev)  # every rank's tiles are in every copy
        self._current = out
        return buf[:, col0:col0 + n]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.fused_gather:
            return super().forward(x)
        lead = x.shape[:-1]
        y_local = self.local(copy_to_split(x.reshape(-1, x.shape[-1]), self.group))
        cur = self._current
        out = _FusedGathered.apply(y_local, cur.tensor, self.world, self.rank)
        cur.handed_out = weakref.ref(out)
        return out.view(*lead, -1)

    def close(self) -> None:
        """Collective: release the fused gather's peer buffers (every rank must call it)."""
        for pool in self._peer.values():
            for buf in pool:
                buf.close(self.group)
        self._peer.clear()
        self._current = None

    @torch.no_grad()
    def load_full_weight(self, weight: torch.Tensor) -> None:
        n = self.out_features // self.world
        self.local.weight.copy_(weight[self.rank * n:(self.rank + 1) * n])
        self.local.invalidate_fp4_cache()

    def full_weight_scale_(self, gs: torch.Tensor) -> torch.Tensor:
        """In place: the slice's global scale -> the full weight's (all-reduce MAX over the ranks)."""
        if self.world > 1:
            dist.all_reduce(gs, op=dist.ReduceOp.MAX, group=self.group)
        return gs

    def refresh_fp4_cache(self) -> None:
        self.local.refresh_fp4_cache(reduce_global_scale=self.full_weight_scale_)

    @torch.no_grad()
    def apply_update_and_refresh_(self, update: torch.Tensor, alpha: float) -> None:
        """``FP4Linear.apply_update_and_refresh_`` for this rank's slice (``update``: the slice's rows),
        with the slice's new global scale reduced to the full weight's before the quantization, as
        ``refresh_fp4_cache`` does."""
        self.local.apply_update_and_refresh_(update, alpha, reduce_global_scale=self.full_weight_scale_)
