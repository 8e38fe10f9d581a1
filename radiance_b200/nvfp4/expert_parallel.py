"""Expert parallelism for the grouped NVFP4 expert linears: each rank owns ``E / g`` experts, and the
rows routed to an expert travel to its owner and back with all-to-alls.

radiance runs its experts on one GPU (``BatchedExperts``, src/radiance/model/ffn.py:148-153, one
``torch.baddbmm`` over ``(experts, capacity, d)``) and has no multi-GPU code; this module is the
exchange step of the expert-partitioned layout, with the routed rows in the stacked, expert-sorted
layout that ``FP4GroupedLinear`` multiplies (groups padded to 128 rows).

The plan is static: every rank knows every rank's routing counts (``counts[s][e]``, the rows of
source rank ``s`` routed to expert ``e``), so the all-to-all split sizes and the row maps are built
once on the host and the exchange itself never synchronises the host.  A source's send buffer holds
its routed rows sorted by expert (expert-major); rows arrive at an owner source-major, and one row
gather turns them into the owner's expert-major layout with zero rows as the 128-row padding.  The
reverse direction (the combine, and both directions' gradients) is the same pair of operations
mirrored: a gather and an all-to-all.  The collective calls go through ``torch.distributed``, so
the logic runs unchanged on gloo (CPU tests) and NCCL (the GPUs).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .grouped import align_offsets


class ExpertParallelPlan:
    """Split sizes and row maps of the expert-parallel exchange for one rank.

    ``counts``: one length-``E`` integer tensor per source rank (``E`` divisible by the world
    size).  Attributes:
      * ``experts``: this rank's experts; ``send[d]`` / ``recv[s]``: rows sent to rank d / received
        from rank s;
      * ``offsets``: the expert-major group offsets (int64, ``len(experts) + 1``, 128-aligned) of
        the received rows, for ``FP4GroupedLinear``; ``rows``: the padded row count;
      * ``dst[i]``: the padded expert-major row of received row i; ``src[p]``: the received row of
        padded row p, or ``routed`` (one zero row appended after the received rows) for padding.
    """

    def __init__(self, counts, rank: int, world: int, device=None, align: int = 128):
        counts = [torch.as_tensor(c, dtype=torch.int64).cpu() for c in counts]
        if len(counts) != world:
            raise ValueError(f"ExpertParallelPlan: {len(counts)} routing count vectors for {world} ranks")
        e = counts[0].numel()
        if e % world:
            raise ValueError(f"ExpertParallelPlan: {e} experts do not divide evenly over {world} ranks")
        per = e // world
        self.rank, self.world, self.per = rank, world, per
        self.experts = list(range(rank * per, (rank + 1) * per))
        self.send = [int(counts[rank][d * per:(d + 1) * per].sum()) for d in range(world)]
        self.recv = [int(counts[s][self.experts].sum()) for s in range(world)]
        exp_counts = torch.stack([counts[s][self.experts] for s in range(world)]).sum(0)
        offsets = align_offsets(exp_counts, align)
        self.rows = int(offsets[-1])
        self.routed = int(exp_counts.sum())
        fill = [int(o) for o in offsets[:-1].tolist()]
        dst = []
        for s in range(world):  # received rows: source-major, each source's rows expert-major
            for j, ex in enumerate(self.experts):
                n = int(counts[s][ex])
                dst.extend(range(fill[j], fill[j] + n))
                fill[j] += n
        src = torch.full((self.rows,), self.routed, dtype=torch.int64)
        dst_t = torch.tensor(dst, dtype=torch.int64)
        src[dst_t] = torch.arange(self.routed, dtype=torch.int64)
        self.offsets = offsets.to(device)
        self.dst = dst_t.to(device)
        self.src = src.to(device)
        self.expert_rows = exp_counts.tolist()

    # -- the two exchanges (no autograd) --------------------------------------------------------
    def _a2a(self, t: torch.Tensor, out_split, in_split, group) -> torch.Tensor:
        if self.world == 1:
            return t
        out = torch.empty(sum(out_split), *t.shape[1:], dtype=t.dtype, device=t.device)
        dist.all_to_all_single(out, t.contiguous(), out_split, in_split, group=group)
        return out

    def dispatch_rows(self, x_send: torch.Tensor, group=None) -> torch.Tensor:
        """Rows this rank routes (expert-major, ``sum(send)`` rows) -> the padded expert-major rows
        of this rank's experts (``rows`` rows; padding rows are zero)."""
        recv = self._a2a(x_send, self.recv, self.send, group)
        ext = torch.cat([recv, recv.new_zeros(1, *recv.shape[1:])])
        return ext.index_select(0, self.src)

    def combine_rows(self, y_exp: torch.Tensor, group=None) -> torch.Tensor:
        """The experts' padded expert-major output rows -> this rank's routed rows, in the order
        they were dispatched (the inverse of ``dispatch_rows``; padding rows are dropped)."""
        return self._a2a(y_exp.index_select(0, self.dst), self.send, self.recv, group)


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_send, plan, group):
        ctx.plan, ctx.group = plan, group
        return plan.dispatch_rows(x_send, group)

    @staticmethod
    def backward(ctx, grad):
        return ctx.plan.combine_rows(grad, ctx.group), None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_exp, plan, group):
        ctx.plan, ctx.group = plan, group
        return plan.combine_rows(y_exp, group)

    @staticmethod
    def backward(ctx, grad):
        return ctx.plan.dispatch_rows(grad, ctx.group), None, None


def dispatch(x_send: torch.Tensor, plan: ExpertParallelPlan, group=None) -> torch.Tensor:
    """Differentiable ``plan.dispatch_rows``: its backward returns the gradient rows to their sources."""
    return _Dispatch.apply(x_send, plan, group)


def combine(y_exp: torch.Tensor, plan: ExpertParallelPlan, group=None) -> torch.Tensor:
    """Differentiable ``plan.combine_rows``: its backward sends the gradient rows to the experts."""
    return _Combine.apply(y_exp, plan, group)
