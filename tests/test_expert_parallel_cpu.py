"""Expert-parallel dispatch / combine (``radiance_b200.nvfp4.expert_parallel``) on CPU with two and
four gloo ranks, against a single-process computation of the same routing.

Every rank routes its own tokens (uneven top-2 counts, one expert that receives no rows from one
source), owns ``E / g`` experts, and runs a stand-in expert (row times ``expert + 1``, in float64, so
every value is exact) on the padded expert-major layout the grouped NVFP4 linears consume.  Checked:
the split sizes and offsets, that padding rows arrive as zeros, that dispatch -> expert -> combine
returns every row to its source in its original order with the right expert applied, and that the
autograd backward of the round trip sends the gradients the reverse way (each input row's gradient
is the upstream gradient times its expert's factor)."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

E = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _routing(src: int, tokens: int = 100):
    """Source rank src's tokens: each routed to 2 distinct experts (top-2 of seeded logits)."""
    g = torch.Generator().manual_seed(100 + src)
    logits = torch.randn(tokens, E, generator=g)
    if src == 1:
        logits[:, 3] = -1e9  # expert 3 receives nothing from source 1
    top = logits.topk(2, dim=-1).indices
    return top


def _send_order(top):
    """(token, expert) pairs sorted expert-major: the order of a source's send buffer."""
    pairs = [(int(t), int(e)) for t in range(top.shape[0]) for e in top[t].tolist()]
    pairs.sort(key=lambda p: (p[1], p[0]))
    return pairs


def _worker(rank, world, port, results):
    import torch.distributed as dist

    from radiance_b200.nvfp4.expert_parallel import ExpertParallelPlan, combine, dispatch

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        tops = [_routing(s) for s in range(world)]
        counts = [torch.bincount(t.flatten(), minlength=E) for t in tops]
        plan = ExpertParallelPlan(counts, rank, world)
        d = 5
        g = torch.Generator().manual_seed(7 + rank)
        tokens = torch.randn(tops[rank].shape[0], d, generator=g, dtype=torch.float64)
        order = _send_order(tops[rank])
        x_send = torch.stack([tokens[t] for t, _ in order]).requires_grad_(True)
        x_exp = dispatch(x_send, plan)
        ok = [x_exp.shape == (plan.rows, d), plan.offsets[-1].item() == plan.rows,
              all(int(o) % 128 == 0 for o in plan.offsets.tolist())]
        # padding rows are zero
        pad = torch.ones(plan.rows, dtype=torch.bool)
        pad[plan.dst] = False
        ok.append(bool((x_exp.detach()[pad] == 0).all()))
        # the stand-in experts: group j (expert plan.experts[j]) scales its rows by expert + 1
        factor = torch.zeros(plan.rows, 1, dtype=torch.float64)
        offs = plan.offsets.tolist()
        for j, ex in enumerate(plan.experts):
            factor[offs[j]:offs[j + 1]] = ex + 1
        y_exp = x_exp * factor
        y_back = combine(y_exp, plan)
        want = torch.stack([tokens[t] * (e + 1) for t, e in order])
        ok.append(torch.equal(y_back.detach(), want))
        gy = torch.randn(y_back.shape, generator=g, dtype=torch.float64)
        (gx,) = torch.autograd.grad(y_back, (x_send,), gy)
        ok.append(torch.equal(gx, gy * torch.tensor([[e + 1.0] for _, e in order], dtype=torch.float64)))
        # split sizes: what rank r sends to d is what d receives from r
        sends = [None] * world
        dist.all_gather_object(sends, plan.send)
        recvs = [None] * world
        dist.all_gather_object(recvs, plan.recv)
        ok.append(all(sends[s][rank] == plan.recv[s] for s in range(world)))
        ok.append(sum(plan.expert_rows) == plan.routed == sum(plan.recv))
        results[rank] = ok
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_dispatch_combine_round_trip(world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert all(results[r]), (r, results[r])


def test_single_rank_plan_is_the_local_layout():
    from radiance_b200.nvfp4.expert_parallel import ExpertParallelPlan

    counts = [torch.tensor([3, 0, 130, 1, 0, 0, 5, 128])]
    plan = ExpertParallelPlan(counts, 0, 1)
    assert plan.send == plan.recv == [267]
    assert plan.offsets.tolist() == [0, 128, 128, 384, 512, 512, 512, 640, 768]
    x = torch.arange(267, dtype=torch.float64).view(-1, 1)
    y = plan.dispatch_rows(x)
    assert y.shape == (768, 1) and torch.equal(plan.combine_rows(y), x)
    with pytest.raises(ValueError, match="divide evenly"):
        ExpertParallelPlan([torch.ones(6, dtype=torch.int64)] * 4, 0, 4)
