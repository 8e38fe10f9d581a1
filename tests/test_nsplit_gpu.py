"""N-split NVFP4 linear on two GPUs (NCCL) against the unsplit FP4Linear on the same inputs:
the forward output is bit-identical (every slice is quantized with the full weight's global
scale); gradients agree to bf16 accumulation (dgrad partials are summed across ranks; each slice's
upstream gradient has its own global scale).  Skipped with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist
    import torch.nn.functional as F

    from radiance_b200 import _lib
    from radiance_b200.nvfp4 import FP4Linear, FP4Recipe
    from radiance_b200.nvfp4.nsplit import FP4ColumnParallelLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(0)
        m, k, n = 512, 512, 1024
        w = (torch.randn(n, k, generator=g) * 0.02).cuda()
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
        dy = (torch.randn(m, n, generator=g) * 1e-3).to(torch.bfloat16).cuda()
        # Round-to-nearest gradients: with stochastic rounding the split and unsplit layers draw
        # different random bits for dY and agree only in distribution.
        recipe = FP4Recipe(stochastic_rounding=False)
        full = FP4Linear(k, n, bias=False, recipe=recipe).cuda()
        with torch.no_grad():
            full.weight.copy_(w)
        full.refresh_fp4_cache()
        split = FP4ColumnParallelLinear(k, n, recipe=recipe, device="cuda")
        split.load_full_weight(w)
        split.refresh_fp4_cache()
        x1 = x.clone().requires_grad_(True)
        y1 = full(x1)
        gx1, gw1 = torch.autograd.grad(y1, (x1, full.weight), dy)
        x2 = x.clone().requires_grad_(True)
        y2 = split(x2)
        gx2, gw2 = torch.autograd.grad(y2, (x2, split.local.weight), dy)
        sl = slice(rank * (n // world), (rank + 1) * (n // world))

        def cos(a, b):
            return F.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0).item()

        cx, cw = cos(gx1, gx2), cos(gw1[sl], gw2)
        # The fused path: the slice's GEMM writes every rank's copy of the output over NVLink, into
        # IPC-shared plain device buffers (no multicast object).
        # Three output buffers: y3 stays alive while the two accumulation forwards below run.
        fused = FP4ColumnParallelLinear(k, n, recipe=recipe, device="cuda", fused_gather=True, output_buffers=3)
        fused.load_full_weight(w)
        fused.refresh_fp4_cache()
        x3 = x.clone().requires_grad_(True)
        y3 = fused(x3)
        same_fused = torch.equal(y1, y3)
        gx3, gw3 = torch.autograd.grad(y3, (x3, fused.local.weight), dy)
        # Two forwards, then one backward through both (gradient accumulation): the second forward
        # must not overwrite the first output, which is still alive.
        xa = x.clone().requires_grad_(True)
        xb = (x * 2).clone().requires_grad_(True)
        ya, yb = fused(xa), fused(xb)
        ya_ok = torch.equal(ya, y1) and torch.equal(yb, full(xb.detach()))
        ga, gb, gwab = torch.autograd.grad((ya * dy).float().sum() + (yb * dy).float().sum(),
                                           (xa, xb, fused.local.weight))
        xa2, xb2 = x.clone().requires_grad_(True), (x * 2).clone().requires_grad_(True)
        wref = full.weight
        ra, rb = full(xa2), full(xb2)
        ra2, rb2, gwref = torch.autograd.grad((ra * dy).float().sum() + (rb * dy).float().sum(), (xa2, xb2, wref))
        accum_ok = cos(ga, ra2) > 0.999 and cos(gb, rb2) > 0.999 and cos(gwab, gwref[sl]) > 0.999
        # One buffer only: a second forward while the first output is alive raises.
        single = FP4ColumnParallelLinear(k, n, recipe=recipe, device="cuda", fused_gather=True, output_buffers=1)
        single.load_full_weight(w)
        single.refresh_fp4_cache()
        keep = single(x)
        try:
            single(x)
            refused = False
        except RuntimeError as e:
            refused = "still referenced" in str(e)
        del keep
        again_ok = torch.equal(single(x), y1)  # the buffer is free again once released
        # The optimizer step fused with the refresh uses the full weight's global scale on a slice.
        upd = (torch.randn(n, k, generator=torch.Generator().manual_seed(1)) * 1e-3).cuda()
        full.apply_update_and_refresh_(upd, -0.5)
        split.apply_update_and_refresh_(upd[sl].contiguous(), -0.5)
        update_ok = (torch.equal(full._w_fwd_gs, split.local._w_fwd_gs)
                     and torch.equal(full._w_fwd_packed[sl], split.local._w_fwd_packed))
        results[rank] = (
            torch.equal(y1, y2),
            cx > 0.999,
            cw > 0.999,
            torch.equal(full._w_fwd_gs, split.local._w_fwd_gs),
            _lib.device_status() == 0,
            same_fused,
            torch.equal(gx2, gx3) and torch.equal(gw2, gw3),
            ya_ok and accum_ok,
            refused and again_ok,
            update_ok,
            f"dgrad cosine {cx:.6f}, wgrad cosine {cw:.6f}",
        )
        fused.close()
        single.close()
    finally:
        dist.destroy_process_group()


def test_nsplit_two_gpus_matches_unsplit():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    # Every wait in the workers is bounded (the process group's 60 s timeout ends any collective a
    # lost rank never joins), so they exit by themselves; nothing here kills a process that may
    # still have work on its GPU.
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert all(results[r][:10]), (r, results[r])
