"""N-split (column-parallel) host logic on CPU with two gloo ranks: the all-gather of output
columns, the local gradient slice, the input-gradient all-reduce, weight slicing and the
full-weight global scale.  The GEMM itself is the GPU's; here the local layer is an fp32
``nn.Linear`` so the collective logic is checked exactly."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist
    import torch.nn as nn

    from radiance_b200.nvfp4.nsplit import ColumnParallel, FP4ColumnParallelLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        m, k, n = 6, 8, 12
        w_full = torch.randn(n, k, dtype=torch.float64)
        x = torch.randn(m, k, dtype=torch.float64, requires_grad=True)
        dy = torch.randn(m, n, dtype=torch.float64)
        local = nn.Linear(k, n // world, bias=False).double()
        with torch.no_grad():
            local.weight.copy_(w_full[rank * (n // world):(rank + 1) * (n // world)])
        layer = ColumnParallel(local)
        y = layer(x)
        y.backward(dy)
        ok_y = torch.allclose(y, x.detach() @ w_full.T)
        ok_dx = torch.allclose(x.grad, dy @ w_full)
        sl = slice(rank * (n // world), (rank + 1) * (n // world))
        ok_dw = torch.allclose(local.weight.grad, dy[:, sl].T @ x.detach())
        # FP4 wrapper: slicing of a full weight and the full-weight global scale (CPU buffers only)
        fp4 = FP4ColumnParallelLinear(16, 128 * world)
        wf = torch.randn(128 * world, 16)
        fp4.load_full_weight(wf)
        ok_slice = torch.equal(fp4.local.weight.detach(), wf[rank * 128:(rank + 1) * 128])
        gs = torch.tensor(float(rank + 1) * 0.5)
        fp4.full_weight_scale_(gs)
        ok_gs = gs.item() == 0.5 * world
        results[rank] = (ok_y, ok_dx, ok_dw, ok_slice, ok_gs, not fp4.local._cache_valid)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_column_parallel_collectives(world):
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


def test_split_shape_contract():
    from radiance_b200.nvfp4.nsplit import FP4ColumnParallelLinear

    with pytest.raises(ValueError, match="multiples of 128"):
        FP4ColumnParallelLinear(64, 100)
    layer = FP4ColumnParallelLinear(64, 256)  # no process group: one rank holds everything
    assert layer.world == 1 and layer.local.out_features == 256
    assert np.isfinite(layer.local.weight.detach().numpy()).all()
