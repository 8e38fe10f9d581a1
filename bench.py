"""Benchmark of the NVFP4 linear path (BASELINE metric: NVFP4 linear fwd+bwd TFLOPS).

Workload: one dense transformer block's linears -- QKV 2048->6144,
O 2048->2048, gate/up 2048->11264, down 5632->2048 -- forward + dgrad + wgrad through
``radiance_b200.nvfp4.FP4Linear`` with the default recipe (stochastic rounding and Hadamard on,
packed activation saving on), 16384 tokens per GPU, weights ~N(0, 0.02), activations ~N(0, 1),
upstream gradients ~N(0, 1e-3).  A step = one micro-batch forward + backward of the four linears.
Token rows shard across ranks with no data-path collective (weak scaling: every rank runs its own
16384-token micro-batch; the data-parallel gradient all-reduce belongs to the optimizer, not to
this path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU implementation of
the path (the NumPy restatement of radiance's pure-torch NVFP4 emulation in ``oracle/``) on the
host cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

D_MODEL = 2048
TOKENS_PER_GPU = 16384
LAYERS = [("qkv", 2048, 6144), ("o", 2048, 2048), ("gate_up", 2048, 11264), ("down", 5632, 2048)]
STEP_FLOPS = 6.0 * TOKENS_PER_GPU * sum(k * n for _, k, n in LAYERS)  # 5.051e12
METRIC = "NVFP4 linear fwd+bwd TFLOPS (BASELINE config 3 block linears, 16384 tokens/GPU)"

# Average DRAM bytes (read + write) per GEMM launch of this workload's twelve GEMMs, from one `ncu`
# capture (profiles/gemm_block_step_traffic.md).
GEMM_DRAM_BYTES_PER_LAUNCH = 130318549


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------------------------------------------
# nvidia-smi clock sampling during the timed region
# --------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------------------------------------------------
# The GPU arm
# --------------------------------------------------------------------------------------------------
def _dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def _make_layers(device, seed):
    import torch

    from radiance_b200 import nvfp4 as nv

    g = torch.Generator(device="cpu").manual_seed(seed)
    layers, xs, dys = [], [], []
    for name, k, n in LAYERS:
        lin = nv.FP4Linear(k, n, bias=False, recipe=nv.FP4Recipe())
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
        lin = lin.to(device)
        lin.refresh_fp4_cache()
        layers.append(lin)
        xs.append((torch.randn(TOKENS_PER_GPU, k, generator=g)).to(torch.bfloat16))
        dys.append((torch.randn(TOKENS_PER_GPU, n, generator=g) * 1e-3).to(torch.bfloat16))
    return layers, xs, dys


def _step(layers, xs, dys, outs=None):
    import torch

    for i, lin in enumerate(layers):
        x = xs[i].detach().requires_grad_(True)
        y = lin(x)
        gx, gw = torch.autograd.grad(y, (x, lin.weight), dys[i])
        if outs is not None:
            outs.append((gx, gw))


def run_ours(args):
    import torch
    import torch.distributed as dist

    from radiance_b200.nvfp4 import _trace

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    layers, xs_host, dys_host = _make_layers(device, seed=1234 + rank)
    xs = [x.to(device) for x in xs_host]
    dys = [d.to(device) for d in dys_host]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing (value) ------------------------------------------------------
    for _ in range(args.warmup):
        _step(layers, xs, dys)
    torch.cuda.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    barrier()
    torch.cuda.synchronize()
    # The step is captured once in a CUDA graph and replayed: every kernel of the step runs on every
    # replay; the graph removes the host's per-launch overhead, which with eight processes sharing
    # the host's cores leaves gaps between kernels.  --eager times the Python loop instead.
    run_step = (lambda: _step(layers, xs, dys))
    graph = None
    if not args.eager:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                _step(layers, xs, dys)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            _step(layers, xs, dys)
        torch.cuda.synchronize()
        run_step = graph.replay
    clocks.start()
    for _ in range(20):  # keep the GPU loaded while the sampler starts up (untimed)
        run_step()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(args.steps):
        run_step()
    stop.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(stop)
    ms_max = max_over_ranks(ms)
    # Per-kernel breakdown (the roofline's live timing): the same steps again, eagerly, with CUDA
    # events around every launch.  Not part of `value`.
    kt_steps = max(3, min(args.steps, 50))
    with _trace.kernel_timer() as kt:
        for _ in range(kt_steps):
            _step(layers, xs, dys)
        torch.cuda.synchronize()
    per_kind = {k: {kk: (int(round(vv * args.steps / kt_steps)) if kk == "launches" else vv * args.steps / kt_steps)
                    for kk, vv in v.items()} for k, v in kt.summary().items()}
    launches = kt.launches * args.steps // kt_steps

    # ---- with the data-parallel weight-gradient reduction (N > 1) -----------------------------
    # Token sharding needs no collective on the fwd/dgrad path, but wgrad contracts over tokens:
    # a data-parallel job sums each linear's fp32 dW across ranks.  Measured separately, the way
    # DDP overlaps it (one async all-reduce per linear, issued as its dW is produced).
    dp = None
    if world > 1:
        def step_allreduce():
            works = []
            for i, lin in enumerate(layers):
                x = xs[i].detach().requires_grad_(True)
                y = lin(x)
                _gx, gw = torch.autograd.grad(y, (x, lin.weight), dys[i])
                works.append(dist.all_reduce(gw, async_op=True))
            for w in works:
                w.wait()

        dp_steps = max(3, min(args.steps, 50))
        for _ in range(3):
            step_allreduce()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ds, de = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ds.record()
        for _ in range(dp_steps):
            step_allreduce()
        de.record()
        torch.cuda.synchronize()
        dp_ms = max_over_ranks(ds.elapsed_time(de)) / dp_steps
        dp_bytes = sum(lin.weight.numel() * 4 for lin in layers)
        dp = {"value": round(world * STEP_FLOPS / (dp_ms * 1e-3) / 1e12, 2), "unit": "TFLOPS",
              "ms_per_step": round(dp_ms, 4), "allreduce_bytes_per_step": dp_bytes,
              "what": "same step plus an async NCCL all-reduce of each linear's fp32 dW (overlapped)"}

    # ---- end-to-end through the public API with host buffers (e2e) --------------------------
    pinned_x = [x.pin_memory() for x in xs_host]
    pinned_dy = [d.pin_memory() for d in dys_host]
    dev_x = [torch.empty_like(x, device=device) for x in xs_host]
    dev_dy = [torch.empty_like(d, device=device) for d in dys_host]
    result_host = torch.empty(D_MODEL, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned_x + pinned_dy)
    d2h = result_host.numel() * result_host.element_size()

    # Two sets of device inputs: while step s computes on one set, the copy stream uploads step
    # s+1's inputs into the other (the way a data loader feeds a training loop), so a step costs
    # the larger of its host-to-device copy and its compute.
    dev_sets = [(dev_x, dev_dy), ([torch.empty_like(x, device=device) for x in xs_host],
                                  [torch.empty_like(d, device=device) for d in dys_host])]
    copy_stream = torch.cuda.Stream(device)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    used = [False, False]

    def issue_copy(b):
        with torch.cuda.stream(copy_stream):
            if used[b]:
                copy_stream.wait_event(consumed[b])
            for i in range(len(layers)):
                dev_sets[b][0][i].copy_(pinned_x[i], non_blocking=True)
                dev_sets[b][1][i].copy_(pinned_dy[i], non_blocking=True)
            copied[b].record(copy_stream)

    def e2e_run(n):
        copy_stream.wait_stream(torch.cuda.current_stream())  # the first copy starts inside the timing
        issue_copy(0)
        for s_ in range(n):
            b = s_ % 2
            if s_ + 1 < n:
                issue_copy(1 - b)
            torch.cuda.current_stream().wait_event(copied[b])
            outs = []
            _step(layers, dev_sets[b][0], dev_sets[b][1], outs)
            consumed[b].record()
            used[b] = True
            result_host.copy_(outs[0][1][0], non_blocking=True)  # first row of dW(qkv)

    e2e_steps = max(3, min(args.steps, 20))
    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    e2e_run(e2e_steps)
    ee.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(es.elapsed_time(ee)) / e2e_steps

    if rank == 0:
        peaks, peak_kind = _peaks()
        ms_step = ms_max / args.steps
        value = world * STEP_FLOPS / (ms_step * 1e-3) / 1e12
        gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0, "work": 0.0})
        quant = per_kind.get("quantize", {"launches": 0, "ms": 0.0, "work": 0.0})
        amax = per_kind.get("amax", {"launches": 0, "ms": 0.0, "work": 0.0})
        fp4_peak = 4.0 * peaks["bf16_tflops"]
        gemm_ms_launch = gemm["ms"] / max(gemm["launches"], 1)
        gemm_tflops = gemm["work"] / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else None
        traffic = GEMM_DRAM_BYTES_PER_LAUNCH
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
            "data": "synthetic (seeded; W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
            "config": {
                "workload": "config3: dense block linears fwd+dgrad+wgrad via FP4Linear",
                "d_model": D_MODEL,
                "layers": {n: [k, o] for n, k, o in LAYERS},
                "tokens_per_gpu": TOKENS_PER_GPU,
                "global_batch_tokens": TOKENS_PER_GPU * world,
                "recipe": "grad_gemms, stochastic_rounding, hadamard, save_activations",
                "parallelism": f"token-sharded dp{world} (no data-path collective)",
                "l2": "inputs larger than L2 (about 1 GB of activations and gradients per step)",
                "timing": "eager Python step loop" if args.eager else
                          "the step captured in one CUDA graph, replayed K times (per-kernel times from an eager pass)",
            },
            "tokens_per_s": round(world * TOKENS_PER_GPU / (ms_step * 1e-3), 1),
            "gpu_launches": launches,
            "kernels": {
                "gemm": {"launches": gemm["launches"], "ms": round(gemm["ms"], 3),
                         "TFLOPS": None if gemm_tflops is None else round(gemm_tflops, 1)},
                "quantize": {"launches": quant["launches"], "ms": round(quant["ms"], 3),
                             "GBps": round(quant["work"] / (quant["ms"] * 1e-3) / 1e9, 1) if quant["ms"] else None},
                "amax": {"launches": amax["launches"], "ms": round(amax["ms"], 3),
                         "GBps": round(amax["work"] / (amax["ms"] * 1e-3) / 1e9, 1) if amax["ms"] else None},
            },
            "roofline": {
                "kernel": "nvfp4_gemm2_kernel (tcgen05 cta_group::2 block-scaled GEMM)",
                "bound": "tensor",
                "achieved": None if gemm_tflops is None else round(gemm_tflops, 1),
                "peak": round(fp4_peak, 1),
                "peak_basis": f"4 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s): B200 NVFP4 dense rate is 4x bf16; nominal 9000",
                "unit": "TFLOP/s",
                "frac": None if gemm_tflops is None else round(gemm_tflops / fp4_peak, 4),
                "traffic": traffic,
                "flops_per_launch": round(gemm["work"] / max(gemm["launches"], 1)),
                "ms_per_launch": round(gemm_ms_launch, 4),
            },
            "e2e": {
                "value": round(world * STEP_FLOPS / (e2e_ms * 1e-3) / 1e12, 2),
                "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3),
                "path": "FP4Linear forward/backward (public API), inputs copied from pinned host memory each step "
                        "(step s+1's copies overlap step s's compute on a second stream)",
            },
            "clocks": clk,
        }
        if dp is not None:
            line["with_dp_grad_allreduce"] = dp
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    del graph, run_step
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------------------
# The CPU arm (the reference's algorithm: quantize -> dequantize -> fp32 matmul emulation)
# --------------------------------------------------------------------------------------------------
def _cpu_linear_step(O, np, w_row, w_col, tokens, rng):
    """One FP4 linear forward + dgrad + wgrad on the CPU oracle (O-projection shape 2048 -> 2048),
    following radiance's _FP4LinearFn (linear.py:63-155) with the default recipe."""
    k = n = D_MODEL
    x = O.bf16_to_f32(O.f32_to_bf16_bits(rng.standard_normal((tokens, k), dtype=np.float32)))
    dy = O.bf16_to_f32(O.f32_to_bf16_bits(rng.standard_normal((tokens, n), dtype=np.float32) * 1e-3))
    had = O.hadamard_matrix()
    gx = O.global_scale_of(x)
    xp, xs = O.quantize_rowblock(x, gx)
    xtp, xts = O.quantize_colblock(x, gx, hadamard=had)
    (wp, ws, gw) = w_row
    y = O.dequantize(xp, xs, gx) @ O.dequantize(wp, ws, gw).T
    gg = O.global_scale_of(dy)
    u = rng.random(dy.shape, dtype=np.float32)
    gp, gsc = O.quantize_rowblock(dy, gg, u=u)
    gtp, gts = O.quantize_colblock(dy, gg, hadamard=had, u=u)
    (wcp, wcs, gwc) = w_col
    dx = O.dequantize(gp, gsc, gg) @ O.dequantize(wcp, wcs, gwc).T
    dw = O.dequantize(gtp, gts, gg) @ O.dequantize(xtp, xts, gx).T
    return y, dx, dw


def _cpu_setup():
    import numpy as np

    from oracle import nvfp4_oracle as O

    rng = np.random.default_rng(0)
    w = O.bf16_to_f32(O.f32_to_bf16_bits(rng.standard_normal((D_MODEL, D_MODEL), dtype=np.float32) * 0.02))
    gw = O.global_scale_of(w)
    wp, ws = O.quantize_rowblock(w, gw)
    wcp, wcs = O.quantize_colblock(w, gw)
    return O, np, (wp, ws, gw), (wcp, wcs, gw), rng


def cpu_baseline(budget_s: float = 15.0) -> dict:
    O, np, w_row, w_col, rng = _cpu_setup()
    tokens = 512
    t0 = time.perf_counter()
    done = 0
    while time.perf_counter() - t0 < budget_s or done == 0:
        _cpu_linear_step(O, np, w_row, w_col, tokens, rng)
        done += 1
    dt = (time.perf_counter() - t0) / done
    flops = 6.0 * tokens * D_MODEL * D_MODEL
    return {
        "value": round(flops / dt / 1e12, 6),
        "unit": "TFLOPS",
        "cores": os.cpu_count(),
        "kind": "port",
        "sample": f"{done} x one 2048->2048 linear fwd+dgrad+wgrad on {tokens} tokens (oracle restatement of "
                  f"radiance's CPU emulation; numpy, BLAS matmuls on all cores), {dt:.2f} s each",
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    O, np, w_row, w_col, rng = _cpu_setup()
    # Size one step so warmup + steps fit in about two minutes.
    t0 = time.perf_counter()
    _cpu_linear_step(O, np, w_row, w_col, 16, rng)
    per16 = time.perf_counter() - t0
    budget = 120.0 / max(args.steps + args.warmup, 1)
    tokens = int(max(16, min(2048, (budget / max(per16, 1e-3)) * 16)) // 16 * 16)
    for _ in range(args.warmup):
        _cpu_linear_step(O, np, w_row, w_col, tokens, rng)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_linear_step(O, np, w_row, w_col, tokens, rng)
    dt = (time.perf_counter() - t0) / args.steps
    flops = 6.0 * tokens * D_MODEL * D_MODEL
    value = flops / dt / 1e12
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 6),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "nvfp4 emulated in fp32 (quantize -> dequantize -> matmul)",
        "data": "synthetic (seeded)",
        "config": {"workload": "config3 block linears, sampled: one 2048->2048 linear fwd+dgrad+wgrad",
                   "tokens_per_step": tokens, "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {
            "value": round(value, 6),
            "unit": "TFLOPS",
            "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"one 2048->2048 FP4 linear fwd+dgrad+wgrad on {tokens} tokens per step (recipe: SR + Hadamard)",
        },
        "e2e": {"value": round(value, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------------
# Config 4: MoE expert FFN (grouped NVFP4 GEMMs), experts partitioned across ranks
# --------------------------------------------------------------------------------------------------
C4_D, C4_E, C4_FFN, C4_TOKENS, C4_TOPK = 2048, 8, 1408, 16384, 2
C4_FLOPS = 6.0 * C4_TOKENS * C4_TOPK * (C4_D * 2 * C4_FFN + C4_FFN * C4_D)  # 1.701e12 per rank
C4_METRIC = "NVFP4 MoE expert linears fwd+bwd TFLOPS (BASELINE config 4: 8 experts, top-2, 16384 tokens/GPU)"


def _c4_counts(src_rank: int):
    """Tokens of source rank s routed to each expert: router logits ~N(0,1) (seed s), softmax, top-2."""
    import torch

    g = torch.Generator().manual_seed(src_rank)
    logits = torch.randn(C4_TOKENS, C4_E, generator=g)
    top = logits.softmax(-1).topk(C4_TOPK, dim=-1).indices
    return torch.bincount(top.flatten(), minlength=C4_E)


def run_config4(args):
    """One step = the expert FFN's two grouped linears (gate+up fused 2048->2816, down 1408->2048),
    forward + dgrad + wgrad, on the rows this rank's experts receive.  With N ranks each rank owns
    E/N experts and routes its own 16384 tokens; the routed rows travel to their expert's owner and
    back with NCCL all-to-alls (dispatch before gate/up, combine after down, and the reverse pair for
    the gradients), inside the timed region.  Work per rank is fixed as N grows (weak scaling)."""
    import torch
    import torch.distributed as dist

    from radiance_b200.nvfp4 import _trace
    from radiance_b200.nvfp4.grouped import FP4GroupedLinear, align_offsets

    rank, world, local = _dist_setup(args)
    if C4_E % world:
        raise SystemExit(f"config 4 needs the {C4_E} experts to divide evenly over {world} ranks")
    device = torch.device("cuda", local if world > 1 else 0)
    per = C4_E // world
    mine = list(range(rank * per, (rank + 1) * per))
    counts = [_c4_counts(s) for s in range(world)]  # every rank knows every rank's routing (seeded)
    send = [int(counts[rank][d * per:(d + 1) * per].sum()) for d in range(world)]
    recv = [int(counts[s][mine].sum()) for s in range(world)]
    # Received rows arrive source-major (each source's rows sorted by expert); the experts need them
    # expert-major and padded to 128-row groups: a fixed gather index, built once.
    exp_counts = torch.stack([counts[s][mine] for s in range(world)]).sum(0)
    offsets = align_offsets(exp_counts).to(device)
    t_pad = int(offsets[-1])
    dst = []
    fill = [int(o) for o in offsets[:-1].tolist()]
    for s in range(world):
        for j, e in enumerate(mine):
            n = int(counts[s][e])
            dst.extend(range(fill[j], fill[j] + n))
            fill[j] += n
    routed = int(exp_counts.sum())
    # The inverse map, for gathers: padded expert-major row p takes received row src[p], or the
    # zero row appended after the received rows when p is padding.
    src = torch.full((t_pad,), routed, dtype=torch.int64)
    src[torch.tensor(dst, dtype=torch.int64)] = torch.arange(routed, dtype=torch.int64)
    src = src.to(device)
    dst = torch.tensor(dst, dtype=torch.int64, device=device)
    flops = 6.0 * routed * (C4_D * 2 * C4_FFN + C4_FFN * C4_D)

    torch.manual_seed(100 + rank)
    gate_up = FP4GroupedLinear(per, C4_D, 2 * C4_FFN, device=device)
    down = FP4GroupedLinear(per, C4_FFN, C4_D, device=device)
    gate_up.refresh_fp4_cache()
    down.refresh_fp4_cache()
    x_send_ext = torch.zeros(sum(send) + 1, C4_D, device=device, dtype=torch.bfloat16)
    x_send = x_send_ext[:sum(send)]
    x_send.copy_(torch.randn(sum(send), C4_D, device=device).to(torch.bfloat16))
    h_in = torch.zeros(t_pad, C4_FFN, device=device, dtype=torch.bfloat16)
    h_in[dst] = torch.randn(routed, C4_FFN, device=device).to(torch.bfloat16)
    dy_gu = torch.zeros(t_pad, 2 * C4_FFN, device=device, dtype=torch.bfloat16)
    dy_gu[dst] = (torch.randn(routed, 2 * C4_FFN, device=device) * 1e-3).to(torch.bfloat16)
    dy_send_ext = torch.zeros(sum(send) + 1, C4_D, device=device, dtype=torch.bfloat16)
    dy_send = dy_send_ext[:sum(send)]
    dy_send.copy_((torch.randn(sum(send), C4_D, device=device) * 1e-3).to(torch.bfloat16))

    def a2a(t, out_rows, out_split, in_split, out=None):
        if world == 1:
            if out is not None:
                out.copy_(t)
                return out
            return t
        if out is None:
            out = torch.empty(out_rows, t.shape[1], device=device, dtype=t.dtype)
        dist.all_to_all_single(out, t, out_split, in_split)
        return out

    # Received rows plus one zero row (the source of the padding rows in the expert-major gathers).
    # On one GPU the received rows are the rank's own, already in place.
    xr_ext = x_send_ext if world == 1 else torch.zeros(routed + 1, C4_D, device=device, dtype=torch.bfloat16)
    dyr_ext = dy_send_ext if world == 1 else torch.zeros(routed + 1, C4_D, device=device, dtype=torch.bfloat16)

    def step():
        # dispatch: routed rows -> their experts' owner, then expert-major with zero padding (one
        # row gather)
        if world > 1:
            a2a(x_send, sum(recv), recv, send, out=xr_ext[:routed])
        x_exp = xr_ext.index_select(0, src)
        x_exp.requires_grad_(True)
        y_gu = gate_up(x_exp, offsets)
        h = h_in.detach().requires_grad_(True)  # silu(gate) * up of y_gu, synthetic here
        y_d = down(h, offsets)
        a2a(y_d[dst], sum(send), send, recv)  # combine: outputs back to the tokens' ranks
        if world > 1:  # gradients of the combined outputs
            a2a(dy_send, sum(recv), recv, send, out=dyr_ext[:routed])
        dy_d = dyr_ext.index_select(0, src)
        torch.autograd.grad(y_d, (h, down.weight), dy_d)
        gx, _gw = torch.autograd.grad(y_gu, (x_exp, gate_up.weight), dy_gu)
        a2a(gx[dst], sum(send), send, recv)  # input gradients back to the tokens' ranks

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    # On one GPU the step (no collectives; routing offsets stay on the device) is captured once in a
    # CUDA graph and replayed, as in config 3; with several ranks it runs eagerly around NCCL.
    run_step = step
    graph = None
    if world == 1 and not args.eager:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        run_step = graph.replay
    clocks.start()
    for _ in range(20):
        run_step()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(args.steps):
        run_step()
    stop.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(stop)) / args.steps
    # Per-kernel breakdown: the same steps again, eagerly, with CUDA events around every launch.
    kt_steps = max(3, min(args.steps, 50))
    with _trace.kernel_timer() as kt:
        for _ in range(kt_steps):
            step()
        torch.cuda.synchronize()
    per_kind = {k: {kk: (int(round(vv * args.steps / kt_steps)) if kk == "launches" else vv * args.steps / kt_steps)
                    for kk, vv in v.items()} for k, v in kt.summary().items()}
    timing_mode = ("the step captured in one CUDA graph, replayed K times (per-kernel times from an eager pass)"
                   if graph is not None else "eager Python step loop around NCCL (per-kernel times from a second pass)")
    if graph is not None:
        del graph
    if rank == 0:
        peaks, peak_kind = _peaks()
        fp4_peak = 4.0 * peaks["bf16_tflops"]
        gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0})
        gemm_ms = gemm["ms"] / args.steps
        gemm_tflops = flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
        line = {
            "metric": C4_METRIC,
            "value": round(world * C4_FLOPS / (ms * 1e-3) / 1e12, 2),
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
            "data": "synthetic (seeded; router logits ~N(0,1), W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
            "config": {
                "workload": "config4: MoE expert FFN linears (gate+up 2048->2816, down 1408->2048) fwd+dgrad+wgrad "
                            "via FP4GroupedLinear",
                "experts": C4_E, "experts_per_rank": per, "top_k": C4_TOPK, "tokens_per_gpu": C4_TOKENS,
                "routed_rows_rank0": routed, "padded_rows_rank0": t_pad,
                "rank0_expert_rows": exp_counts.tolist(),
                "parallelism": f"expert-parallel ep{world} (NCCL all-to-all dispatch/combine)" if world > 1
                else "single GPU, all experts",
                "flops_basis": "6 x routed rows x (2048 x 2816 + 1408 x 2048); padding rows are overhead",
                "timing": timing_mode,
            },
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3)} for k, v in per_kind.items()},
            "roofline": {
                "kernel": "nvfp4_gemm2_kernel (grouped)",
                "bound": "tensor",
                "achieved": None if gemm_tflops is None else round(gemm_tflops, 1),
                "peak": round(fp4_peak, 1),
                "peak_basis": f"4 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s)",
                "unit": "TFLOP/s",
                "frac": None if gemm_tflops is None else round(gemm_tflops / fp4_peak, 4),
                "traffic": None,
            },
            "gpu_launches": kt.launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------------------
# Config 2: one NVFP4 linear forward, both operands quantized in the step
# --------------------------------------------------------------------------------------------------
C2_M, C2_K, C2_N = 8192, 4096, 4096
C2_FLOPS = 2.0 * C2_M * C2_N * C2_K  # 274.9e9
C2_ROT = 3
C2_METRIC = "NVFP4 linear forward TFLOPS (BASELINE config 2: 8192 x 4096 x 4096, both operands quantized)"


def run_config2(args):
    """One step = global scales of X and W, rowblock quantization of both, the block-scaled GEMM with
    bf16 output (the forward of radiance's FP4Linear with its weight quantized in the step).
    X ~ N(0,1) with 0.1% of its channels scaled x20 (outlier columns); W ~ N(0, 1/sqrt(K)); seed 0.
    One GPU (with N ranks, each runs its own copy: replicas)."""
    import torch
    import torch.distributed as dist

    import radiance_b200.nvfp4 as nv
    from radiance_b200.nvfp4 import _trace
    from radiance_b200.nvfp4.quantize import _gemm

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(C2_M, C2_K, generator=g)
    cols = torch.randperm(C2_K, generator=g)[: round(0.001 * C2_K)]
    x[:, cols] *= 20.0
    w = torch.randn(C2_N, C2_K, generator=g) / C2_K ** 0.5
    # Three copies of the inputs (288 MiB, more than L2), used in turn: no step finds its inputs in L2.
    xs = [x.to(device, torch.bfloat16) for _ in range(C2_ROT)]
    ws = [w.to(device, torch.bfloat16) for _ in range(C2_ROT)]
    gx = torch.empty((), device=device)
    gw = torch.empty((), device=device)
    xq = (torch.empty(C2_M, C2_K // 2, dtype=torch.uint8, device=device),
          torch.empty(nv.row_scale_bytes(C2_M, C2_K), dtype=torch.uint8, device=device))
    wq = (torch.empty(C2_N, C2_K // 2, dtype=torch.uint8, device=device),
          torch.empty(nv.row_scale_bytes(C2_N, C2_K), dtype=torch.uint8, device=device))
    out = torch.empty(C2_M, C2_N, dtype=torch.bfloat16, device=device)

    def one(x, w):
        nv.global_scale_of(x, out=gx)
        nv.global_scale_of(w, out=gw)
        nv.quantize_into_(x, global_scale=gx, row=xq)
        nv.quantize_into_(w, global_scale=gw, row=wq)
        _gemm(xq[0], xq[1], wq[0], wq[1], gx, gw, None, torch.bfloat16, out)

    def step():  # C2_ROT forwards, one per input copy
        for r in range(C2_ROT):
            one(xs[r], ws[r])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    run_step = step
    graph = None
    if not args.eager:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        run_step = graph.replay
    clocks.start()
    for _ in range(20):
        run_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, args.steps // C2_ROT)
    start.record()
    for _ in range(reps):
        run_step()
    stop.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(stop) / (reps * C2_ROT)
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kt_reps = max(1, min(reps, 16))
    with _trace.kernel_timer() as kt:
        for _ in range(kt_reps):
            step()
        torch.cuda.synchronize()
    n_fwd = reps * C2_ROT  # forwards timed; per-kernel totals are scaled to them
    per_kind = {k: {"launches": int(round(v["launches"] * reps / kt_reps)),
                    "ms": round(v["ms"] * reps / kt_reps, 3)} for k, v in kt.summary().items()}
    if graph is not None:
        del graph
    if rank == 0:
        peaks, peak_kind = _peaks()
        fp4_peak = 4.0 * peaks["bf16_tflops"]
        gemm_ms = per_kind.get("gemm", {"ms": 0.0})["ms"] / n_fwd
        gemm_tflops = C2_FLOPS / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
        qms = per_kind.get("quantize", {"ms": 0.0})["ms"] / n_fwd
        qbytes = (C2_M + C2_N) * C2_K * 2.5625
        line = {
            "metric": C2_METRIC,
            "value": round(world * C2_FLOPS / (ms * 1e-3) / 1e12, 2),
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": n_fwd,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out)",
            "data": "synthetic (seeded; X~N(0,1) with 0.1% channels x20, W~N(0,1/sqrt(K)))",
            "config": {
                "workload": "config2: one linear forward, amax + rowblock quantization of X and W + GEMM",
                "m": C2_M, "k": C2_K, "n": C2_N,
                "parallelism": "one GPU" if world == 1 else f"{world} independent replicas",
                "timing": "the step captured in one CUDA graph, replayed K times (per-kernel times from an eager pass)"
                if not args.eager else "eager Python step loop",
                "l2": f"{C2_ROT} copies of X (64 MiB) and W (32 MiB) used in turn: each step's inputs are not in L2",
            },
            "kernels": per_kind,
            "quantizer_GBps": round(qbytes / (qms * 1e-3) / 1e9, 1) if qms else None,
            "roofline": {
                "kernel": "nvfp4_gemm2_kernel (tcgen05 cta_group::2 block-scaled GEMM)",
                "bound": "tensor",
                "achieved": None if gemm_tflops is None else round(gemm_tflops, 1),
                "peak": round(fp4_peak, 1),
                "peak_basis": f"4 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s)",
                "unit": "TFLOP/s",
                "frac": None if gemm_tflops is None else round(gemm_tflops / fp4_peak, 4),
                "traffic": None,
            },
            "gpu_launches": kt.launches * reps // kt_reps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------------------
# Config 5: large dense block, attention linears token-sharded, FFN N-split with output all-gather
# --------------------------------------------------------------------------------------------------
C5_TOKENS = 65536
C5_TOKEN_SHARDED = [("qkv", 4096, 6144), ("o", 4096, 4096), ("down", 14336, 4096)]
C5_NSPLIT = [("gate_up", 4096, 28672)]  # the largest layer
C5_FLOPS = 6.0 * C5_TOKENS * sum(k * n for _, k, n in C5_TOKEN_SHARDED + C5_NSPLIT)  # 85.76e12 per step (whole job)
C5_METRIC = "NVFP4 linear fwd+bwd TFLOPS (BASELINE config 5: d_model 4096 block, 65536 tokens per job)"


def run_config5(args):
    """One step = the block's four linears fwd + dgrad + wgrad for a fixed 65536-token job.  QKV,
    O and down are token-sharded (65536/N rows per rank, no collective).  The largest layer,
    gate/up (4096 -> 28672), is split along N: every rank holds 28672/N rows of the weight
    (quantized with the full weight's global scale), computes its column slice for all 65536 rows
    and all-gathers the bf16 output; the partial input gradients are all-reduced.  Total work is
    fixed as N grows (strong scaling)."""
    import torch
    import torch.distributed as dist

    from radiance_b200 import nvfp4 as nv
    from radiance_b200.nvfp4 import _trace
    from radiance_b200.nvfp4.nsplit import FP4ColumnParallelLinear

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    if C5_TOKENS % (128 * world):
        raise SystemExit(f"config 5 needs 65536 tokens to shard into multiples of 128 over {world} ranks")
    m_local = C5_TOKENS // world
    # The N-split layer's rows (all 65536 tokens of the job) are replicated over the group: every
    # rank computes its column slice of gate_up for all of them.
    m_ffn = C5_TOKENS
    gen = torch.Generator(device=device).manual_seed(777)  # same on every rank: replicated weights/rows
    layers, inputs, grads = [], [], []
    for name, k, n in C5_TOKEN_SHARDED:
        lin = nv.FP4Linear(k, n, bias=False, device=device)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, device=device, generator=gen) * 0.02)
        lin.refresh_fp4_cache()
        layers.append((lin, lin.weight))
        g_local = torch.Generator(device=device).manual_seed(1000 + rank)
        inputs.append(torch.randn(m_local, k, device=device, generator=g_local).to(torch.bfloat16))
        grads.append((torch.randn(m_local, n, device=device, generator=g_local) * 1e-3).to(torch.bfloat16))
    for name, k, n in C5_NSPLIT:
        lin = FP4ColumnParallelLinear(k, n, device=device, fused_gather=args.nsplit == "fused")
        lin.load_full_weight(torch.randn(n, k, device=device, generator=gen) * 0.02)
        lin.refresh_fp4_cache()
        layers.append((lin, lin.local.weight))
        inputs.append(torch.randn(m_ffn, k, device=device, generator=gen).to(torch.bfloat16))
        grads.append((torch.randn(m_ffn, n, device=device, generator=gen) * 1e-3).to(torch.bfloat16))
    flops_rank = 6.0 * (m_local * sum(k * n for _, k, n in C5_TOKEN_SHARDED)
                        + m_ffn * sum(k * n for _, k, n in C5_NSPLIT) / world)
    gather_bytes = sum(m_ffn * n * 2 * (world - 1) // world for _, k, n in C5_NSPLIT) if world > 1 else 0
    reduce_bytes = sum(m_ffn * k * 2 for _, k, n in C5_NSPLIT) if world > 1 else 0

    def step():
        for (lin, w), x0, dy in zip(layers, inputs, grads):
            x = x0.detach().requires_grad_(True)
            y = lin(x)
            torch.autograd.grad(y, (x, w), dy)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    steps = max(3, min(args.steps, 20))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    clocks.start()
    for _ in range(3):
        step()
    with _trace.kernel_timer() as kt:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(steps):
            step()
        stop.record()
        torch.cuda.synchronize()
        barrier()
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(stop)) / steps
    per_kind = kt.summary()
    if rank == 0:
        peaks, peak_kind = _peaks()
        fp4_peak = 4.0 * peaks["bf16_tflops"]
        gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0, "work": 0.0})
        gemm_tflops = gemm["work"] / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else None
        line = {
            "metric": C5_METRIC,
            "value": round(C5_FLOPS / (ms * 1e-3) / 1e12, 2),
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
            "data": "synthetic (seeded; W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
            "config": {
                "workload": "config5: d_model 4096 block linears fwd+dgrad+wgrad; QKV/O/down token-sharded, "
                            "gate_up (the largest) N-split with an NCCL all-gather of its bf16 output",
                "tokens_per_job": C5_TOKENS, "attention_rows_per_rank": m_local, "ffn_rows": m_ffn,
                "layers": {n: [k, o] for n, k, o in C5_TOKEN_SHARDED + C5_NSPLIT},
                "flops_per_rank_per_step": flops_rank,
                "allgather_bytes_received_per_rank_per_step": gather_bytes,
                "dgrad_allreduce_bytes_per_rank_per_step": reduce_bytes,
                "parallelism": f"gate_up N-split over {world} + token-sharded QKV/O/down",
                "nsplit_gather": ("GEMM epilogue stores each tile into every rank's output over NVLink "
                                  "(rb_nvfp4_gemm_allgather, symmetric memory)") if args.nsplit == "fused"
                else "NCCL all_gather_into_tensor + column permute",
            },
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3)} for k, v in per_kind.items()},
            "roofline": {
                "kernel": "nvfp4_gemm2_kernel",
                "bound": "tensor",
                "achieved": None if gemm_tflops is None else round(gemm_tflops, 1),
                "peak": round(fp4_peak, 1),
                "peak_basis": f"4 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s)",
                "unit": "TFLOP/s",
                "frac": None if gemm_tflops is None else round(gemm_tflops / fp4_peak, 4),
                "traffic": None,
            },
            "gpu_launches": kt.launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--eager", action="store_true",
                    help="config 3: time the Python step loop instead of a captured CUDA graph of the step")
    ap.add_argument("--nsplit", choices=["fused", "nccl"], default="fused",
                    help="config 5: the N-split layer's output all-gather (fused into the GEMM, or NCCL)")
    ap.add_argument("--config", choices=["2", "3", "4", "5"], default="3",
                    help="2: one linear forward (8192 x 4096 x 4096); 3: dense block linears (the headline "
                         "line); 4: MoE expert linears; 5: d_model 4096 block with the FFN N-split")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "2":
        run_config2(args)
    elif args.config == "4":
        run_config4(args)
    elif args.config == "5":
        run_config5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
