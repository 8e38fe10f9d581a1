"""Benchmark of the NVFP4 linear path (BASELINE metric: NVFP4 linear fwd+bwd TFLOPS).

Workload: one dense transformer block's linears -- QKV 2048->6144,
O 2048->2048, gate/up 2048->11264, down 5632->2048 -- forward + dgrad + wgrad through
``radiance_b200.nvfp4.FP4Linear`` with the default recipe (stochastic rounding and Hadamard on,
packed activation saving on), weights ~N(0, 0.02), activations ~N(0, 1), upstream gradients
~N(0, 1e-3).  A step = the job's 16384 tokens (batch 8 x seq 2048): the four forwards, then the four
backwards.  With N ranks the tokens are sharded (16384/N per rank, strong scaling) and each linear's
fp32 weight gradient is reduce-scattered over the ranks inside the step, as data-parallel training
needs; the weak-scaled replica number (16384 tokens on every rank, no reduction) is reported beside
it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5]
    python bench.py case quant|gemm|swiglu|block-gemms [...]   (one kernel's workload, for ncu or --time)

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU implementation of
the path on the host cores, on a bounded token sample of the same workload: radiance's own torch
emulation when it is installed under baseline/_ref, else the NumPy restatement of it in ``oracle/``.
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
TOKENS = 16384  # tokens per step of the whole job (batch 8 x seq 2048)
LAYERS = [("qkv", 2048, 6144), ("o", 2048, 2048), ("gate_up", 2048, 11264), ("down", 5632, 2048)]
LAYER_KN = sum(k * n for _, k, n in LAYERS)
STEP_FLOPS = 6.0 * TOKENS * LAYER_KN  # 5.051e12 per step of the job
METRIC = "NVFP4 linear fwd+bwd TFLOPS (BASELINE config 3 block linears, 16384 tokens per step, token-sharded)"
# SMs left to the dW reduce-scatter per world size (measured best of 0/8/16/24/32 at N=2 and 0/16/32 at
# N=8: the collective's share of the step grows with N while each rank's GEMM work shrinks).
COMM_SMS_DEFAULT = {2: 16, 4: 24, 8: 32}

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


class Block:
    """The block's NVFP4 layers, identical on every rank (data-parallel replicas of one model).

    ``ffn=True`` (the headline): QKV and O as ``FP4Linear``, and the FFN as radiance's FeedForward
    (``down_proj(F.silu(gate_proj(x)) * up_proj(x))``, src/radiance/model/ffn.py:32) built as
    ``FP4FeedForward``: the gate/up GEMM writes h = silu(g) * u and h's global scale in its epilogue,
    and down_proj quantizes h with that scale.  ``ffn=False``: the four linears on independent inputs.
    Either way the linears are BASELINE config 3's (QKV 2048->6144, O 2048->2048, gate/up
    2048->11264, down 5632->2048) and the GEMM work per token is the same.
    ``units``: (name, module, in_features, out_features, FP4Linear modules holding weights)."""

    def __init__(self, device, ffn=True):
        import torch

        from radiance_b200 import nvfp4 as nv

        g = torch.Generator(device="cpu").manual_seed(1234)
        rec = nv.FP4Recipe()

        def linear(k, n):
            lin = nv.FP4Linear(k, n, bias=False, recipe=rec)
            with torch.no_grad():
                lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
            return lin.to(device)

        self.ffn = ffn
        self.units = []
        names = LAYERS if not ffn else LAYERS[:2]
        for name, k, n in names:
            lin = linear(k, n)
            self.units.append((name, lin, k, n, [lin]))
        if ffn:
            d, hid = LAYERS[2][1], LAYERS[3][1]
            mod = nv.FP4FeedForward(d, hid, bias=False, recipe=rec)
            with torch.no_grad():
                mod.gate_up.weight.copy_(torch.randn(2 * hid, d, generator=g) * 0.02)
                mod.down_proj.weight.copy_(torch.randn(d, hid, generator=g) * 0.02)
            mod = mod.to(device)
            self.units.append(("ffn", mod, d, d, [mod.gate_up, mod.down_proj]))
        for unit in self.units:
            for lin in unit[4]:
                lin.refresh_fp4_cache()

    def linears(self):
        return [lin for unit in self.units for lin in unit[4]]

    def inputs(self, tokens, seed):
        """This rank's token shard: activations ~N(0,1) and upstream gradients ~N(0,1e-3), bf16, on
        the host."""
        import torch

        g = torch.Generator(device="cpu").manual_seed(seed)
        xs, dys = [], []
        for _, _, k, n, _ in self.units:
            xs.append(torch.randn(tokens, k, generator=g).to(torch.bfloat16))
            dys.append((torch.randn(tokens, n, generator=g) * 1e-3).to(torch.bfloat16))
        return xs, dys


class BlockStep:
    """One training step of the block on this rank's token shard: the forwards, then the backwards
    in reverse order (as a block's backward runs).  With several ranks, each linear's fp32 dW is
    reduce-scattered over the ranks (ZeRO-style: rank r keeps the summed rows r*N/g .. (r+1)*N/g) on
    a side stream, issued from the layer's wgrad hook the moment its wgrad GEMM has produced dW, so
    the reduction overlaps that layer's dgrad and the layers still to come."""

    def __init__(self, block, world, device, reduce=True, group=None):
        import torch

        self.block, self.world, self.group = block, world, group
        self.reduce = reduce and world > 1
        self.side = torch.cuda.Stream(device)
        lins = block.linears()
        self.shards = {id(lin): torch.empty(lin.out_features // world, lin.in_features, device=device) for lin in lins}
        self.reduce_bytes = sum(lin.weight.numel() * 4 for lin in lins) if self.reduce else 0
        self._pending = []

    def _hook(self, lin):
        import torch
        import torch.distributed as dist

        from radiance_b200.nvfp4 import _trace

        shard = self.shards[id(lin)]

        def hook(grad_w):
            self.side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.side):
                tok = _trace.begin("reduce_scatter", grad_w.numel() * 4)
                dist.reduce_scatter_tensor(shard, grad_w, group=self.group)
                _trace.end(tok)
            self._pending.append(grad_w)  # keeps dW alive until the side stream has consumed it
        return hook

    def __call__(self, xs, dys, outs=None):
        import torch

        lins = self.block.linears()
        if self.reduce:
            for lin in lins:
                lin.wgrad_hook = self._hook(lin)
        ins, ys = [], []
        for i, unit in enumerate(self.block.units):
            x = xs[i].detach().requires_grad_(True)
            ins.append(x)
            ys.append(unit[1](x))
        for i in reversed(range(len(self.block.units))):
            params = [lin.weight for lin in self.block.units[i][4]]
            grads = torch.autograd.grad(ys[i], (ins[i], *params), dys[i])
            if outs is not None:
                dws = [self.shards[id(lin)] for lin in self.block.units[i][4]] if self.reduce else list(grads[1:])
                outs.append((i, grads[0], dws))
        if self.reduce:
            torch.cuda.current_stream().wait_stream(self.side)
            self._pending.clear()
            for lin in lins:
                lin.wgrad_hook = None


def _capture(fn):
    """Capture fn() in a CUDA graph after two warm-up calls on a side stream; returns the graph."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    return graph


def _graph_kernel_times(fn, replays):
    """Per-kind device time of one step, measured inside a CUDA graph of the step: the step is
    captured with timing events around every library launch (and every reduce-scatter), replayed,
    and the event pairs of each replay are summed.  Returns (per-kind totals averaged per step,
    launches per step)."""
    import torch

    from radiance_b200.nvfp4 import _trace

    with _trace.kernel_timer() as kt:
        graph = _capture(fn)
        # The two warm-up calls inside _capture recorded events too; keep only the captured ones.
        per_step = kt.launches // 3
        kt.records = kt.records[-per_step:]
    totals: dict = {}
    for _ in range(replays):
        graph.replay()
        torch.cuda.synchronize()
        for kind, v in kt.summary().items():
            t = totals.setdefault(kind, {"launches": 0, "ms": 0.0, "work": 0.0})
            t["launches"] += v["launches"]
            t["ms"] += v["ms"]
            t["work"] += v["work"]
    del graph
    out = {k: {"launches": v["launches"] / replays, "ms": v["ms"] / replays, "work": v["work"] / replays}
           for k, v in totals.items()}
    launches = sum(v["launches"] for k, v in out.items() if k != "reduce_scatter")
    return out, int(round(launches))


def _timed_replays(run_step, steps, barrier, clocks=None):
    """K replays between CUDA events, bracketed by a barrier and a synchronize on both sides."""
    import torch

    if clocks is not None:
        clocks.start()
    for _ in range(20):  # keep the GPU loaded while the clock sampler starts (untimed)
        run_step()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        run_step()
    stop.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    return start.elapsed_time(stop), clk


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    if args.tokens_per_rank:
        tokens, scaling = args.tokens_per_rank, "weak"
    else:
        if TOKENS % (128 * world):
            raise SystemExit(f"{TOKENS} tokens do not shard into multiples of 128 over {world} ranks")
        tokens, scaling = TOKENS // world, "strong"
    step_flops = 6.0 * tokens * LAYER_KN  # this rank's GEMM work per step
    block = Block(device, ffn=not args.linears_only)
    xs_host, dys_host = block.inputs(tokens, seed=1000 + rank)
    xs = [x.to(device) for x in xs_host]
    dys = [d.to(device) for d in dys_host]
    rs_group = None
    comm_sms = 0
    if world > 1:
        # The gradient reduce-scatters get their own communicator, limited to --comm-sms CTAs, and
        # this library's kernels leave that many SMs free, so the collective runs beside the GEMMs
        # and quantizers instead of waiting for SMs between them.
        from radiance_b200 import _lib

        comm_sms = max(0, args.comm_sms) if args.comm_sms >= 0 else COMM_SMS_DEFAULT.get(world, 32)
        opts = dist.ProcessGroupNCCL.Options()
        if comm_sms:
            opts.config.max_ctas = comm_sms
            opts.config.min_ctas = min(comm_sms, 4)
            _lib.set_sm_budget(torch.cuda.get_device_properties(device).multi_processor_count - comm_sms)
        rs_group = dist.new_group(ranks=list(range(world)), backend="nccl", pg_options=opts)
    step = BlockStep(block, world, device, group=rs_group)

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
        step(xs, dys)
    torch.cuda.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    # The step is captured once in a CUDA graph and replayed: every kernel and every reduce-scatter
    # of the step runs on every replay; the graph removes the host's per-launch overhead, which with
    # eight processes sharing the host's cores leaves gaps between kernels.  --eager times the
    # Python loop instead.
    graph = None
    run_step = (lambda: step(xs, dys))
    if not args.eager:
        graph = _capture(run_step)
        run_step = graph.replay
    ms, clk = _timed_replays(run_step, args.steps, barrier, ClockSampler(phys))
    ms_max = max_over_ranks(ms)
    per_kind, launches_per_step = _graph_kernel_times(lambda: step(xs, dys), replays=max(3, min(args.steps, 20)))
    del graph, run_step

    # ---- the same shard without the gradient reduction (N > 1): fwd + dgrad + wgrad on 16384/N
    # tokens per rank and nothing else -- token sharding as a pure partition ("Token (M) rows shard
    # with no communication"); the difference to `value` is the reduce-scatter's exposed time.
    no_reduce = None
    if world > 1:
        nstep = BlockStep(block, world, device, reduce=False)
        for _ in range(3):
            nstep(xs, dys)
        ngraph = _capture(lambda: nstep(xs, dys))
        nms, _ = _timed_replays(ngraph.replay, args.steps, barrier)
        nms_max = max_over_ranks(nms) / args.steps
        no_reduce = {"value": round(step_flops * world / (nms_max * 1e-3) / 1e12, 2), "unit": "TFLOPS",
                     "ms_per_step": round(nms_max, 4), "tokens_per_gpu": tokens, "scaling": scaling,
                     "what": "the same token-sharded step without the dW reduce-scatter"}
        del ngraph, nstep
        torch.cuda.synchronize()

    # ---- the four linears alone (N = 1): the same GEMM work on independent inputs, no SwiGLU
    linears_only = None
    if world == 1 and block.ffn and not args.no_subrecords:
        lblock = Block(device, ffn=False)
        lx_host, ldy_host = lblock.inputs(tokens, seed=3000)
        lxs = [x.to(device) for x in lx_host]
        ldys = [d.to(device) for d in ldy_host]
        lstep = BlockStep(lblock, 1, device, reduce=False)
        for _ in range(3):
            lstep(lxs, ldys)
        lgraph = _capture(lambda: lstep(lxs, ldys))
        lms, _ = _timed_replays(lgraph.replay, args.steps, barrier)
        lms /= args.steps
        linears_only = {"value": round(step_flops / (lms * 1e-3) / 1e12, 2), "unit": "TFLOPS", "ms_per_step": round(lms, 4),
                        "what": "the four linears fwd+dgrad+wgrad on independent inputs (no SwiGLU between gate/up and "
                                "down): the same GEMM work as the headline step"}
        del lgraph, lstep, lxs, ldys, lblock
        torch.cuda.synchronize()

    # ---- weak-scaled replicas (N > 1): every rank a whole 16384-token micro-batch, no collective
    weak = None
    if world > 1 and not args.tokens_per_rank:
        from radiance_b200 import _lib

        _lib.set_sm_budget(0)  # replicas have no collective to make room for
        wx_host, wdy_host = block.inputs(TOKENS, seed=2000 + rank)
        wxs = [x.to(device) for x in wx_host]
        wdys = [d.to(device) for d in wdy_host]
        wstep = BlockStep(block, world, device, reduce=False)
        for _ in range(3):
            wstep(wxs, wdys)
        wgraph = _capture(lambda: wstep(wxs, wdys))
        wms, _ = _timed_replays(wgraph.replay, args.steps, barrier)
        wms_max = max_over_ranks(wms) / args.steps
        weak = {"value": round(world * 6.0 * TOKENS * LAYER_KN / (wms_max * 1e-3) / 1e12, 2), "unit": "TFLOPS",
                "ms_per_step": round(wms_max, 4), "tokens_per_gpu": TOKENS, "scaling": "weak",
                "what": "every rank runs its own 16384-token micro-batch, no gradient reduction (replicas)"}
        del wgraph, wxs, wdys
        torch.cuda.synchronize()
        if comm_sms:
            _lib.set_sm_budget(torch.cuda.get_device_properties(device).multi_processor_count - comm_sms)

    # ---- end-to-end through the public API with host buffers (e2e) --------------------------
    e2e = _e2e(block, xs_host, dys_host, step, device, world, args, barrier, max_over_ranks)
    reducing, reduce_bytes = step.reduce, step.reduce_bytes
    if comm_sms:
        from radiance_b200 import _lib

        _lib.set_sm_budget(0)
    comparators = None
    if world == 1 and not args.no_subrecords and not args.tokens_per_rank:
        comparators = measure_comparators(block, xs, dys, device)
    del xs, dys, step

    # ---- configs 4 and 5 as sub-records (with their parity checks at N > 1) --------------------
    subs = {}
    if not args.no_subrecords and not args.tokens_per_rank:
        for name, fn, n_steps in (("config4", measure_config4, max(3, min(args.steps, 50))),
                                  ("config5", measure_config5, max(3, min(args.steps, 10)))):
            torch.cuda.empty_cache()
            try:
                rec = fn(args, rank, world, device, barrier, max_over_ranks, n_steps)
            except Exception as e:  # a sub-record must not take the headline line down with it
                rec = {"error": f"{type(e).__name__}: {e}"[:400]}
            if rank == 0:
                subs[name] = rec

    if rank == 0:
        peaks, peak_kind = _peaks()
        ms_step = ms_max / args.steps
        job_flops = step_flops * world
        value = job_flops / (ms_step * 1e-3) / 1e12
        gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0, "work": 0.0})
        quant = per_kind.get("quantize", {"launches": 0, "ms": 0.0, "work": 0.0})
        amax = per_kind.get("amax", {"launches": 0, "ms": 0.0, "work": 0.0})
        rs = per_kind.get("reduce_scatter")
        fp4_peak = 4.0 * peaks["bf16_tflops"]
        gemm_tflops = gemm["work"] / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else None
        quant_gbs = quant["work"] / (quant["ms"] * 1e-3) / 1e9 if quant["ms"] else None
        hbm = peaks["hbm_gbs"]
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
            "data": "synthetic (seeded; W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
            "config": {
                "workload": ("config3: dense block linears fwd+dgrad+wgrad; QKV and O via FP4Linear, the FFN (gate/up "
                             "-> SwiGLU -> down) via FP4FeedForward (SwiGLU and h's global scale in the gate/up GEMM's "
                             "epilogue)") if block.ffn else "config3: the four block linears fwd+dgrad+wgrad via FP4Linear "
                                                            "on independent inputs",
                "d_model": D_MODEL,
                "layers": {n: [k, o] for n, k, o in LAYERS},
                "global_batch_tokens": tokens * world,
                "tokens_per_gpu": tokens,
                "recipe": "grad_gemms, stochastic_rounding, hadamard, save_activations",
                "parallelism": (f"token-sharded dp{world}: 16384 tokens per step split over the ranks, each linear's "
                                "fp32 dW reduce-scattered (NCCL, overlapped from the wgrad hook) inside the step")
                if world > 1 and reducing else "one GPU" if world == 1 else f"{world} replicas",
                "grad_reduce_bytes_per_step": reduce_bytes,
                "comm_sms": comm_sms,
                "l2": "inputs larger than L2 (about 1 GB of activations and gradients per 16384 tokens)",
                "timing": "eager Python step loop" if args.eager else
                          "the step captured in one CUDA graph, replayed K times; per-kernel times from event pairs "
                          "captured in a second graph of the same step",
            },
            "tokens_per_s": round(tokens * world / (ms_step * 1e-3), 1),
            "gpu_launches": launches_per_step * args.steps,
            "kernels": {
                "gemm": {"launches_per_step": gemm["launches"], "ms_per_step": round(gemm["ms"], 4),
                         "TFLOPS": None if gemm_tflops is None else round(gemm_tflops, 1)},
                "quantize": {"launches_per_step": quant["launches"], "ms_per_step": round(quant["ms"], 4),
                             "GBps": None if quant_gbs is None else round(quant_gbs, 1)},
                "amax": {"launches_per_step": amax["launches"], "ms_per_step": round(amax["ms"], 4),
                         "GBps": round(amax["work"] / (amax["ms"] * 1e-3) / 1e9, 1) if amax["ms"] else None},
            },
            "roofline": {
                "kernel": "nvfp4_gemm2_kernel (tcgen05 cta_group::2 block-scaled GEMM)",
                "bound": "tensor",
                "achieved": None if gemm_tflops is None else round(gemm_tflops, 1),
                "peak": round(fp4_peak, 1),
                "peak_basis": f"4 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s): B200 NVFP4 dense rate is 4x "
                              "bf16; nominal 9000",
                "unit": "TFLOP/s",
                "frac": None if gemm_tflops is None else round(gemm_tflops / fp4_peak, 4),
                "frac_of_nominal_9000": None if gemm_tflops is None else round(gemm_tflops / 9000.0, 4),
                "traffic": GEMM_DRAM_BYTES_PER_LAUNCH if tokens == TOKENS else None,
                "flops_per_launch": round(gemm["work"] / max(gemm["launches"], 1)),
                "ms_per_launch": round(gemm["ms"] / max(gemm["launches"], 1), 5),
            },
            "roofline_quantizer": {
                "kernel": "nvfp4_quantize_kernel (both layouts; Hadamard colblock; SR on gradients)",
                "bound": "hbm",
                "achieved": None if quant_gbs is None else round(quant_gbs, 1),
                "peak": hbm,
                "unit": "GB/s",
                "frac": None if quant_gbs is None else round(quant_gbs / hbm, 4),
                "peak_basis": f"{peak_kind} HBM copy bandwidth",
                "traffic": None,
                "bytes_per_launch": round(quant["work"] / max(quant["launches"], 1)),
                "ms_per_launch": round(quant["ms"] / max(quant["launches"], 1), 5),
            },
            "e2e": e2e,
            "clocks": clk,
        }
        if rs is not None:
            line["kernels"]["reduce_scatter"] = {
                "calls_per_step": rs["launches"], "ms_per_step": round(rs["ms"], 4),
                "GBps_algbw": round(rs["work"] / (rs["ms"] * 1e-3) / 1e9, 1) if rs["ms"] else None,
                "note": "NCCL on a side stream, overlapped with the GEMMs; its time is not additive"}
        if no_reduce is not None:
            line["without_grad_reduction"] = no_reduce
        if linears_only is not None:
            line["linears_only"] = linears_only
        if weak is not None:
            line["weak_replicas"] = weak
        if comparators is not None:
            line["comparators"] = comparators
        for name, rec in subs.items():
            line[name] = rec
        flags = [rec.get("parity_ok") for rec in subs.values() if "parity_ok" in rec]
        if flags:
            line["parity_ok"] = all(flags)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _e2e(block, xs_host, dys_host, step, device, world, args, barrier, max_over_ranks):
    """The same step through the public API with host buffers: every step copies its inputs from
    pinned host memory and copies its results (every input gradient, and this rank's weight-gradient
    rows -- the reduce-scattered shards with several ranks) back to pinned host memory, inside the
    timed region.  Step s+1's uploads run on a copy stream during step s (double-buffered inputs,
    the way a data loader feeds a training loop), and step s's downloads on another while step s+1
    computes."""
    import torch

    pinned_x = [x.pin_memory() for x in xs_host]
    pinned_dy = [d.pin_memory() for d in dys_host]
    tokens = xs_host[0].shape[0]
    out_dx = [torch.empty(tokens, unit[2], dtype=torch.bfloat16).pin_memory() for unit in block.units]
    out_dw = [[torch.empty(lin.out_features // world if step.reduce else lin.out_features, lin.in_features,
                           dtype=torch.float32).pin_memory() for lin in unit[4]] for unit in block.units]
    h2d = sum(t.numel() * t.element_size() for t in pinned_x + pinned_dy)
    d2h = sum(t.numel() * t.element_size() for t in out_dx) + sum(t.numel() * 4 for ws in out_dw for t in ws)
    n_in = len(block.units)
    dev_sets = [([torch.empty_like(x, device=device) for x in xs_host],
                 [torch.empty_like(d, device=device) for d in dys_host]) for _ in range(2)]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    used = [False, False]

    def issue_copy(b):
        with torch.cuda.stream(up):
            if used[b]:
                up.wait_event(consumed[b])
            for i in range(n_in):
                dev_sets[b][0][i].copy_(pinned_x[i], non_blocking=True)
                dev_sets[b][1][i].copy_(pinned_dy[i], non_blocking=True)
            copied[b].record(up)

    def run(n):
        cur = torch.cuda.current_stream()
        up.wait_stream(cur)  # the first upload starts inside the timing
        issue_copy(0)
        for s_ in range(n):
            b = s_ % 2
            if s_ + 1 < n:
                issue_copy(1 - b)
            cur.wait_event(copied[b])
            step.side.wait_stream(down)  # the reduce-scatter reuses the dW shards the last download reads
            outs = []
            step(dev_sets[b][0], dev_sets[b][1], outs)
            consumed[b].record()
            used[b] = True
            down.wait_stream(cur)
            with torch.cuda.stream(down):
                for i, gx, gws in outs:
                    out_dx[i].copy_(gx, non_blocking=True)
                    gx.record_stream(down)
                    for j, gw in enumerate(gws):
                        out_dw[i][j].copy_(gw, non_blocking=True)
                        gw.record_stream(down)
        cur.wait_stream(down)

    e2e_steps = max(3, min(args.steps, 20))
    run(max(3, args.warmup))
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    run(e2e_steps)
    ee.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(es.elapsed_time(ee)) / e2e_steps
    return {
        "value": round(world * 6.0 * tokens * LAYER_KN / (e2e_ms * 1e-3) / 1e12, 2),
        "unit": "TFLOPS",
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": d2h,
        "ms_per_step": round(e2e_ms, 3),
        "path": "FP4Linear forward/backward (public API) per rank; inputs from pinned host memory each step "
                "(uploads of step s+1 overlap step s), results (every dX and this rank's dW rows) copied back to "
                "pinned host memory each step; eager launches",
    }


def _import_reference():
    """radiance itself, installed unmodified under baseline/_ref (pip install --no-deps of the
    reference), or (None, why)."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "radiance")):
        return None, "the reference is not installed under baseline/_ref"
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import radiance.nvfp4 as rnv
    except Exception as e:  # report, do not fail the line
        return None, f"import radiance.nvfp4 failed: {type(e).__name__}: {e}"[:300]
    return rnv, None


def _graph_ms(fn, reps=5, warm=3):
    """Device milliseconds per call of fn: captured in a CUDA graph (falls back to eager calls when
    capture fails), best of `reps` timed replays after `warm` calls."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    run, mode = fn, "eager"
    try:
        graph = _capture(fn)
        run, mode = graph.replay, "graph"
    except Exception:
        torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        run()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        best = ms if best is None else min(best, ms)
    return best, mode


def measure_comparators(block, xs, dys, device):
    """One GPU, the config-3 shapes: (1) the reference's own GPU path -- radiance's FP4Linear
    (Triton quantizers, torch._scaled_mm_v2 GEMMs) from baseline/_ref -- on the same block step, and
    (2) the step's twelve GEMMs through cuBLASLt's NVFP4 GEMM (torch._scaled_mm_v2, the GEMM radiance
    uses) against this library's, on identical operands.  Timing only; the reference's kernels are
    never read."""
    import torch

    from radiance_b200.nvfp4.quantize import _gemm, quantize

    out = {}
    tokens = xs[0].shape[0]
    # (2) the twelve GEMMs of the step: ours vs cuBLASLt on the same operands and output types
    try:
        from torch._C import _ScalingType, _SwizzleType

        blk = [_ScalingType.BlockWise1x16.value]
        swz = [_SwizzleType.SWIZZLE_32_4_4.value]
        g = torch.Generator(device="cpu").manual_seed(13)
        calls = []
        for _, k, n in LAYERS:
            for (m_, n_, k_, od) in ((tokens, n, k, torch.bfloat16), (tokens, k, n, torch.bfloat16),
                                     (n, k, tokens, torch.float32)):
                a = quantize(torch.randn(m_, k_, generator=g).to(device, torch.bfloat16), -1)
                b = quantize((torch.randn(n_, k_, generator=g) * 0.02).to(device, torch.bfloat16), -1)
                calls.append((a, b, torch.empty(m_, n_, dtype=od, device=device), od))

        def ours():
            for a, b, o, od in calls:
                _gemm(a.packed.view(torch.uint8), a.scale.view(torch.uint8), b.packed.view(torch.uint8),
                      b.scale.view(torch.uint8), a.global_scale, b.global_scale, None, od, o)

        def cublaslt():
            for a, b, o, od in calls:
                torch._scaled_mm_v2(a.packed, b.packed.t(), scale_a=[a.scale], recipe_a=blk, swizzle_a=swz,
                                    scale_b=[b.scale], recipe_b=blk, swizzle_b=swz, bias=None, out_dtype=od)

        flops = 6.0 * tokens * LAYER_KN
        ms_o, _ = _graph_ms(ours)
        ms_c, mode = _graph_ms(cublaslt)
        # Each GEMM alone, 4 back-to-back launches per graph replay (the operands stay in L2 only
        # where they fit, as they do inside the step).
        per_gemm = []
        names = [f"{name}.{kind}" for name, _, _ in LAYERS for kind in ("fwd", "dgrad", "wgrad")]
        for name, (a, b, o, od) in zip(names, calls):
            def one_ours(a=a, b=b, o=o, od=od):
                for _ in range(4):
                    _gemm(a.packed.view(torch.uint8), a.scale.view(torch.uint8), b.packed.view(torch.uint8),
                          b.scale.view(torch.uint8), a.global_scale, b.global_scale, None, od, o)

            def one_cublaslt(a=a, b=b, od=od):
                for _ in range(4):
                    torch._scaled_mm_v2(a.packed, b.packed.t(), scale_a=[a.scale], recipe_a=blk, swizzle_a=swz,
                                        scale_b=[b.scale], recipe_b=blk, swizzle_b=swz, bias=None, out_dtype=od)

            po, _ = _graph_ms(one_ours)
            pc, _ = _graph_ms(one_cublaslt)
            m_, k2 = a.packed.shape
            per_gemm.append({"gemm": name, "mnk": [m_, b.packed.shape[0], 2 * k2],
                             "ours_us": round(po * 250, 1), "cublaslt_us": round(pc * 250, 1),
                             "ratio": round(pc / po, 3)})
        out["gemms_vs_cublaslt"] = {
            "ours_ms": round(ms_o, 4), "cublaslt_ms": round(ms_c, 4),
            "ours_TFLOPS": round(flops / (ms_o * 1e-3) / 1e12, 1), "cublaslt_TFLOPS": round(flops / (ms_c * 1e-3) / 1e12, 1),
            "ratio": round(ms_c / ms_o, 4), "timing": mode,
            "slower_than_cublaslt": [p["gemm"] for p in per_gemm if p["ratio"] < 1.0],
            "per_gemm": per_gemm,
            "what": "the step's 12 GEMMs (fwd, dgrad, wgrad of the 4 linears; bf16, bf16, fp32 outputs) on identical "
                    "NVFP4 operands: rb_nvfp4_gemm vs torch._scaled_mm_v2 (cuBLASLt, the GEMM radiance calls); "
                    "ratio = cuBLASLt time / ours; per_gemm times each alone (4 launches per graph replay)",
        }
        del calls
    except Exception as e:
        out["gemms_vs_cublaslt"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    # (1) the reference's own layers on the same block step: radiance's FP4Linear for QKV and O, and
    # its FeedForward for the FFN (gate_proj and up_proj as separate FP4Linears, F.silu(g) * u in
    # torch, down_proj), ffn.py:21-36
    rnv, why = _import_reference()
    if rnv is None:
        out["reference_gpu_step"] = {"unavailable": why}
        return out
    try:
        import torch.nn.functional as F

        from radiance_b200.nvfp4 import split_gate_up

        def ref_linear(weight):
            r = rnv.FP4Linear(weight.shape[1], weight.shape[0], bias=False)
            with torch.no_grad():
                r.weight.copy_(weight.detach().cpu())
            r = r.to(device)
            r.refresh_fp4_cache()
            return r

        units = []
        for name, mod, k, n, lins in block.units:
            if name == "ffn":
                g_t, u_t = split_gate_up(mod.gate_up.weight.detach().t())
                gate, up = ref_linear(g_t.t().contiguous()), ref_linear(u_t.t().contiguous())
                down = ref_linear(mod.down_proj.weight)

                def ffn(x, gate=gate, up=up, down=down):
                    return down(F.silu(gate(x)) * up(x))
                units.append((ffn, [gate.weight, up.weight, down.weight]))
            else:
                r = ref_linear(mod.weight)
                units.append((r, [r.weight]))

        def ref_step():
            ins, ys = [], []
            for i, (fn, _) in enumerate(units):
                x = xs[i].detach().requires_grad_(True)
                ins.append(x)
                ys.append(fn(x))
            for i in reversed(range(len(units))):
                torch.autograd.grad(ys[i], (ins[i], *units[i][1]), dys[i])

        ms_r, mode = _graph_ms(ref_step)
        flops = 6.0 * tokens * LAYER_KN
        out["reference_gpu_step"] = {
            "value": round(flops / (ms_r * 1e-3) / 1e12, 2), "unit": "TFLOPS", "ms_per_step": round(ms_r, 4),
            "timing": mode,
            "what": "radiance's own layers (src/radiance/nvfp4: Triton quantizers + torch._scaled_mm_v2; its FeedForward "
                    "with separate gate/up projections and torch SwiGLU), installed unmodified under baseline/_ref, on the "
                    "same block step (same weights, inputs and recipe)",
        }
        del units
    except Exception as e:
        out["reference_gpu_step"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return out


# --------------------------------------------------------------------------------------------------
# The CPU arm (the reference's algorithm: quantize -> dequantize -> fp32 matmul emulation)
# --------------------------------------------------------------------------------------------------
class _HostPath:
    """The NVFP4 linear path on the host cores, the way radiance defines it on a CPU: quantize both
    operands (global_scale_of, ref_quantize_rowblock / ref_quantize_colblock with the Hadamard
    rotation and stochastic rounding of the recipe), dequantize, fp32 matmul (quantize.py:205-320,
    the emulation BASELINE config 1 names; radiance's kernels run only on a GPU).  It runs radiance's
    own code, installed unmodified under baseline/_ref, when that is present (kind "reference"),
    else the oracle's numpy restatement of the same functions (kind "port").  All host threads."""

    def __init__(self):
        import torch

        self.rnv, self.why = _import_reference()
        self.kind = "reference" if self.rnv is not None else "port"
        self.cores = os.cpu_count()
        torch.set_num_threads(self.cores)
        if self.rnv is None:
            import numpy as np

            from oracle import nvfp4_oracle as O

            self.O, self.np = O, np

    # -- one layer's operands ----------------------------------------------------------------
    def weight_cache(self, w):
        """Once per optimizer step: the weight quantized both ways and dequantized (fp32)."""
        if self.rnv is not None:
            r = self.rnv
            gw = r.global_scale_of(w)
            wr = r.dequantize(*r.ref_quantize_rowblock(w, gw), gw)
            wc = r.dequantize(*r.ref_quantize_colblock(w, gw), gw)
            return wr, wc
        O = self.O
        gw = O.global_scale_of(w)
        return O.dequantize(*O.quantize_rowblock(w, gw), gw), O.dequantize(*O.quantize_colblock(w, gw), gw)

    def linear_step(self, cache, x, dy, had):
        """fwd + dgrad + wgrad of one linear (linear.py:63-155 with the default recipe)."""
        wr, wc = cache
        if self.rnv is not None:
            import torch

            r = self.rnv
            gx = r.global_scale_of(x)
            xr = r.dequantize(*r.ref_quantize_rowblock(x, gx), gx)
            xc = r.dequantize(*r.ref_quantize_colblock(x, gx, hadamard=had), gx)
            y = (xr @ wr.T).to(torch.bfloat16)
            gg = r.global_scale_of(dy)
            u = torch.rand(dy.shape)
            gr = r.dequantize(*r.ref_quantize_rowblock(dy, gg, u=u), gg)
            gc = r.dequantize(*r.ref_quantize_colblock(dy, gg, hadamard=had, u=u), gg)
            return y, (gr @ wc.T).to(torch.bfloat16), gc @ xc.T
        O, np = self.O, self.np
        gx = O.global_scale_of(x)
        xr = O.dequantize(*O.quantize_rowblock(x, gx), gx)
        xc = O.dequantize(*O.quantize_colblock(x, gx, hadamard=had), gx)
        y = xr @ wr.T
        gg = O.global_scale_of(dy)
        u = np.random.default_rng(0).random(dy.shape, dtype=np.float32)
        gr = O.dequantize(*O.quantize_rowblock(dy, gg, u=u), gg)
        gc = O.dequantize(*O.quantize_colblock(dy, gg, hadamard=had, u=u), gg)
        return y, gr @ wc.T, gc @ xc.T

    # -- inputs --------------------------------------------------------------------------------
    def tensors(self, rows, cols, std, seed, bf16=True):
        import torch

        g = torch.Generator().manual_seed(seed)
        t = torch.randn(rows, cols, generator=g) * std
        t = t.to(torch.bfloat16) if bf16 else t
        if self.rnv is not None:
            return t
        return t.float().numpy()

    def hadamard(self):
        if self.rnv is not None:
            return self.rnv.hadamard_matrix(16)
        return self.O.hadamard_matrix()

    def block(self, tokens, seed=0):
        """The config-3 block's four linears on `tokens` tokens: (weight caches, inputs)."""
        caches, ins = [], []
        for i, (_, k, n) in enumerate(LAYERS):
            caches.append(self.weight_cache(self.tensors(n, k, 0.02, 100 + i, bf16=False)))
            ins.append((self.tensors(tokens, k, 1.0, 200 + i + seed), self.tensors(tokens, n, 1e-3, 300 + i + seed)))
        return caches, ins

    def block_step(self, caches, ins, had):
        for cache, (x, dy) in zip(caches, ins):
            self.linear_step(cache, x, dy, had)

    def config1_forward(self):
        """torch.manual_seed(0); x = randn(256, 1024) bf16, w = randn(1024, 1024) * 0.02
        bf16; both quantized (rowblock, round to nearest), dequantized, fp32 matmul, bf16 out."""
        import torch

        torch.manual_seed(0)
        x = torch.randn(256, 1024).bfloat16()
        w = (torch.randn(1024, 1024) * 0.02).bfloat16()
        if self.rnv is not None:
            r = self.rnv

            def fwd():
                gx, gw = r.global_scale_of(x), r.global_scale_of(w)
                a = r.dequantize(*r.ref_quantize_rowblock(x, gx), gx)
                b = r.dequantize(*r.ref_quantize_rowblock(w, gw), gw)
                return (a @ b.T).to(torch.bfloat16)
            return fwd
        O = self.O
        xf, wf = x.float().numpy(), w.float().numpy()

        def fwd():
            gx, gw = O.global_scale_of(xf), O.global_scale_of(wf)
            return O.dequantize(*O.quantize_rowblock(xf, gx), gx) @ O.dequantize(*O.quantize_rowblock(wf, gw), gw).T
        return fwd


def cpu_baseline(budget_s: float = 15.0) -> dict:
    """BASELINE config 1 (256 x 1024 x 1024 forward) through the host path, repeated for about
    `budget_s` seconds."""
    hp = _HostPath()
    fwd = hp.config1_forward()
    fwd()
    t0 = time.perf_counter()
    done = 0
    while time.perf_counter() - t0 < budget_s or done == 0:
        fwd()
        done += 1
    dt = (time.perf_counter() - t0) / done
    flops = 2.0 * 256 * 1024 * 1024
    what = ("radiance's own CPU emulation (baseline/_ref: global_scale_of, ref_quantize_rowblock, dequantize, "
            "fp32 matmul)") if hp.kind == "reference" else f"the oracle's numpy restatement ({hp.why})"
    return {
        "value": round(flops / dt / 1e12, 6),
        "unit": "TFLOPS",
        "cores": hp.cores,
        "kind": hp.kind,
        "sample": f"BASELINE config 1: {done} x one 256x1024x1024 NVFP4 linear forward (x, w quantized, dequantized, "
                  f"fp32 matmul) through {what}, {dt * 1e3:.2f} ms each, torch threads = {hp.cores}",
    }


def run_reference(args):
    """The reference arm: the config-3 block step (fwd + dgrad + wgrad of the four linears) through
    the host path, on a token sample sized so the whole run takes about two minutes.  Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    hp = _HostPath()
    had = hp.hadamard()
    caches, ins = hp.block(128)
    t0 = time.perf_counter()
    hp.block_step(caches, ins, had)
    per128 = time.perf_counter() - t0
    budget = 120.0 / max(args.steps + args.warmup, 1)
    tokens = int(max(128, min(16384, budget / max(per128, 1e-3) * 128)) // 128 * 128)
    if tokens != 128:
        _, ins = hp.block(tokens)
    for _ in range(args.warmup):
        hp.block_step(caches, ins, had)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        hp.block_step(caches, ins, had)
    dt = (time.perf_counter() - t0) / args.steps
    value = 6.0 * tokens * LAYER_KN / dt / 1e12
    what = ("radiance's own CPU emulation from baseline/_ref" if hp.kind == "reference"
            else f"the oracle's numpy restatement of radiance's CPU emulation ({hp.why})")
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
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "nvfp4 emulated in fp32 (quantize -> dequantize -> matmul)",
        "data": "synthetic (seeded; W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
        "config": {"workload": "config3 block linears fwd+dgrad+wgrad (qkv, o, gate_up, down), sampled tokens",
                   "tokens_per_step": tokens, "parallelism": "host CPU, rank 0 only",
                   "recipe": "stochastic rounding on dY, Hadamard on the wgrad operands; weight caches prepared "
                             "once (outside the step), as the per-optimizer-step refresh does"},
        "cpu_baseline": {
            "value": round(value, 6),
            "unit": "TFLOPS",
            "cores": hp.cores,
            "kind": hp.kind,
            "sample": f"the four config-3 linears fwd+dgrad+wgrad on {tokens} tokens per step through {what}",
        },
        "e2e": {"value": round(value, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------------
# Config 4: MoE expert FFN (grouped NVFP4 GEMMs), experts partitioned across ranks
# --------------------------------------------------------------------------------------------------
C4_D, C4_E, C4_FFN, C4_TOKENS, C4_TOPK = 2048, 8, 1408, 16384, 2
C4_ROUTED = C4_TOKENS * C4_TOPK
C4_FLOPS = 6.0 * C4_ROUTED * (C4_D * 2 * C4_FFN + C4_FFN * C4_D)  # 1.701e12 per step of the job
C4_METRIC = "NVFP4 MoE expert FFN fwd+bwd TFLOPS (BASELINE config 4: 8 experts, top-2 over 16384 tokens)"


def _c4_routing():
    """The job's routing: router logits ~N(0,1) (seed 0) for 16384 tokens, softmax, top-2."""
    import torch

    logits = torch.randn(C4_TOKENS, C4_E, generator=torch.Generator().manual_seed(0))
    return logits.softmax(-1).topk(C4_TOPK, dim=-1).indices


def _c4_source_pairs(top, s, world):
    """(token, expert) pairs of source rank s (tokens s*T/N ..), sorted expert-major then by token:
    the order of the source's send buffer."""
    import torch

    per = C4_TOKENS // world
    tok = torch.arange(s * per, (s + 1) * per).repeat_interleave(C4_TOPK)
    ex = top[s * per:(s + 1) * per].flatten()
    order = torch.argsort(ex * C4_TOKENS + tok)
    return tok[order], ex[order]


class _MoEFFN:
    """The expert FFN of config 4 for the experts of one rank: dispatch -> gate/up (grouped NVFP4)
    -> SwiGLU (one kernel, eager torch's roundings) -> down (grouped NVFP4) -> combine, the expert half of radiance's MoE layer
    (BatchedExperts.forward, src/radiance/model/ffn.py:148-153, with its [gate | up] split)."""

    def __init__(self, plan, w_gu, w_dn, device, recipe=None):
        import torch

        from radiance_b200.nvfp4.grouped import FP4GroupedLinear

        per = len(plan.experts)
        self.plan = plan
        self.gate_up = FP4GroupedLinear(per, C4_D, 2 * C4_FFN, recipe=recipe, device=device)
        self.down = FP4GroupedLinear(per, C4_FFN, C4_D, recipe=recipe, device=device)
        with torch.no_grad():
            self.gate_up.weight.copy_(w_gu[plan.experts])
            self.down.weight.copy_(w_dn[plan.experts])
        self.gate_up.refresh_fp4_cache()
        self.down.refresh_fp4_cache()

    def __call__(self, x_send, group=None):
        from radiance_b200.nvfp4 import swiglu
        from radiance_b200.nvfp4.expert_parallel import combine, dispatch

        x_exp = dispatch(x_send, self.plan, group)
        y_gu = self.gate_up(x_exp, self.plan.offsets)
        h = swiglu(y_gu, "split")  # F.silu(g) * u on the [gate | up] halves, one kernel each way
        return combine(self.down(h, self.plan.offsets), self.plan, group)


def measure_config4(args, rank, world, device, barrier, max_over_ranks, steps):
    """Config 4 for a fixed job of 16384 tokens: rank r routes tokens r*16384/N .. and owns experts
    r*8/N ..; the routed rows go to their expert's owner and back with all-to-alls (dispatch before
    gate/up, combine after down, the reverse pair for the gradients) inside the timed step.  With
    N > 1, rank 0 also checks that its tokens' forward output through the expert-parallel exchange
    equals the single-GPU expert FFN on the whole job, bit for bit.  Returns the record (rank 0)."""
    import torch

    from radiance_b200.nvfp4 import _trace
    from radiance_b200.nvfp4.expert_parallel import ExpertParallelPlan

    if C4_E % world or C4_TOKENS % world:
        raise SystemExit(f"config 4 needs the {C4_E} experts and {C4_TOKENS} tokens to divide over {world} ranks")
    top = _c4_routing()
    counts = [torch.bincount(_c4_source_pairs(top, s, world)[1], minlength=C4_E) for s in range(world)]
    plan = ExpertParallelPlan(counts, rank, world, device)
    gen = torch.Generator(device=device).manual_seed(404)  # every rank draws every expert's weights
    w_gu = torch.randn(C4_E, C4_D, 2 * C4_FFN, generator=gen, device=device) * 0.02
    w_dn = torch.randn(C4_E, C4_FFN, C4_D, generator=gen, device=device) * 0.02
    ffn = _MoEFFN(plan, w_gu, w_dn, device)
    x_job = torch.randn(C4_TOKENS, C4_D, generator=gen, device=device).to(torch.bfloat16)
    tok, _ex = _c4_source_pairs(top, rank, world)
    x_send = x_job[tok.to(device)]
    g_rank = torch.Generator(device=device).manual_seed(500 + rank)
    dy_send = (torch.randn(x_send.shape[0], C4_D, generator=g_rank, device=device) * 1e-3).to(torch.bfloat16)
    weights = (ffn.gate_up.weight, ffn.down.weight)

    def step():
        xs = x_send.detach().requires_grad_(True)
        y = ffn(xs)
        torch.autograd.grad(y, (xs, *weights), dy_send)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph = None
    run_step = step
    if world == 1 and not args.eager:
        graph = _capture(step)
        run_step = graph.replay
    ms, _clk = _timed_replays(run_step, steps, barrier)
    ms = max_over_ranks(ms) / steps
    with _trace.kernel_timer() as kt:
        step()
        per_kind = kt.summary()
    del graph

    parity = None
    if world > 1:
        with torch.no_grad():
            y_ep = ffn(x_send)
        if rank == 0:
            all_counts = [torch.bincount(top.flatten(), minlength=C4_E)]
            plan1 = ExpertParallelPlan(all_counts, 0, 1, device)
            ref = _MoEFFN(plan1, w_gu, w_dn, device)
            tok1, ex1 = _c4_source_pairs(top, 0, 1)
            with torch.no_grad():
                y_ref = ref(x_job[tok1.to(device)])
            keys1 = ex1 * C4_TOKENS + tok1  # sorted: the single-GPU row order
            tok0, ex0 = _c4_source_pairs(top, 0, world)
            rows = torch.searchsorted(keys1, ex0 * C4_TOKENS + tok0).to(device)
            parity = bool(torch.equal(y_ep, y_ref.index_select(0, rows)))
            del y_ep
            del ref, y_ref
        barrier()
    if rank != 0:
        return None
    peaks, peak_kind = _peaks()
    fp4_peak = 4.0 * peaks["bf16_tflops"]
    gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0, "work": 0.0})
    # The grouped launches' group sizes live on the device, so the kernel timer carries no work for
    # them: the GEMM work of this rank's step is its routed rows through both expert linears.
    gemm_work = gemm["work"] or 6.0 * plan.routed * (C4_D * 2 * C4_FFN + C4_FFN * C4_D)
    gemm_tflops = gemm_work / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else None
    rec = {
        "metric": C4_METRIC,
        "value": round(C4_FLOPS / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": steps,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "config": {
            "workload": "config4: MoE expert FFN (dispatch, grouped gate+up 2048->2816, fused SwiGLU, grouped down "
                        "1408->2048, combine) fwd+dgrad+wgrad via FP4GroupedLinear",
            "experts": C4_E, "experts_per_rank": C4_E // world, "top_k": C4_TOPK, "tokens_per_job": C4_TOKENS,
            "routed_rows_rank0": plan.routed, "padded_rows_rank0": plan.rows, "rank0_expert_rows": plan.expert_rows,
            "parallelism": f"expert-parallel ep{world} (NCCL all-to-all dispatch/combine)" if world > 1
            else "single GPU, all experts",
            "flops_basis": "6 x 32768 routed rows x (2048 x 2816 + 1408 x 2048) per job step; padding is overhead",
            "timing": "the step captured in one CUDA graph, replayed" if world == 1 and not args.eager
            else "eager Python step loop around NCCL",
        },
        "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 4)} for k, v in per_kind.items()},
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
        "gpu_launches": kt.launches * steps,
    }
    if parity is not None:
        rec["parity_ok"] = parity
        rec["parity"] = ("rank 0's tokens: forward output through dispatch/experts/combine equals the single-GPU "
                         "expert FFN over the whole job, bit for bit")
    return rec


def _dist_helpers(world, device):
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    return barrier, max_over_ranks


def run_config4(args):
    import torch
    import torch.distributed as dist

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    barrier, max_over_ranks = _dist_helpers(world, device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    clocks.start()
    rec = measure_config4(args, rank, world, device, barrier, max_over_ranks, max(3, min(args.steps, 50)))
    clk = clocks.stop()
    if rank == 0:
        rec.update({"warmup": args.warmup, "vs_baseline": None,
                    "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
                    "data": "synthetic (seeded; router logits ~N(0,1), W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))",
                    "clocks": clk})
        print(json.dumps(rec), flush=True)
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


def measure_config5(args, rank, world, device, barrier, max_over_ranks, steps):
    """One step = the block's four linears fwd + dgrad + wgrad for a fixed 65536-token job.  QKV,
    O and down are token-sharded (65536/N rows per rank); their fp32 weight gradients are
    reduce-scattered over the ranks inside the step (NCCL on a side stream, from the wgrad hooks).
    The largest layer, gate/up (4096 -> 28672), is split along N: every rank holds 28672/N rows of
    the weight (quantized with the full weight's global scale), computes its column slice for all
    65536 rows and all-gathers the bf16 output (fused into the GEMM epilogue, or NCCL); the partial
    input gradients are all-reduced.  Total work is fixed as N grows (strong scaling).  With N > 1,
    rank 0 checks that the N-split layer's output rows equal the unsplit FP4Linear's (same full-input
    global scale), bit for bit.  Returns the record (rank 0)."""
    import torch
    import torch.distributed as dist

    from radiance_b200 import nvfp4 as nv
    from radiance_b200.nvfp4 import _trace
    from radiance_b200.nvfp4.nsplit import FP4ColumnParallelLinear

    if C5_TOKENS % (128 * world):
        raise SystemExit(f"config 5 needs 65536 tokens to shard into multiples of 128 over {world} ranks")
    m_local = C5_TOKENS // world
    # gate_up is N-split over groups of `nsr` ranks (all of them by default).  With nsr < N the split
    # is 2-D: the job's tokens are divided over the N / nsr groups, each group N-splits gate_up over
    # its own tokens (replicated inside the group), and each weight slice's fp32 gradient is
    # reduce-scattered over the groups (the ranks holding the same slice).
    nsr = args.c5_nsplit_ranks if 0 < args.c5_nsplit_ranks < world else world
    if world % nsr or (C5_NSPLIT[0][2] // nsr) % (128 * (world // nsr)):
        raise SystemExit(f"config 5: --c5-nsplit-ranks {nsr} does not divide {world} ranks and gate_up's rows")
    n_groups = world // nsr
    split_group, slice_group = None, None
    if n_groups > 1:
        for g0 in range(n_groups):  # every rank creates every group, in the same order
            grp = dist.new_group(list(range(g0 * nsr, (g0 + 1) * nsr)))
            if rank // nsr == g0:
                split_group = grp
        for s0 in range(nsr):
            grp = dist.new_group(list(range(s0, world, nsr)))
            if rank % nsr == s0:
                slice_group = grp
    # The N-split layer's rows (this group's share of the job's tokens) are replicated over the
    # group: every rank computes its column slice of gate_up for all of them.
    m_ffn = C5_TOKENS // n_groups
    gen = torch.Generator(device=device).manual_seed(777)  # same on every rank: replicated weights/rows
    gen_ffn = gen if n_groups == 1 else torch.Generator(device=device).manual_seed(5000 + rank // nsr)
    layers, inputs, grads = [], [], []
    side = torch.cuda.Stream(device)
    shards, pending = [], []
    for name, k, n in C5_TOKEN_SHARDED:
        lin = nv.FP4Linear(k, n, bias=False, device=device)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, device=device, generator=gen) * 0.02)
        lin.refresh_fp4_cache()
        if world > 1:
            shard = torch.empty(n // world, k, device=device)
            shards.append(shard)

            def hook(grad_w, shard=shard):
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    dist.reduce_scatter_tensor(shard, grad_w)
                pending.append(grad_w)
            lin.wgrad_hook = hook
        layers.append((lin, lin.weight))
        g_local = torch.Generator(device=device).manual_seed(1000 + rank)
        inputs.append(torch.randn(m_local, k, device=device, generator=g_local).to(torch.bfloat16))
        grads.append((torch.randn(m_local, n, device=device, generator=g_local) * 1e-3).to(torch.bfloat16))
    full_w = None
    for name, k, n in C5_NSPLIT:
        lin = FP4ColumnParallelLinear(k, n, group=split_group, device=device, fused_gather=args.nsplit == "fused")
        full_w = torch.randn(n, k, device=device, generator=gen) * 0.02
        lin.load_full_weight(full_w)
        lin.refresh_fp4_cache()
        if n_groups > 1:
            shard = torch.empty(n // nsr // n_groups, k, device=device)
            shards.append(shard)

            def slice_hook(grad_w, shard=shard):
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    dist.reduce_scatter_tensor(shard, grad_w, group=slice_group)
                pending.append(grad_w)
            lin.local.wgrad_hook = slice_hook
        layers.append((lin, lin.local.weight))
        inputs.append(torch.randn(m_ffn, k, device=device, generator=gen_ffn).to(torch.bfloat16))
        grads.append((torch.randn(m_ffn, n, device=device, generator=gen_ffn) * 1e-3).to(torch.bfloat16))
    flops_rank = 6.0 * (m_local * sum(k * n for _, k, n in C5_TOKEN_SHARDED)
                        + m_ffn * sum(k * n for _, k, n in C5_NSPLIT) / nsr)
    gather_bytes = sum(m_ffn * n * 2 * (nsr - 1) // nsr for _, k, n in C5_NSPLIT) if nsr > 1 else 0
    reduce_bytes = sum(m_ffn * k * 2 for _, k, n in C5_NSPLIT) if nsr > 1 else 0
    wgrad_rs_bytes = sum(n * k * 4 for _, k, n in C5_TOKEN_SHARDED) if world > 1 else 0
    if n_groups > 1:
        wgrad_rs_bytes += sum(n // nsr * k * 4 for _, k, n in C5_NSPLIT)

    def step():
        for (lin, w), x0, dy in zip(layers, inputs, grads):
            x = x0.detach().requires_grad_(True)
            y = lin(x)
            torch.autograd.grad(y, (x, w), dy)
            del y
        if world > 1:
            torch.cuda.current_stream().wait_stream(side)
            pending.clear()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
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
    ms = max_over_ranks(start.elapsed_time(stop)) / steps
    per_kind = kt.summary()
    parity = None
    if world > 1:
        lin = layers[-1][0]
        with torch.no_grad():
            y_split = lin(inputs[-1])
            if rank == 0:
                k, n = C5_NSPLIT[0][1], C5_NSPLIT[0][2]
                ref = nv.FP4Linear(k, n, bias=False, device=device)
                ref.weight.copy_(full_w)
                ref.refresh_fp4_cache()
                gs = nv.global_scale_of(inputs[-1])
                y_ref = ref(inputs[-1][:4096], global_scale=gs)
                parity = bool(torch.equal(y_split[:4096], y_ref))
                del ref, y_ref
            del y_split
        barrier()
        for lin, _w in layers:
            if isinstance(lin, FP4ColumnParallelLinear):
                lin.local.wgrad_hook = None
                lin.close()
            else:
                lin.wgrad_hook = None
    if rank != 0:
        return None
    peaks, peak_kind = _peaks()
    fp4_peak = 4.0 * peaks["bf16_tflops"]
    gemm = per_kind.get("gemm", {"launches": 0, "ms": 0.0, "work": 0.0})
    gemm_tflops = gemm["work"] / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else None
    rec = {
        "metric": C5_METRIC,
        "value": round(C5_FLOPS / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": steps,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "config": {
            "workload": "config5: d_model 4096 block linears fwd+dgrad+wgrad; QKV/O/down token-sharded with their "
                        "fp32 dW reduce-scattered in the step, gate_up (the largest) N-split with an all-gather of "
                        "its bf16 output",
            "tokens_per_job": C5_TOKENS, "attention_rows_per_rank": m_local, "ffn_rows": m_ffn,
            "layers": {n: [k, o] for n, k, o in C5_TOKEN_SHARDED + C5_NSPLIT},
            "flops_per_rank_per_step": flops_rank,
            "allgather_bytes_received_per_rank_per_step": gather_bytes,
            "dgrad_allreduce_bytes_per_rank_per_step": reduce_bytes,
            "wgrad_reduce_scatter_bytes_per_step": wgrad_rs_bytes,
            "parallelism": (f"gate_up N-split over {world} + token-sharded QKV/O/down" if n_groups == 1 else
                            f"2-D: gate_up N-split over groups of {nsr} ranks, the job's tokens over the {n_groups} "
                            f"groups, each slice's fp32 dW reduce-scattered over the groups; token-sharded QKV/O/down"),
            "nsplit_gather": ("GEMM epilogue stores each tile into every rank's output over NVLink "
                              "(rb_nvfp4_gemm_allgather, IPC-shared buffers)") if args.nsplit == "fused"
            else "NCCL all_gather_into_tensor + column permute",
            "timing": "eager Python step loop (CUDA events around the K steps; per-kernel events inside)",
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
    }
    if parity is not None:
        rec["parity_ok"] = parity
        rec["parity"] = ("rank 0: rows 0..4095 of the N-split gate_up output (every rank's slice, gathered) equal "
                         "the unsplit FP4Linear's with the same full-input global scale, bit for bit")
    return rec


def run_config5(args):
    import torch
    import torch.distributed as dist

    rank, world, local = _dist_setup(args)
    device = torch.device("cuda", local if world > 1 else 0)
    barrier, max_over_ranks = _dist_helpers(world, device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = visible.split(",")[torch.cuda.current_device()] if visible else str(torch.cuda.current_device())
    clocks = ClockSampler(phys)
    clocks.start()
    rec = measure_config5(args, rank, world, device, barrier, max_over_ranks, max(3, min(args.steps, 20)))
    clk = clocks.stop()
    if rank == 0:
        rec.update({"warmup": args.warmup, "vs_baseline": None,
                    "dtype": "nvfp4 (e2m1 x e4m3 block scales, fp32 accumulate; bf16 in/out, fp32 dW)",
                    "data": "synthetic (seeded; W~N(0,0.02), X~N(0,1), dY~N(0,1e-3))", "clocks": clk})
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------------------
# Profiling cases: one kernel's fixed workload at a time (for ncu, or timed with --time)
# --------------------------------------------------------------------------------------------------
CASES_DOC = """python bench.py case <name> [options]

One kernel's fixed workload, run --iters times with nothing else in between and between
cudaProfilerStart/Stop (so `ncu --profile-from-start off` captures only those launches), or, with
--time, captured in a CUDA graph, replayed and timed with CUDA events (one JSON line).

  quant        one quantization per iteration: --rows --cols --form row|col|both --hadamard --sr
               --scale given (a precomputed global scale) | auto (the fused global-scale quantizer)
               | separate (the amax kernel, then the quantizer)
  gemm         one block-scaled GEMM, bf16 out: --m --n --k; --variant cublas runs cuBLASLt's NVFP4
               GEMM (torch._scaled_mm_v2) on the same operands instead, for comparison
  swiglu       the SwiGLU producer of a config-3 FFN: --variant fused (the gate/up GEMM whose epilogue
               writes h and its global scale) | unfused (GEMM, torch F.silu(g) * u, amax); each then
               quantizes h both ways; --variant fused-gemm times the SwiGLU GEMM alone
  block-gemms  the twelve GEMMs of one config-3 block step (four linears x fwd, dgrad, wgrad): --tokens
  swiglu-bwd   the fused SwiGLU backward (grad_gu and its global scale): --m --hidden
  block-step   one whole config-3 block step (QKV, O, fused FFN; forward then backward): --tokens

Inputs are seeded synthetic tensors (activations ~N(0, 1), weights ~N(0, 0.02)); a timed case reuses
its inputs every iteration."""


def _case_quant(args, dev):
    import torch

    from radiance_b200.nvfp4.quantize import (col_scale_bytes, global_scale_of, hadamard_matrix,
                                              quantize_auto_scale_into_, quantize_into_, row_scale_bytes)

    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(args.rows, args.cols, generator=g).to(dev, torch.bfloat16)
    gs = global_scale_of(x)
    h = hadamard_matrix(device=dev) if args.hadamard else None
    seed = torch.tensor(3, device=dev, dtype=torch.int64)
    row = (torch.empty(args.rows, args.cols // 2, dtype=torch.uint8, device=dev),
           torch.empty(row_scale_bytes(args.rows, args.cols), dtype=torch.uint8, device=dev))
    col = (torch.empty(args.cols, args.rows // 2, dtype=torch.uint8, device=dev),
           torch.empty(col_scale_bytes(args.rows, args.cols), dtype=torch.uint8, device=dev))
    r = row if args.form in ("row", "both") else None
    c = col if args.form in ("col", "both") else None

    def run():
        if args.scale == "auto":
            quantize_auto_scale_into_(x, out_scale=gs, row=r, col=c, hadamard=h, stochastic=args.sr, seed=seed)
            return
        if args.scale == "separate":
            global_scale_of(x, out=gs)
        quantize_into_(x, global_scale=gs, row=r, col=c, hadamard=h, stochastic=args.sr, seed=seed)

    forms = (r is not None) + (c is not None)
    return run, {"work": args.rows * args.cols * (2 + 0.5625 * forms), "unit": "GB/s",
                 "basis": "algorithmic bytes of the quantizer: 2 B read + 0.5625 B written per element and form"}


def _operands(m, n, k, dev, g, a_scale=1.0, b_scale=0.02):
    import torch

    from radiance_b200.nvfp4.quantize import quantize

    a = quantize((torch.randn(m, k, generator=g) * a_scale).to(dev, torch.bfloat16), -1)
    b = quantize((torch.randn(n, k, generator=g) * b_scale).to(dev, torch.bfloat16), -1)
    return a, b


def _case_gemm(args, dev):
    import torch

    from radiance_b200.nvfp4.quantize import _gemm

    g = torch.Generator(device="cpu").manual_seed(11)
    a, b = _operands(args.m, args.n, args.k, dev, g)
    out = torch.empty(args.m, args.n, dtype=torch.bfloat16, device=dev)
    if args.variant == "cublas":
        from torch._C import _ScalingType, _SwizzleType

        blk = [_ScalingType.BlockWise1x16.value]
        swz = [_SwizzleType.SWIZZLE_32_4_4.value]

        def run():
            torch._scaled_mm_v2(a.packed, b.packed.t(), scale_a=[a.scale], recipe_a=blk, swizzle_a=swz,
                                scale_b=[b.scale], recipe_b=blk, swizzle_b=swz, bias=None, out_dtype=torch.bfloat16)
    else:
        def run():
            _gemm(a.packed.view(torch.uint8), a.scale.view(torch.uint8), b.packed.view(torch.uint8),
                  b.scale.view(torch.uint8), a.global_scale, b.global_scale, None, torch.bfloat16, out)
    return run, {"work": 2.0 * args.m * args.n * args.k, "unit": "TFLOP/s", "basis": "2*M*N*K"}


def _case_swiglu(args, dev):
    import torch
    import torch.nn.functional as F

    from radiance_b200.nvfp4.quantize import (_gemm, col_scale_bytes, global_scale_of, hadamard_matrix,
                                              interleave_gate_up, quantize, quantize_into_, row_scale_bytes,
                                              swiglu_mm)

    g = torch.Generator(device="cpu").manual_seed(17)
    m, k, hid = args.m, args.k, args.hidden
    xq = quantize(torch.randn(m, k, generator=g).to(dev, torch.bfloat16), -1)
    w = interleave_gate_up((torch.randn(hid, k, generator=g) * 0.02).to(dev, torch.bfloat16),
                           (torch.randn(hid, k, generator=g) * 0.02).to(dev, torch.bfloat16))
    wq = quantize(w, -1)
    gu = torch.empty(m, 2 * hid, dtype=torch.bfloat16, device=dev)
    h = torch.empty(m, hid, dtype=torch.bfloat16, device=dev)
    gs = torch.empty((), dtype=torch.float32, device=dev)
    rot = hadamard_matrix(device=dev)
    row = (torch.empty(m, hid // 2, dtype=torch.uint8, device=dev),
           torch.empty(row_scale_bytes(m, hid), dtype=torch.uint8, device=dev))
    col = (torch.empty(hid, m // 2, dtype=torch.uint8, device=dev),
           torch.empty(col_scale_bytes(m, hid), dtype=torch.uint8, device=dev))

    def run():
        if args.variant == "fused-gemm":  # the SwiGLU GEMM alone
            swiglu_mm(xq, wq, out=gu, h=h, h_global_scale=gs)
            return
        if args.variant == "fused":
            swiglu_mm(xq, wq, out=gu, h=h, h_global_scale=gs)
            hh = h
        else:  # separate gate_proj / up_proj outputs, as radiance has them
            _gemm(xq.packed.view(torch.uint8), xq.scale.view(torch.uint8), wq.packed.view(torch.uint8),
                  wq.scale.view(torch.uint8), xq.global_scale, wq.global_scale, None, torch.bfloat16, gu)
            hh = F.silu(gu[:, :hid]) * gu[:, hid:]
            global_scale_of(hh, out=gs)
        quantize_into_(hh, global_scale=gs, row=row, col=col, hadamard=rot)

    return run, {"work": 2.0 * m * 2 * hid * k, "unit": "TFLOP/s", "basis": "2*M*N*K of the gate/up GEMM"}


def _case_block_gemms(args, dev):
    """Per linear (in k, out n, T tokens): fwd (T x n x k, bf16 out), dgrad (T x k x n, bf16 out),
    wgrad (n x k x T, fp32 out) -- the three ``mm`` calls of ``_FP4LinearFn``."""
    import torch

    from radiance_b200.nvfp4.quantize import _gemm

    g = torch.Generator(device="cpu").manual_seed(13)
    tokens = args.tokens
    calls = []
    for _, k, n in LAYERS:
        for (m_, n_, k_, out_dtype) in ((tokens, n, k, torch.bfloat16), (tokens, k, n, torch.bfloat16),
                                        (n, k, tokens, torch.float32)):
            a, b = _operands(m_, n_, k_, dev, g)
            out = torch.empty(m_, n_, dtype=out_dtype, device=dev)
            calls.append((a, b, out, out_dtype))

    def run():
        for a, b, out, out_dtype in calls:
            _gemm(a.packed.view(torch.uint8), a.scale.view(torch.uint8), b.packed.view(torch.uint8),
                  b.scale.view(torch.uint8), a.global_scale, b.global_scale, None, out_dtype, out)

    return run, {"work": 6.0 * tokens * LAYER_KN, "unit": "TFLOP/s", "basis": "6*T*sum(K*N) over the four linears"}


def _case_swiglu_bwd(args, dev):
    """The fused SwiGLU backward of a config-3 FFN: grad_h (--m x --hidden) and the interleaved
    pre-activations in, grad_gu and its global scale out."""
    import torch

    from radiance_b200.nvfp4.quantize import swiglu_backward

    g = torch.Generator(device="cpu").manual_seed(19)
    gu = (torch.randn(args.m, 2 * args.hidden, generator=g) * 2).to(dev, torch.bfloat16)
    gh = (torch.randn(args.m, args.hidden, generator=g) * 1e-3).to(dev, torch.bfloat16)
    out = torch.empty_like(gu)
    gs = torch.empty((), dtype=torch.float32, device=dev)
    return (lambda: swiglu_backward(gh, gu, out=out, out_scale=gs)), {
        "work": args.m * args.hidden * 2 * 4.0, "unit": "GB/s",
        "basis": "8 B per hidden unit: grad_h, g, u read and grad_g, grad_u written, bf16"}


def _case_block_step(args, dev):
    """One config-3 block step (QKV, O, the fused FFN; forward then backward) on --tokens tokens,
    one GPU, no collective."""
    block = Block(dev, ffn=True)
    xs_host, dys_host = block.inputs(args.tokens, seed=1000)
    xs = [x.to(dev) for x in xs_host]
    dys = [d.to(dev) for d in dys_host]
    step = BlockStep(block, 1, dev)
    return (lambda: step(xs, dys)), {"work": 6.0 * args.tokens * LAYER_KN, "unit": "TFLOP/s",
                                     "basis": "6*T*sum(K*N) over the block's four linears"}


def run_case(argv):
    import torch

    ap = argparse.ArgumentParser(prog="bench.py case", description=CASES_DOC,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("name", choices=["quant", "gemm", "swiglu", "swiglu-bwd", "block-gemms", "block-step"])
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=6144)
    ap.add_argument("--form", choices=["row", "col", "both"], default="both")
    ap.add_argument("--hadamard", action="store_true")
    ap.add_argument("--sr", action="store_true")
    ap.add_argument("--scale", choices=["given", "auto", "separate"], default="given")
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=5632)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--variant", default="ours", help="gemm: ours|cublas; swiglu: fused|fused-gemm|unfused")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="graph-capture the iterations and time them (one JSON line)")
    args = ap.parse_args(argv)
    if args.name == "swiglu" and args.variant == "ours":
        args.variant = "fused"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    run, info = {"quant": _case_quant, "gemm": _case_gemm, "swiglu": _case_swiglu,
                 "swiglu-bwd": _case_swiglu_bwd, "block-gemms": _case_block_gemms,
                 "block-step": _case_block_step}[args.name](args, dev)
    if not args.time:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(args.iters):
            run()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return
    reps = max(args.iters, 3)
    for _ in range(3):
        run()
    graph = _capture(lambda: [run() for _ in range(reps)])
    graph.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
        best = ms if best is None else min(best, ms)
    scale = 1e9 if info["unit"] == "GB/s" else 1e12
    print(json.dumps({"case": args.name, "args": {k: v for k, v in vars(args).items() if k != "time"},
                      "us_per_iter": round(best * 1e3, 2), "value": round(info["work"] / (best * 1e-3) / scale, 1),
                      "unit": info["unit"], "basis": info["basis"],
                      "timing": f"{reps} iterations per CUDA graph replay, best of 5 replays"}), flush=True)


def main():
    if sys.argv[1:2] == ["case"]:
        run_case(sys.argv[2:])
        return
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--tokens-per-rank", type=int, default=0,
                    help="config 3: run this many tokens on every rank instead of sharding the job's 16384 "
                         "(weak scaling; no gradient reduction unless N > 1)")
    ap.add_argument("--comm-sms", type=int, default=-1,
                    help="config 3, N > 1: SMs left to the gradient reduce-scatter (its communicator's CTA limit; "
                         "this library's kernels size their grids for the rest); default by N: "
                         "16 at N=2, 24 at N=4, 32 at N=8")
    ap.add_argument("--linears-only", action="store_true",
                    help="config 3: the four linears on independent inputs instead of QKV, O and the fused FFN")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="config 3: skip the config 4 and config 5 sub-records of the headline line")
    ap.add_argument("--eager", action="store_true",
                    help="config 3: time the Python step loop instead of a captured CUDA graph of the step")
    ap.add_argument("--nsplit", choices=["fused", "nccl"], default="fused",
                    help="config 5: the N-split layer's output all-gather (fused into the GEMM, or NCCL)")
    ap.add_argument("--c5-nsplit-ranks", type=int, default=0,
                    help="config 5: N-split gate_up over groups of this many ranks and divide the tokens over the "
                         "groups (a 2-D split); 0 = one group of all ranks")
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
