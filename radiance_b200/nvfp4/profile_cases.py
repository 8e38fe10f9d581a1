"""Fixed workloads for profiling the NVFP4 kernels one at a time (for example under ``ncu``).

Each case allocates its inputs once, runs the kernel(s) ``--iters`` times with nothing else in
between and exits, so a profiler can skip and capture launches by count:

    python -m radiance_b200.nvfp4.profile_cases quant --rows 16384 --cols 6144 --hadamard --sr
        one fused quantization (rowblock + colblock) per iteration
    python -m radiance_b200.nvfp4.profile_cases gemm --m 16384 --n 6144 --k 2048
        one block-scaled GEMM (bf16 out) per iteration; ``--impl cublas`` runs cuBLASLt's NVFP4
        GEMM (torch._scaled_mm_v2) on the same operands instead, for comparison
    python -m radiance_b200.nvfp4.profile_cases swiglu --m 16384 --k 2048 --hidden 5632
        the SwiGLU producer of a config-3 FFN per iteration: ``--impl fused`` runs the gate/up GEMM
        whose epilogue writes h and its global scale (``swiglu_mm``); ``--impl unfused`` runs the
        plain GEMM, torch's F.silu(g) * u and the global-scale pass; each then quantizes h both
        ways (down_proj's forward operand and saved wgrad operand)
    python -m radiance_b200.nvfp4.profile_cases block-gemms
        the twelve GEMMs of one config-3 block step (four linears x fwd, dgrad, wgrad) per
        iteration, with the operand shapes and output types ``FP4Linear`` uses

Inputs are seeded synthetic tensors (activations ~N(0, 1), weights ~N(0, 0.02)).  The iterations
run between cudaProfilerStart and cudaProfilerStop, so ``ncu --profile-from-start off`` captures
only them (not the operand preparation).
"""

from __future__ import annotations

import argparse

import torch

from .quantize import (_gemm, col_scale_bytes, global_scale_of, hadamard_matrix, interleave_gate_up, quantize,
                       quantize_into_, row_scale_bytes, swiglu_mm)

BLOCK_LAYERS = [("qkv", 2048, 6144), ("o", 2048, 2048), ("gate_up", 2048, 11264), ("down", 5632, 2048)]


def _quant_case(args, dev):
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(args.rows, args.cols, generator=g).to(dev, torch.bfloat16)
    gs = global_scale_of(x)
    h = hadamard_matrix(device=dev) if args.hadamard else None
    seed = torch.tensor(3, device=dev, dtype=torch.int64)
    row = (torch.empty(args.rows, args.cols // 2, dtype=torch.uint8, device=dev),
           torch.empty(row_scale_bytes(args.rows, args.cols), dtype=torch.uint8, device=dev))
    col = (torch.empty(args.cols, args.rows // 2, dtype=torch.uint8, device=dev),
           torch.empty(col_scale_bytes(args.rows, args.cols), dtype=torch.uint8, device=dev))
    form = args.form
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.iters):
        quantize_into_(x, global_scale=gs, row=row if form in ("row", "both") else None,
                       col=col if form in ("col", "both") else None, hadamard=h, stochastic=args.sr, seed=seed)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def _operands(m, n, k, dev, g, a_scale=1.0, b_scale=0.02):
    a = quantize((torch.randn(m, k, generator=g) * a_scale).to(dev, torch.bfloat16), -1)
    b = quantize((torch.randn(n, k, generator=g) * b_scale).to(dev, torch.bfloat16), -1)
    return a, b


def _gemm_case(args, dev):
    g = torch.Generator(device="cpu").manual_seed(11)
    a, b = _operands(args.m, args.n, args.k, dev, g)
    out = torch.empty(args.m, args.n, dtype=torch.bfloat16, device=dev)
    if args.impl == "cublas":
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
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.iters):
        run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def _swiglu_case(args, dev):
    import torch.nn.functional as F

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
        if args.impl == "fused":
            swiglu_mm(xq, wq, out=gu, h=h, h_global_scale=gs)
            hh = h
        else:  # separate gate_proj / up_proj outputs, as radiance has them
            _gemm(xq.packed.view(torch.uint8), xq.scale.view(torch.uint8), wq.packed.view(torch.uint8),
                  wq.scale.view(torch.uint8), xq.global_scale, wq.global_scale, None, torch.bfloat16, gu)
            hh = F.silu(gu[:, :hid]) * gu[:, hid:]
            global_scale_of(hh, out=gs)
        quantize_into_(hh, global_scale=gs, row=row, col=col, hadamard=rot)

    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.iters):
        run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def _block_gemms_case(args, dev):
    """Per linear (in k, out n, T tokens): fwd (T x n x k, bf16 out), dgrad (T x k x n, bf16 out),
    wgrad (n x k x T, fp32 out) -- the three ``mm`` calls of ``_FP4LinearFn``."""
    g = torch.Generator(device="cpu").manual_seed(13)
    tokens = args.tokens
    calls = []
    for _, k, n in BLOCK_LAYERS:
        for (m_, n_, k_, out_dtype) in ((tokens, n, k, torch.bfloat16), (tokens, k, n, torch.bfloat16),
                                        (n, k, tokens, torch.float32)):
            a, b = _operands(m_, n_, k_, dev, g)
            out = torch.empty(m_, n_, dtype=out_dtype, device=dev)
            calls.append((a, b, out, out_dtype))
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.iters):
        for a, b, out, out_dtype in calls:
            _gemm(a.packed.view(torch.uint8), a.scale.view(torch.uint8), b.packed.view(torch.uint8),
                  b.scale.view(torch.uint8), a.global_scale, b.global_scale, None, out_dtype, out)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="case", required=True)
    pq = sub.add_parser("quant")
    pq.add_argument("--rows", type=int, default=16384)
    pq.add_argument("--cols", type=int, default=6144)
    pq.add_argument("--form", choices=["row", "col", "both"], default="both")
    pq.add_argument("--hadamard", action="store_true")
    pq.add_argument("--sr", action="store_true")
    pq.add_argument("--iters", type=int, default=3)
    pg = sub.add_parser("gemm")
    pg.add_argument("--m", type=int, default=16384)
    pg.add_argument("--n", type=int, default=6144)
    pg.add_argument("--k", type=int, default=2048)
    pg.add_argument("--iters", type=int, default=3)
    pg.add_argument("--impl", choices=["ours", "cublas"], default="ours")
    ps = sub.add_parser("swiglu")
    ps.add_argument("--m", type=int, default=16384)
    ps.add_argument("--k", type=int, default=2048)
    ps.add_argument("--hidden", type=int, default=5632)
    ps.add_argument("--iters", type=int, default=3)
    ps.add_argument("--impl", choices=["fused", "unfused"], default="fused")
    pb = sub.add_parser("block-gemms")
    pb.add_argument("--tokens", type=int, default=16384)
    pb.add_argument("--iters", type=int, default=2)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    {"quant": _quant_case, "gemm": _gemm_case, "swiglu": _swiglu_case, "block-gemms": _block_gemms_case}[args.case](
        args, dev)


if __name__ == "__main__":
    main()
