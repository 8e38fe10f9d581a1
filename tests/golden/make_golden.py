"""Generate ``nvfp4_golden.npz`` from the reference implementation itself.

Run in a container that has the reference checkout (jamespa16/radiance) on disk::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/radiance

It imports ``radiance.nvfp4`` from ``<radiance>/src`` (the pure-torch emulation in
``src/radiance/nvfp4/quantize.py``) and records, for seeded inputs, exactly what the reference
computes: global scales, packed e2m1 nibbles, swizzled e4m3 scale bytes (row, col and
col+Hadamard forms), stochastic-rounding results for a stored uniform draw, the SWIZZLE_32_4_4
permutation, the RNE tie table, the Hadamard matrix, and BASELINE config 1's forward output.
The fixture is what pins ``oracle/nvfp4_oracle.py`` (``tests/test_oracle_golden.py``); the GPU
tests then compare the CUDA kernels with the oracle.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch


def _bits(x: torch.Tensor) -> np.ndarray:
    if x.dtype == torch.bfloat16:
        return x.view(torch.int16).numpy().view(np.uint16).copy()
    return x.float().numpy().copy()


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from radiance import nvfp4  # noqa: E402  (the reference)

    out: dict[str, np.ndarray] = {}
    h0 = nvfp4.hadamard_matrix(nvfp4.BLOCK)  # seed 0: what FP4Linear registers
    h1 = nvfp4.hadamard_matrix(nvfp4.BLOCK, seed=1)  # the tests' mismatched rotation
    out["hadamard_seed0"] = h0.numpy()
    out["hadamard_seed1"] = h1.numpy()

    cases = []

    def add_quant_case(name: str, x: torch.Tensor, with_sr: bool = False) -> None:
        cases.append(name)
        out[f"{name}/x"] = _bits(x)
        out[f"{name}/dtype"] = np.array(0 if x.dtype == torch.bfloat16 else 1)
        gs = nvfp4.global_scale_of(x)
        out[f"{name}/gs"] = gs.numpy().astype(np.float32).reshape(())
        for tag, axis, had in (("row", -1, None), ("col", 0, None), ("colh", 0, h0), ("colh1", 0, h1)):
            q = nvfp4.quantize_reference(x, axis, global_scale=gs, hadamard=had)
            out[f"{name}/{tag}_packed"] = q.packed.view(torch.uint8).numpy().copy()
            out[f"{name}/{tag}_scale"] = q.scale.view(torch.uint8).numpy().copy()
        if with_sr:
            u = torch.rand(x.shape, generator=torch.Generator().manual_seed(7))
            out[f"{name}/u"] = u.numpy().copy()
            p, s = nvfp4.ref_quantize_rowblock(x, gs, u=u)
            out[f"{name}/sr_row_packed"] = p.view(torch.uint8).numpy().copy()
            out[f"{name}/sr_row_scale"] = nvfp4.ref_to_blocked(s).view(torch.uint8).numpy().copy()
            p, s = nvfp4.ref_quantize_colblock(x, gs, hadamard=h0, u=u)
            out[f"{name}/sr_colh_packed"] = p.view(torch.uint8).numpy().copy()
            out[f"{name}/sr_colh_scale"] = nvfp4.ref_to_blocked(s).view(torch.uint8).numpy().copy()

    # The reference's own bit-exact matrix (tests/test_nvfp4.py:277-295), at fixture-friendly sizes.
    for i, (shape, dtype) in enumerate(
        [
            ((128, 64), torch.bfloat16),
            ((256, 128), torch.bfloat16),
            ((128, 1408), torch.bfloat16),
            ((384, 640), torch.bfloat16),
            ((128, 64), torch.float32),
            ((256, 128), torch.float32),
        ]
    ):
        torch.manual_seed(100 + i)
        add_quant_case(f"rand{i}", torch.randn(*shape).to(dtype), with_sr=(i == 1))

    # Magnitude sweep (tests/test_nvfp4.py:298-311).
    for e in (-4, -2, 0, 2, 4):
        torch.manual_seed(200 + e)
        add_quant_case(f"mag{e:+d}", (torch.randn(256, 256) * 10.0**e).bfloat16())

    # Zero blocks (tests/test_nvfp4.py:114-129, :366-383).
    torch.manual_seed(300)
    x = torch.randn(256, 128).bfloat16()
    x[:, :16] = 0.0
    x[:16, :] = 0.0
    add_quant_case("zeroblk", x)
    add_quant_case("allzero", torch.zeros(256, 128, dtype=torch.bfloat16))

    # Outlier channels, as in BASELINE config 2 (0.1% of channels x20).
    torch.manual_seed(400)
    x = torch.randn(128, 2048)
    ch = torch.randperm(2048, generator=torch.Generator().manual_seed(401))[:2]
    x[:, ch] *= 20.0
    add_quant_case("outlier", x.bfloat16())

    # Signed zeros, bf16 subnormals next to huge values, and exact e2m1 ties.
    torch.manual_seed(500)
    x = torch.randn(256, 128) * 1e30
    x[0::7, 1::5] = -0.0
    x[3::11, 2::3] = 1e-39
    x[5::13, 4::7] = -1e-39
    x[1::9, :] = torch.randn(1, 128) * 1e-36
    add_quant_case("edge", x.bfloat16())
    # Negative zeros inside ordinary blocks (the reference's code for q = -0 is 0: its sign is
    # q < 0), plus whole blocks and one column of -0.
    torch.manual_seed(502)
    x = torch.randn(256, 128)
    x[0::3, 2::5] = -0.0
    x[16:32, 40:56] = -0.0
    x[:, 77] = -0.0
    add_quant_case("negzero", x.bfloat16())
    torch.manual_seed(501)
    lv = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 3.0])
    x = lv[torch.randint(0, len(lv), (256, 128))] * torch.where(torch.rand(256, 128) < 0.5, -1.0, 1.0)
    x[:, 0::16] = 6.0  # every block's amax is 6 -> scale 1/gs-exact, so the listed values are ties
    add_quant_case("ties", x.bfloat16())

    out["cases"] = np.array(cases)

    # SWIZZLE_32_4_4 (tests/test_nvfp4.py:84-101).
    for rows, cols in [(128, 4), (256, 8), (4096, 80), (100, 16), (64, 16)]:
        scale = (torch.arange(rows * cols, dtype=torch.float32).reshape(rows, cols) % 200).to(torch.float8_e4m3fn)
        out[f"blocked/{rows}x{cols}/scale"] = scale.view(torch.uint8).numpy().copy()
        out[f"blocked/{rows}x{cols}/expected"] = nvfp4.ref_to_blocked(scale).view(torch.uint8).numpy().copy()

    # RNE tie table (tests/test_nvfp4.py:52-59) and the SR ladder on a grid of magnitudes.
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    out["encode/ties"] = nvfp4.encode_e2m1(ties, sign=torch.zeros_like(ties, dtype=torch.bool)).numpy()
    a = torch.linspace(0, 6, 4097)
    u = torch.rand(4097, generator=torch.Generator().manual_seed(11))
    out["encode/grid"] = a.numpy()
    out["encode/grid_u"] = u.numpy()
    out["encode/grid_rn"] = nvfp4.encode_e2m1(a, sign=torch.zeros_like(a, dtype=torch.bool)).numpy()
    out["encode/grid_sr"] = nvfp4.encode_e2m1(a, sign=torch.zeros_like(a, dtype=torch.bool), u=u).numpy()

    # dequantize (quantize.py:308-320) on the rand1 case.
    torch.manual_seed(101)
    x = torch.randn(256, 128).bfloat16()
    gs = nvfp4.global_scale_of(x)
    p, s = nvfp4.ref_quantize_rowblock(x, gs)
    out["dequant/x"] = _bits(x)
    out["dequant/out"] = nvfp4.dequantize(p, s, gs).numpy()

    # M=256, K=1024, N=1024 forward, seed 0.  Inputs are regenerated by the
    # test with the same torch calls and checked against these digests first.
    torch.manual_seed(0)
    x = torch.randn(256, 1024).bfloat16()
    w = (torch.randn(1024, 1024) * 0.02).bfloat16()
    out["config1/x_sha256"] = np.array(hashlib.sha256(_bits(x).tobytes()).hexdigest())
    out["config1/w_sha256"] = np.array(hashlib.sha256(_bits(w).tobytes()).hexdigest())
    gx, gw = nvfp4.global_scale_of(x), nvfp4.global_scale_of(w)
    xp, xs = nvfp4.ref_quantize_rowblock(x, gx)
    wp, ws = nvfp4.ref_quantize_rowblock(w, gw)
    y = (nvfp4.dequantize(xp, xs, gx) @ nvfp4.dequantize(wp, ws, gw).t()).to(torch.bfloat16)
    out["config1/gx"] = gx.numpy().reshape(())
    out["config1/gw"] = gw.numpy().reshape(())
    out["config1/x_packed_sha256"] = np.array(hashlib.sha256(xp.view(torch.uint8).numpy().tobytes()).hexdigest())
    out["config1/w_packed_sha256"] = np.array(hashlib.sha256(wp.view(torch.uint8).numpy().tobytes()).hexdigest())
    out["config1/y_bf16"] = _bits(y)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "nvfp4_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <path to the radiance checkout>")
    main(sys.argv[1])
