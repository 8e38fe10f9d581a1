"""radiance's NVFP4 format definition, in plain torch: the ``quantize_reference`` family of
``radiance.nvfp4`` (src/radiance/nvfp4/quantize.py:86-320, :412-433 in jamespa16/radiance).

radiance exports these alongside its kernels: they *define* the format (the kernels are asserted
bit-identical to them) and its tests call them to build expected values.  They are re-exported here
so that code written against ``radiance.nvfp4`` -- those tests included -- finds the same names with
the same arguments and results.  They run on any device, one element-wise torch op at a time, and
nothing in the NVFP4 path calls them: ``quantize``, ``mm`` and ``FP4Linear`` run only on the CUDA
library and raise on a CPU tensor.

The Hadamard rotation of ``ref_quantize_colblock`` is written as an explicit left-to-right fp32 sum
over the 16 rows of a block (each product rounded, then added), the order the CUDA kernel and the
golden vectors use, so the result does not depend on a BLAS library's summation order.
"""

from __future__ import annotations

import torch

from .quantize import (BLOCK, E4M3_MAX, FP4_MAX, FP4_VALUES, TINY, NVFP4Tensor, blocked_offset, pack_nibbles,
                       scale_denominator, unpack_nibbles)

# The round-to-nearest-even ladder on the e2m1 grid (0, .5, 1, 1.5, 2, 3, 4, 6): a magnitude moves
# up past the midpoints in _STRICT when strictly above them and past those in _INCLUSIVE when at or
# above them, which sends every exact midpoint to the even code (quantize.py:93-118).
_STRICT = (0.25, 1.25, 2.5, 5.0)
_INCLUSIVE = (0.75, 1.75, 3.5)


def _reference_global_scale(x: torch.Tensor) -> torch.Tensor:
    """``global_scale_of`` (quantize.py:205-213) as a torch reduction: max|x| / 2688, at least 1e-12."""
    return (x.abs().amax().float() / (FP4_MAX * E4M3_MAX)).clamp(min=TINY)


def encode_e2m1(a: torch.Tensor, *, sign: torch.Tensor, u: torch.Tensor | None = None) -> torch.Tensor:
    """Magnitudes in [0, 6] -> uint8 e2m1 codes with the sign in bit 3 (quantize.py:93-139).

    Without ``u``: round to nearest, ties to the even code.  With ``u`` (one uniform [0, 1) draw
    per element): stochastic rounding, up to the next level with probability
    ``(a - lo) / (hi - lo)``."""
    a = a.float()
    dev = a.device
    if u is None:
        code = (torch.bucketize(a, torch.tensor(_STRICT, device=dev), right=False)
                + torch.bucketize(a, torch.tensor(_INCLUSIVE, device=dev), right=True))
    else:
        levels = torch.tensor(FP4_VALUES + (FP4_MAX,), device=dev, dtype=torch.float32)
        lo = torch.bucketize(a, levels[1:-1], right=True)  # the level at or below a
        lo_v, hi_v = levels[lo], levels[lo + 1]
        step = (hi_v - lo_v).clamp(min=TINY)
        frac = torch.where(hi_v > lo_v, (a - lo_v) / step, torch.zeros_like(a))
        code = (lo + (u.float() < frac).long()).clamp(max=7)
    return code.to(torch.uint8) | (sign.to(torch.uint8) << 3)


def _block_scale(amax: torch.Tensor, global_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Block amax -> (e4m3 block scale, fp32 divisor) (quantize.py:160-187).

    The scale is ``clamp(amax / (6 gs), 1e-12, 448)`` rounded *up* to the next e4m3 value (never to
    the NaN byte 0x7F), so no element of the block quantizes above 6; the divisor is that e4m3 value,
    or 1 for an all-zero block."""
    s = (amax.float() / scale_denominator(global_scale)).clamp(min=TINY, max=E4M3_MAX)
    byte = s.to(torch.float8_e4m3fn).view(torch.uint8)
    below = (byte.view(torch.float8_e4m3fn).float() < s) & (byte < 0x7E)
    scale = (byte + below.to(torch.uint8)).view(torch.float8_e4m3fn)
    divisor = torch.where(amax > 0, scale.float(), torch.ones_like(s))
    return scale, divisor


def _quantize_blocks(xb: torch.Tensor, global_scale: torch.Tensor, u: torch.Tensor | None, dim: int):
    """Blocks of 16 along ``dim`` of ``xb`` (fp32) -> codes and per-block e4m3 scales."""
    scale, divisor = _block_scale(xb.abs().amax(dim, keepdim=True), global_scale)
    q = (xb / (divisor * global_scale)).clamp(-FP4_MAX, FP4_MAX)
    return encode_e2m1(q.abs(), sign=q < 0, u=u), scale.squeeze(dim)


def ref_quantize_rowblock(x: torch.Tensor, global_scale: torch.Tensor, *, u: torch.Tensor | None = None):
    """(M, K) -> packed (M, K/2) ``float4_e2m1fn_x2``, unswizzled e4m3 scales (M, K/16); blocks of 16
    along the last dim (quantize.py:216-232)."""
    m, k = x.shape
    code, scale = _quantize_blocks(x.float().reshape(m, k // BLOCK, BLOCK), global_scale,
                                   None if u is None else u.reshape(m, k // BLOCK, BLOCK), -1)
    return pack_nibbles(code.reshape(m, k)), scale


def _rotate(xb: torch.Tensor, hadamard: torch.Tensor) -> torch.Tensor:
    """``R^T`` applied to every 16-row block of ``xb`` (blocks, 16, K): output row i is
    sum_j R[j, i] * x_j, summed left to right in fp32 (quantize.py:261-262)."""
    r = hadamard.to(device=xb.device, dtype=torch.float32)
    out = []
    for i in range(BLOCK):
        acc = r[0, i] * xb[:, 0]
        for j in range(1, BLOCK):
            acc = acc + r[j, i] * xb[:, j]
        out.append(acc)
    return torch.stack(out, dim=1)


def ref_quantize_colblock(x: torch.Tensor, global_scale: torch.Tensor, *, hadamard: torch.Tensor | None = None,
                          u: torch.Tensor | None = None):
    """(M, K) -> packed (K, M/2), unswizzled e4m3 scales (K, M/16): blocks of 16 along the first dim,
    optionally rotated by ``R^T``, output transposed (quantize.py:235-268)."""
    m, k = x.shape
    xb = x.float().reshape(m // BLOCK, BLOCK, k)
    if hadamard is not None:
        xb = _rotate(xb, hadamard)
    code, scale = _quantize_blocks(xb, global_scale, None if u is None else u.reshape(m // BLOCK, BLOCK, k), 1)
    return pack_nibbles(code.reshape(m, k).t().contiguous()), scale.t().contiguous()


def ref_to_blocked(scale: torch.Tensor) -> torch.Tensor:
    """(rows, cols) block scales -> the flat SWIZZLE_32_4_4 layout, zero-padded to whole 128 x 4
    tiles (quantize.py:271-290)."""
    rows, cols = scale.shape
    n_row_tiles, n_col_tiles = (rows + 127) // 128, (cols + 3) // 4
    raw = scale.view(torch.uint8) if scale.dtype == torch.float8_e4m3fn else scale
    flat = torch.zeros(n_row_tiles * n_col_tiles * 512, dtype=raw.dtype, device=raw.device)
    r = torch.arange(rows, device=raw.device).view(-1, 1)
    c = torch.arange(cols, device=raw.device).view(1, -1)
    flat[blocked_offset(r, c, n_col_tiles).reshape(-1)] = raw.reshape(-1)
    return flat.view(scale.dtype) if scale.dtype == torch.float8_e4m3fn else flat


def dequantize(packed: torch.Tensor, scale_e4m3: torch.Tensor, global_scale: torch.Tensor) -> torch.Tensor:
    """Packed codes + unswizzled block scales -> fp32 (quantize.py:308-320)."""
    code = unpack_nibbles(packed).long()
    grid = torch.tensor(FP4_VALUES, device=packed.device, dtype=torch.float32)
    value = grid[code & 7] * (1.0 - 2.0 * (code >> 3).float())
    rows, cols = value.shape
    per_block = (scale_e4m3.float() * global_scale).unsqueeze(-1)
    return (value.view(rows, cols // BLOCK, BLOCK) * per_block).view(rows, cols)


def quantize_reference(x: torch.Tensor, axis: int, *, global_scale: torch.Tensor | None = None,
                       hadamard: torch.Tensor | None = None, u: torch.Tensor | None = None) -> NVFP4Tensor:
    """The format's definition of ``quantize`` (quantize.py:412-433): ``axis=-1`` blocks along the
    last dim, ``axis=0`` along the first (with the optional rotation); scales swizzled."""
    if global_scale is None:
        global_scale = _reference_global_scale(x)
    if axis in (-1, x.dim() - 1):
        packed, scale = ref_quantize_rowblock(x, global_scale, u=u)
    elif axis == 0:
        packed, scale = ref_quantize_colblock(x, global_scale, hadamard=hadamard, u=u)
    else:
        raise ValueError(f"nvfp4.quantize supports axis 0 or -1, got {axis}")
    return NVFP4Tensor(packed=packed, scale=ref_to_blocked(scale), global_scale=global_scale)
