"""``FP4Linear``: radiance's NVFP4 linear layer on the B200-native library.

Drop-in for ``src/radiance/nvfp4/linear.py`` (jamespa16/radiance): same classes, buffers, recipe
and fallback rules.  What changes is underneath:

* The activation and the upstream gradient are each quantized **both ways in one pass**
  (``quantize_both``) instead of two full reads (linear.py:80+99, :129+133).
* The global-scale fold, the bias add and the output cast live in the GEMM epilogue.
* ``refresh_fp4_cache`` quantizes the weight straight into the cache buffers (no ``copy_``).

There is no CPU path: a CUDA input on an sm_100 GPU runs NVFP4; a non-CUDA input raises.  The
reference's bf16 fallback is kept only where the reference pins it -- token counts or widths the
kernels cannot tile, and an unprimed cache -- with its one-time warning.
"""

from __future__ import annotations

from typing import NamedTuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .quantize import (
    BLOCK,
    NVFP4Tensor,
    _supported_cached,
    col_scale_bytes,
    global_scale_and_column_sums,
    global_scale_of,
    hadamard_matrix,
    mm,
    quantize,
    quantize_both,
    quantize_into_,
    quantize_supported_shape,
    require_nvfp4,
    row_scale_bytes,
)


class FP4Recipe(NamedTuple):
    """Which parts of the NVFP4 training recipe are live (linear.py:33-39)."""

    grad_gemms: bool = True
    stochastic_rounding: bool = True
    hadamard: bool = True
    save_activations: bool = True


class _FP4LinearFn(torch.autograd.Function):
    """``y = x W^T + b`` with all three GEMMs in NVFP4 (linear.py:42-155).

    Quantization happens inside forward/backward, out of autograd's sight; the gradient computed
    against the quantized operands is returned for the full-precision input (straight-through).
    """

    @staticmethod
    def forward(ctx, x, weight, bias, w_fwd_packed, w_fwd_scale, w_fwd_gs, w_dgrad_packed, w_dgrad_scale,
                w_dgrad_gs, hadamard, seed, recipe, reduce_grad_scale=None, output_gemm=None):
        gx = global_scale_of(x)
        rot = hadamard if recipe.hadamard and hadamard.numel() else None
        save_quantized = recipe.save_activations and recipe.grad_gemms and quantize_supported_shape(*x.shape)
        if save_quantized:
            # One read of x emits the forward operand and the packed wgrad operand (1.125 B/elt saved).
            xq, xqt = quantize_both(x, global_scale=gx, hadamard=rot)
        else:
            xq = quantize(x, -1, global_scale=gx)
        wq = NVFP4Tensor(w_fwd_packed, w_fwd_scale, w_fwd_gs)
        if output_gemm is None:
            y = mm(xq, wq, out_dtype=x.dtype, bias=bias)
        else:  # e.g. an N-split slice whose GEMM also writes the peers' copies of the output
            y = output_gemm(xq, wq, bias, x.dtype)
        if save_quantized:
            saved = (xqt.packed, xqt.scale, weight, w_dgrad_packed, w_dgrad_scale, w_dgrad_gs, hadamard, seed, gx)
        else:
            saved = (x, x, weight, w_dgrad_packed, w_dgrad_scale, w_dgrad_gs, hadamard, seed, gx)
        ctx.save_for_backward(*saved)
        ctx.recipe = recipe
        ctx.reduce_grad_scale = reduce_grad_scale
        ctx.has_bias = bias is not None
        ctx.save_quantized = save_quantized
        ctx.x_dtype = x.dtype
        ctx.x_shape = x.shape
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x_or_packed, x_or_scale, weight, wdp, wds, wdg, hadamard, seed, gx = ctx.saved_tensors
        recipe: FP4Recipe = ctx.recipe
        if grad_y.stride(-1) != 1:  # row-strided gradients (an N-split slice) are read in place
            grad_y = grad_y.contiguous()
        x_dtype = ctx.x_dtype
        fp4_backward = recipe.grad_gemms and quantize_supported_shape(*grad_y.shape)
        if fp4_backward:
            rot = hadamard if recipe.hadamard and hadamard.numel() else None
            if ctx.has_bias:  # the bias gradient's column sums come from the same read of dY
                gg, colsum = global_scale_and_column_sums(grad_y)
            else:
                gg = global_scale_of(grad_y)
            if ctx.reduce_grad_scale is not None:  # e.g. the full gradient's scale for an N-split slice
                ctx.reduce_grad_scale(gg)
            # dgrad operand (rowblock) and wgrad operand (colblock, rotated) from one read of dY,
            # both stochastically rounded with the same seed (linear.py:129, :133-136).
            gq, gqt = quantize_both(grad_y, global_scale=gg, hadamard=rot,
                                    stochastic=recipe.stochastic_rounding, seed=seed)
            grad_x = mm(gq, NVFP4Tensor(wdp, wds, wdg), out_dtype=x_dtype)
            if ctx.save_quantized:
                xqt = NVFP4Tensor(x_or_packed, x_or_scale, gx)
            else:
                xqt = quantize(x_or_packed, 0, global_scale=gx, hadamard=rot)
            grad_w = mm(gqt, xqt, out_dtype=torch.float32)
        else:
            grad_x = grad_y @ weight.to(grad_y.dtype)
            grad_w = grad_y.t() @ x_or_packed
        grad_b = None
        if ctx.has_bias:
            # The reference's grad_y.sum(0) is a bf16 tensor (fp32 accumulation, one rounding).
            grad_b = colsum.to(grad_y.dtype) if fp4_backward else grad_y.sum(0)
        return (
            grad_x.to(x_dtype),
            grad_w.to(weight.dtype),
            None if grad_b is None else grad_b.to(weight.dtype),
            None, None, None, None, None, None, None, None, None, None, None,
        )


class FP4Linear(nn.Linear):
    """``nn.Linear`` whose three GEMMs run in NVFP4, with a per-optimizer-step weight cache
    (linear.py:158-235).  Buffers are ``persistent=False`` and written in place."""

    def __init__(self, in_features, out_features, bias=True, recipe: FP4Recipe | None = None, device=None,
                 dtype=None):
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        self.recipe = recipe or FP4Recipe()
        self._cache_valid = False
        n, k = out_features, in_features
        dev = self.weight.device
        self.register_buffer("_w_fwd_packed", torch.empty(n, k // 2, dtype=torch.uint8, device=dev), persistent=False)
        self.register_buffer("_w_fwd_scale", torch.empty(row_scale_bytes(n, k), dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_fwd_gs", torch.ones((), dtype=torch.float32, device=dev), persistent=False)
        self.register_buffer("_w_dgrad_packed", torch.empty(k, n // 2, dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_dgrad_scale", torch.empty(col_scale_bytes(n, k), dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_dgrad_gs", torch.ones((), dtype=torch.float32, device=dev), persistent=False)
        self.register_buffer("_hadamard", hadamard_matrix(BLOCK, device=dev), persistent=False)
        self.register_buffer("_seed", torch.zeros((), dtype=torch.int64, device=dev), persistent=False)
        # Optional in-place reduction of the upstream gradient's global scale (set by N-split layers,
        # whose slices must share the full gradient's scale), and an optional replacement for the
        # forward GEMM, called as output_gemm(xq, wq, bias, out_dtype) (set by the fused N-split).
        self.reduce_grad_scale = None
        self.output_gemm = None
        self.register_load_state_dict_post_hook(lambda module, *_: module.invalidate_fp4_cache())

    def invalidate_fp4_cache(self) -> None:
        self._cache_valid = False

    @torch.no_grad()
    def refresh_fp4_cache(self, reduce_global_scale=None) -> None:
        """Re-quantize the weight into both orientations, in place (linear.py:193-210).

        One read of W writes the forward operand (rowblock) and the dgrad operand (colblock)
        directly into the cache buffers, so their data pointers never move.
        ``reduce_global_scale``, when given, is applied in place to the 0-d global-scale tensor
        before quantizing -- an N-split layer passes an all-reduce(MAX) over its ranks so every
        slice uses the full weight's scale.
        """
        w = self.weight.detach()
        if not w.is_cuda:
            require_nvfp4("FP4Linear.refresh_fp4_cache")
            raise RuntimeError("FP4Linear.refresh_fp4_cache: the weight must be on the CUDA device")
        global_scale_of(w, out=self._w_fwd_gs)
        if reduce_global_scale is not None:
            reduce_global_scale(self._w_fwd_gs)
        self._w_dgrad_gs.copy_(self._w_fwd_gs)
        quantize_into_(
            w, global_scale=self._w_fwd_gs,
            row=(self._w_fwd_packed, self._w_fwd_scale), col=(self._w_dgrad_packed, self._w_dgrad_scale),
        )
        self._cache_valid = True

    def _eligible(self, x: torch.Tensor) -> bool:
        return self._cache_valid and quantize_supported_shape(x.numel() // self.in_features, self.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or not _supported_cached(x.device):
            require_nvfp4("FP4Linear")
            raise RuntimeError("FP4Linear: input must be a CUDA tensor on the sm_100 device (no CPU path)")
        if not self._eligible(x):
            _warn_fallback_once(self, x)
            return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        flat = x.reshape(-1, self.in_features).contiguous()
        y = _FP4LinearFn.apply(
            flat, self.weight, self.bias,
            self._w_fwd_packed.view(torch.float4_e2m1fn_x2), self._w_fwd_scale.view(torch.float8_e4m3fn),
            self._w_fwd_gs,
            self._w_dgrad_packed.view(torch.float4_e2m1fn_x2), self._w_dgrad_scale.view(torch.float8_e4m3fn),
            self._w_dgrad_gs,
            self._hadamard, self._seed, self.recipe, self.reduce_grad_scale, self.output_gemm,
        )
        return y.view(*x.shape[:-1], self.out_features)


_warned_fp4_fallback = False


def _warn_fallback_once(module: FP4Linear, x: torch.Tensor) -> None:
    """linear.py:238-257 -- a silent fallback would make the measurement uninterpretable."""
    global _warned_fp4_fallback
    if _warned_fp4_fallback:
        return
    _warned_fp4_fallback = True
    tokens = x.numel() // module.in_features
    print(
        f"[radiance] nvfp4: falling back to bf16 for at least one linear "
        f"(tokens={tokens}, in_features={module.in_features}, cuda={x.is_cuda}, "
        f"cache_valid={module._cache_valid}). FP4 needs tokens % 128 == 0 and in_features % 64 == 0."
    )


def refresh_fp4_weights(model: nn.Module) -> None:
    """Re-quantize every ``FP4Linear``'s weight cache; call once per optimizer step (linear.py:260-275)."""
    for module in model.modules():
        if isinstance(module, FP4Linear):
            module.refresh_fp4_cache()
            module._seed.add_(1)
