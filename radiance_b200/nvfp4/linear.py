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
    quantize_auto_scale_into_,
    quantize_both,
    quantize_into_,
    quantize_supported_shape,
    require_nvfp4,
    row_scale_bytes,
    SWIGLU_GROUP,
    interleave_gate_up,
    merge_gate_up,
    split_gate_up,
    swiglu_backward,
    swiglu_mm,
    update_and_global_scale_,
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
                w_dgrad_gs, hadamard, seed, recipe, reduce_grad_scale=None, output_gemm=None, x_global_scale=None,
                wgrad_hook=None):
        # The input's global scale comes from its producer when that computed it (a SwiGLU epilogue);
        # otherwise the quantizer computes it in the same launch (global_scale_of, linear.py:79).
        rot = hadamard if recipe.hadamard and hadamard.numel() else None
        save_quantized = recipe.save_activations and recipe.grad_gemms and quantize_supported_shape(*x.shape)
        if save_quantized:
            # One read of x emits the forward operand and the packed wgrad operand (1.125 B/elt saved).
            xq, xqt = quantize_both(x, global_scale=x_global_scale, hadamard=rot)
        else:
            xq = quantize(x, -1, global_scale=x_global_scale)
        gx = xq.global_scale
        wq = NVFP4Tensor(w_fwd_packed, w_fwd_scale, w_fwd_gs)
        if output_gemm is None:
            y = mm(xq, wq, out_dtype=x.dtype, bias=bias)
        else:  # e.g. an N-split slice whose GEMM also writes the peers' copies of the output
            y = output_gemm(xq, wq, bias, x.dtype)
        # Saved for backward: the packed wgrad operand (or x itself when it is not saved quantized),
        # the weight's dgrad operand, the rotation, the seed and x's global scale.
        if save_quantized:
            saved = (xqt.packed, xqt.scale, weight, w_dgrad_packed, w_dgrad_scale, w_dgrad_gs, hadamard, seed, gx)
        else:
            saved = (x, x, weight, w_dgrad_packed, w_dgrad_scale, w_dgrad_gs, hadamard, seed, gx)
        ctx.save_for_backward(*saved)
        ctx.recipe = recipe
        ctx.reduce_grad_scale = reduce_grad_scale
        ctx.wgrad_hook = wgrad_hook
        ctx.has_bias = bias is not None
        ctx.save_quantized = save_quantized
        ctx.x_dtype = x.dtype
        ctx.x_shape = x.shape
        return y

    @staticmethod
    def backward(ctx, grad_y):
        xt_or_x, xt_scale, weight, wt_packed, wt_scale, wt_gs, hadamard, seed, gx = ctx.saved_tensors
        recipe: FP4Recipe = ctx.recipe
        if grad_y.stride(-1) != 1:  # row-strided gradients (an N-split slice) are read in place
            grad_y = grad_y.contiguous()
        x_dtype = ctx.x_dtype
        fp4_backward = recipe.grad_gemms and quantize_supported_shape(*grad_y.shape)
        if fp4_backward:
            rot = hadamard if recipe.hadamard and hadamard.numel() else None
            # dY's global scale: from its producer when that computed it (the SwiGLU backward), else
            # computed by the quantizer in the same launch.
            gg = getattr(ctx, "grad_global_scale", None)
            if ctx.has_bias:  # the bias gradient's column sums come from the same read of dY
                gg, colsum = global_scale_and_column_sums(grad_y)
            elif ctx.reduce_grad_scale is not None and gg is None:
                gg = global_scale_of(grad_y)
            if ctx.reduce_grad_scale is not None:  # e.g. the full gradient's scale for an N-split slice
                ctx.reduce_grad_scale(gg)
            # dgrad operand (rowblock) and wgrad operand (colblock, rotated) from one read of dY,
            # both stochastically rounded with the same seed (linear.py:129, :133-136).
            gq, gqt = quantize_both(grad_y, global_scale=gg, hadamard=rot,
                                    stochastic=recipe.stochastic_rounding, seed=seed)
            if ctx.save_quantized:
                xqt = NVFP4Tensor(xt_or_x, xt_scale, gx)
            else:
                xqt = quantize(xt_or_x, 0, global_scale=gx, hadamard=rot)
            # wgrad first: a hook (a data-parallel gradient reduction) can start on it while dgrad runs.
            grad_w = mm(gqt, xqt, out_dtype=torch.float32)
            if ctx.wgrad_hook is not None:
                ctx.wgrad_hook(grad_w)
            grad_x = mm(gq, NVFP4Tensor(wt_packed, wt_scale, wt_gs), out_dtype=x_dtype)
        else:
            grad_x = grad_y @ weight.to(grad_y.dtype)
            grad_w = grad_y.t() @ xt_or_x
        grad_b = None
        if ctx.has_bias:
            # The reference's grad_y.sum(0) is a bf16 tensor (fp32 accumulation, one rounding).
            grad_b = colsum.to(grad_y.dtype) if fp4_backward else grad_y.sum(0)
        return (
            grad_x.to(x_dtype),
            grad_w.to(weight.dtype),
            None if grad_b is None else grad_b.to(weight.dtype),
            None, None, None, None, None, None, None, None, None, None, None, None, None,
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
        # Optional callable given the fp32 weight gradient as soon as the wgrad GEMM has produced it,
        # before dgrad runs (a data-parallel job starts the gradient's reduction there).
        self.wgrad_hook = None
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
        row, col = (self._w_fwd_packed, self._w_fwd_scale), (self._w_dgrad_packed, self._w_dgrad_scale)
        if reduce_global_scale is None:  # global scale and both layouts in one launch
            quantize_auto_scale_into_(w, out_scale=self._w_fwd_gs, row=row, col=col)
        else:
            global_scale_of(w, out=self._w_fwd_gs)
            reduce_global_scale(self._w_fwd_gs)
            quantize_into_(w, global_scale=self._w_fwd_gs, row=row, col=col)
        self._w_dgrad_gs.copy_(self._w_fwd_gs)
        self._cache_valid = True

    @torch.no_grad()
    def apply_update_and_refresh_(self, update: torch.Tensor, alpha: float, reduce_global_scale=None) -> None:
        """The optimizer's last in-place step on this weight, ``weight.add_(update, alpha=alpha)``
        (radiance's Muon step, optim.py:518), fused with the cache refresh: one kernel applies the
        update and computes the new weight's global scale, then one pass quantizes both layouts.
        Same cache contents as ``refresh_fp4_cache()`` after the update, without its amax read.
        ``reduce_global_scale`` is applied to the new global scale before quantizing, as in
        ``refresh_fp4_cache`` (an N-split slice passes the all-reduce(MAX) to the full weight's)."""
        w = self.weight.data
        update_and_global_scale_(w, update, alpha, out=self._w_fwd_gs)
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

    def _check_device(self, x: torch.Tensor) -> None:
        if not x.is_cuda or not _supported_cached(x.device):
            require_nvfp4(type(self).__name__)
            raise RuntimeError(f"{type(self).__name__}: input must be a CUDA tensor on the sm_100 device (no CPU path)")

    def _fn_args(self, flat: torch.Tensor) -> tuple:
        return (
            flat, self.weight, self.bias,
            self._w_fwd_packed.view(torch.float4_e2m1fn_x2), self._w_fwd_scale.view(torch.float8_e4m3fn),
            self._w_fwd_gs,
            self._w_dgrad_packed.view(torch.float4_e2m1fn_x2), self._w_dgrad_scale.view(torch.float8_e4m3fn),
            self._w_dgrad_gs,
            self._hadamard, self._seed, self.recipe, self.reduce_grad_scale,
        )

    def forward(self, x: torch.Tensor, global_scale: torch.Tensor | None = None) -> torch.Tensor:
        """``global_scale``: the input's 0-d fp32 global scale when its producer has computed it
        (``FP4SwiGLU``); by default the layer computes it (linear.py:79)."""
        self._check_device(x)
        if not self._eligible(x):
            _warn_fallback_once(self, x)
            return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        flat = x.reshape(-1, self.in_features).contiguous()
        y = _FP4LinearFn.apply(*self._fn_args(flat), self.output_gemm, global_scale, self.wgrad_hook)
        return y.view(*x.shape[:-1], self.out_features)


class _FP4SwiGLUFn(torch.autograd.Function):
    """``h = F.silu(x Wg^T + bg) * (x Wu^T + bu)`` with the gate/up GEMM in NVFP4 and the activation
    and h's global scale computed in the GEMM's epilogue.  Same inputs as ``_FP4LinearFn``; the
    weight is the interleaved gate/up matrix.  Returns ``(h, global_scale(h))``.

    Forward and the gate/up weight/input gradients are ``_FP4LinearFn``'s, with the output GEMM
    replaced by ``swiglu_mm``; the pre-activations are kept for the SwiGLU backward, which runs as one
    kernel (``swiglu_backward``) that also hands the gate/up backward its gradient's global scale.
    """

    @staticmethod
    def forward(ctx, x, weight, bias, w_fwd_packed, w_fwd_scale, w_fwd_gs, w_dgrad_packed, w_dgrad_scale,
                w_dgrad_gs, hadamard, seed, recipe, reduce_grad_scale=None, output_gemm=None, x_global_scale=None,
                wgrad_hook=None):
        produced = {}

        def gemm(xq, wq, b, out_dtype):
            gu, h, gs = swiglu_mm(xq, wq, bias=b)
            produced["h"], produced["gs"] = h, gs
            return gu

        gu = _FP4LinearFn.forward(ctx, x, weight, bias, w_fwd_packed, w_fwd_scale, w_fwd_gs, w_dgrad_packed,
                                  w_dgrad_scale, w_dgrad_gs, hadamard, seed, recipe, reduce_grad_scale, gemm,
                                  x_global_scale, wgrad_hook)
        ctx.gu = gu  # an intermediate, kept on ctx for the SwiGLU backward
        ctx.mark_non_differentiable(produced["gs"])
        return produced["h"], produced["gs"]

    @staticmethod
    def backward(ctx, grad_h, _grad_gs):
        # One kernel: the SwiGLU derivative (eager autograd's roundings) and its global scale.
        grad_gu, ctx.grad_global_scale = swiglu_backward(grad_h, ctx.gu)
        del ctx.gu
        return _FP4LinearFn.backward(ctx, grad_gu)


class FP4SwiGLU(FP4Linear):
    """The ``gate_proj`` / ``up_proj`` pair of radiance's ``FeedForward`` (src/radiance/model/ffn.py:21-22,
    :32) as one NVFP4 linear of ``2 * hidden_features`` rows, interleaved in blocks of 32 hidden
    units (``interleave_gate_up``).  ``forward(x)`` returns ``(h, gs)``: ``h = F.silu(gate_proj(x)) *
    up_proj(x)`` and ``gs`` its global scale, both from the GEMM's epilogue, so the next
    ``FP4Linear`` (``down_proj(h, global_scale=gs)``) skips its amax pass and nothing re-reads the
    pre-activations in the forward.  ``gs`` is None on the bf16 fallback path."""

    def __init__(self, in_features, hidden_features, bias=True, recipe: FP4Recipe | None = None, device=None,
                 dtype=None):
        if hidden_features % SWIGLU_GROUP:
            raise ValueError(f"FP4SwiGLU: hidden_features must be a multiple of {SWIGLU_GROUP}")
        super().__init__(in_features, 2 * hidden_features, bias=bias, recipe=recipe, device=device, dtype=dtype)
        self.hidden_features = hidden_features

    @classmethod
    @torch.no_grad()
    def from_gate_up(cls, gate_proj: nn.Linear, up_proj: nn.Linear, recipe: FP4Recipe | None = None) -> "FP4SwiGLU":
        """Build from the two ``nn.Linear`` layers of a radiance ``FeedForward`` (weights copied)."""
        w = gate_proj.weight
        mod = cls(gate_proj.in_features, gate_proj.out_features, bias=gate_proj.bias is not None, recipe=recipe,
                  device=w.device, dtype=w.dtype)
        mod.weight.copy_(interleave_gate_up(gate_proj.weight, up_proj.weight))
        if gate_proj.bias is not None:
            mod.bias.copy_(interleave_gate_up(gate_proj.bias, up_proj.bias))
        mod.invalidate_fp4_cache()
        return mod

    def gate_up_weights(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The gate and up projections' weights (copies, in their own row order)."""
        g, u = split_gate_up(self.weight.detach().t())
        return g.t().contiguous(), u.t().contiguous()

    def _eligible(self, x: torch.Tensor) -> bool:
        return super()._eligible(x) and x.dtype == torch.bfloat16

    def forward(self, x: torch.Tensor, global_scale: torch.Tensor | None = None):
        self._check_device(x)
        if not self._eligible(x):
            _warn_fallback_once(self, x)
            gu = F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
            g, u = split_gate_up(gu)
            return F.silu(g) * u, None
        flat = x.reshape(-1, self.in_features).contiguous()
        h, gs = _FP4SwiGLUFn.apply(*self._fn_args(flat), None, global_scale, self.wgrad_hook)
        return h.view(*x.shape[:-1], self.hidden_features), gs


class FP4FeedForward(nn.Module):
    """radiance's one-hidden-layer ``FeedForward`` (ffn.py:10-39, ``ffn_depth == 1``, no LoRA):
    ``down_proj(F.silu(gate_proj(x)) * up_proj(x))``, with the gate/up pair as ``FP4SwiGLU`` and
    ``down_proj`` an ``FP4Linear`` fed the global scale the SwiGLU epilogue computed."""

    def __init__(self, d_model, ffn_dim, bias=True, dropout: float = 0.0, recipe: FP4Recipe | None = None,
                 device=None, dtype=None):
        super().__init__()
        self.gate_up = FP4SwiGLU(d_model, ffn_dim, bias=bias, recipe=recipe, device=device, dtype=dtype)
        self.down_proj = FP4Linear(ffn_dim, d_model, bias=bias, recipe=recipe, device=device, dtype=dtype)
        self.dropout = nn.Dropout(dropout)

    @classmethod
    @torch.no_grad()
    def from_feedforward(cls, ff: nn.Module, recipe: FP4Recipe | None = None) -> "FP4FeedForward":
        """Build from a module with ``gate_proj``, ``up_proj`` and ``down_proj`` ``nn.Linear`` layers."""
        w = ff.down_proj.weight
        mod = cls(ff.gate_proj.in_features, ff.gate_proj.out_features, bias=ff.down_proj.bias is not None,
                  recipe=recipe, device=w.device, dtype=w.dtype)
        mod.gate_up = FP4SwiGLU.from_gate_up(ff.gate_proj, ff.up_proj, recipe=recipe)
        mod.down_proj.weight.copy_(ff.down_proj.weight)
        if ff.down_proj.bias is not None:
            mod.down_proj.bias.copy_(ff.down_proj.bias)
        mod.down_proj.invalidate_fp4_cache()
        return mod

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h, gs = self.gate_up(x)
        return self.dropout(self.down_proj(h, global_scale=gs))


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
