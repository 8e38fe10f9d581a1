"""Grouped (mixture-of-experts) NVFP4 linears on the B200-native library.

radiance runs its experts as stacked bf16 batched matmuls -- ``BatchedExperts.forward``
(src/radiance/model/ffn.py:148-153), ``torch.baddbmm`` over ``(experts, capacity, d)`` with weights
stored ``(experts, in, out)`` -- and rejects FP4 with MoE (transformer.py:204-213).  This module
gives that expert path NVFP4 GEMMs with radiance's per-linear semantics (``_FP4LinearFn``,
linear.py:63-155) applied to every expert on its own tokens:

* forward: each expert's token group is quantized rowblock with its own global scale, each expert
  weight with its own; one grouped GEMM covers every expert (``rb_nvfp4_gemm_grouped``);
* dgrad: the upstream gradient's groups quantized rowblock with stochastic rounding, against the
  per-expert dgrad weight operands;
* wgrad: both operands quantized colblock with the Hadamard rotation (and SR for the gradient),
  one grouped GEMM over each expert's range of token columns.

Layout: the tokens routed to the experts sit in one ``(T, d)`` tensor sorted by expert; expert
``g`` owns rows ``offsets[g]:offsets[g+1]``, and every group is padded to a multiple of 128 rows
with zero rows (``align_offsets``).  ``offsets`` is a device tensor: nothing here synchronises
with the host, so routing counts never leave the GPU.  ``FP4BatchedExperts`` keeps radiance's
``(experts, capacity, d)`` interface on top (capacity a multiple of 128).
"""

from __future__ import annotations

import weakref

import torch
import torch.nn as nn

from .. import _lib
from . import _trace
from .linear import FP4Recipe
from .quantize import (
    BLOCK,
    _default_seed,
    _dtype_code,
    _prep_input,
    _require_cuda,
    _stream_ptr,
    col_scale_bytes,
    global_scale_of,
    hadamard_matrix,
    quantize_into_,
    require_nvfp4,
    row_scale_bytes,
    swiglu,
)

ALIGN = 128

_GROUP_WS: dict[tuple[torch.device, int, int], torch.Tensor] = {}


def align_offsets(counts: torch.Tensor, align: int = ALIGN) -> torch.Tensor:
    """Per-expert token counts ``(E,)`` -> row offsets ``(E + 1,)`` int64 with every group padded up
    to a multiple of ``align`` (a device op, no host sync)."""
    c = counts.to(torch.int64)
    padded = (c + (align - 1)) // align * align
    return torch.cat([torch.zeros(1, dtype=torch.int64, device=c.device), torch.cumsum(padded, 0)])


def _group_workspace(device: torch.device, n: int) -> torch.Tensor:
    key = (device, _stream_ptr(device), n)
    ws = _GROUP_WS.get(key)
    if ws is None:
        ws = torch.zeros(n + 1, dtype=torch.int32, device=device)
        _GROUP_WS[key] = ws
    return ws


def _check_offsets(offsets: torch.Tensor, device: torch.device) -> torch.Tensor:
    if offsets.dim() != 1 or offsets.numel() < 2:
        raise ValueError("nvfp4 grouped: offsets must be a 1-D tensor of num_groups + 1 row offsets")
    if offsets.dtype != torch.int64 or offsets.device != device or not offsets.is_contiguous():
        offsets = offsets.to(device=device, dtype=torch.int64).contiguous()
    return offsets


def global_scale_grouped(x: torch.Tensor, offsets: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-group global scales ``(E,)`` fp32: ``global_scale_of`` (quantize.py:205-213) of every row
    group ``x[offsets[g]:offsets[g+1]]``, one kernel (an empty group gets 1e-12)."""
    _require_cuda(x, "nvfp4.global_scale_grouped")
    lib = _lib.load()
    x2 = _prep_input(x)
    offsets = _check_offsets(offsets, x.device)
    e = offsets.numel() - 1
    if out is None:
        out = torch.empty(e, dtype=torch.float32, device=x.device)
    rows, cols = x2.shape
    tok = _trace.begin("amax", rows * cols * x2.element_size())
    _lib.check(
        lib.rb_nvfp4_global_scale_grouped(
            x2.data_ptr(), _dtype_code(x2), rows, cols, x2.stride(0), offsets.data_ptr(), e, out.data_ptr(),
            _group_workspace(x.device, e).data_ptr(), _stream_ptr(x.device),
        ),
        "nvfp4.global_scale_grouped",
    )
    _trace.end(tok)
    return out


def quantize_grouped_into_(
    x: torch.Tensor,
    offsets: torch.Tensor,
    group_gs: torch.Tensor,
    *,
    row: tuple[torch.Tensor, torch.Tensor] | None = None,
    col: tuple[torch.Tensor, torch.Tensor] | None = None,
    hadamard: torch.Tensor | None = None,
    stochastic: bool = False,
    seed: torch.Tensor | int = 0,
) -> None:
    """``quantize_into_`` with one global scale per row group: each 128-row tile uses the scale of
    the group holding its first row.  Outputs have the single-tensor sizes (rowblock: ``(T, K/2)``
    and ``row_scale_bytes(T, K)``; colblock: ``(K, T/2)`` and ``col_scale_bytes(T, K)``)."""
    _require_cuda(x, "nvfp4.quantize_grouped")
    lib = _lib.load()
    x = _prep_input(x)
    m, k = x.shape
    if m % ALIGN or k % 64:
        raise ValueError(f"nvfp4.quantize_grouped needs rows % 128 == 0 and cols % 64 == 0, got {(m, k)}")
    offsets = _check_offsets(offsets, x.device)
    gs = group_gs.to(device=x.device, dtype=torch.float32).contiguous()
    seed_t = None
    if stochastic:
        seed_t = seed if isinstance(seed, torch.Tensor) else _default_seed(x.device, int(seed))
        seed_t = seed_t.to(device=x.device, dtype=torch.int64)
    had = None
    if hadamard is not None and hadamard.numel():
        had = hadamard.to(device=x.device, dtype=torch.float32).contiguous()
    forms = (row is not None) + (col is not None)
    tok = _trace.begin("quantize", m * k * (x.element_size() + 0.5625 * forms))
    _lib.check(
        lib.rb_nvfp4_quantize_grouped(
            x.data_ptr(), _dtype_code(x), m, k, x.stride(0), offsets.data_ptr(), offsets.numel() - 1, gs.data_ptr(),
            None if had is None else had.data_ptr(), None if seed_t is None else seed_t.data_ptr(),
            None if row is None else row[0].data_ptr(), None if row is None else row[1].data_ptr(),
            None if col is None else col[0].data_ptr(), None if col is None else col[1].data_ptr(),
            _stream_ptr(x.device),
        ),
        "nvfp4.quantize_grouped",
    )
    _trace.end(tok)


def _row_buffers(m: int, k: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    return (torch.empty(m, k // 2, dtype=torch.uint8, device=device),
            torch.empty(row_scale_bytes(m, k), dtype=torch.uint8, device=device))


def _col_buffers(m: int, k: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    return (torch.empty(k, m // 2, dtype=torch.uint8, device=device),
            torch.empty(col_scale_bytes(m, k), dtype=torch.uint8, device=device))


_OUT_CODES = {torch.bfloat16: _lib.RB_OUT_BF16, torch.float32: _lib.RB_OUT_F32}


def grouped_mm(
    a: tuple[torch.Tensor, torch.Tensor],
    b: tuple[torch.Tensor, torch.Tensor],
    groups: torch.Tensor,
    *,
    n: int,
    k_total: int,
    out_rows: int,
    alpha_a: torch.Tensor | None = None,
    alpha_b: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """One grouped block-scaled GEMM (``rb_nvfp4_gemm_grouped``): for each row of the device tensor
    ``groups`` = (a_row0, b_row0, out_row0, m, k0, k),
    ``out[out_row0 + i, :n] = alpha_a[g] alpha_b[g] * sum_{k0 <= c < k0 + k} A[a_row0 + i, c] B[b_row0 + :n, c]``.
    ``a`` and ``b`` are (packed, scale) rowblock-layout operands over one contraction axis of
    ``k_total`` elements.  Rows of ``out`` outside every group are left as they were."""
    a_packed, a_scale = a
    b_packed, b_scale = b
    _require_cuda(a_packed, "nvfp4.grouped_mm")
    lib = _lib.load()
    if a_packed.shape[1] * 2 != k_total or b_packed.shape[1] * 2 != k_total:
        raise ValueError(f"nvfp4.grouped_mm: operands must have k_total / 2 = {k_total // 2} packed columns")
    groups = groups.to(device=a_packed.device, dtype=torch.int64).contiguous()
    if groups.dim() != 2 or groups.shape[1] != 6:
        raise ValueError("nvfp4.grouped_mm: groups must be (num_groups, 6) int64")
    native = out_dtype if out_dtype in _OUT_CODES else torch.float32
    if out is None:
        out = torch.empty(out_rows, n, dtype=native, device=a_packed.device)
    num = groups.shape[0]
    aa = None if alpha_a is None else alpha_a.to(torch.float32).contiguous()
    ab = None if alpha_b is None else alpha_b.to(torch.float32).contiguous()
    tok = _trace.begin("gemm", 0.0)
    _lib.check(
        lib.rb_nvfp4_gemm_grouped(
            a_packed.data_ptr(), a_scale.data_ptr(), a_packed.shape[0], b_packed.data_ptr(), b_scale.data_ptr(),
            b_packed.shape[0], n, k_total, groups.data_ptr(), num, None if aa is None else aa.data_ptr(),
            None if ab is None else ab.data_ptr(), out.data_ptr(), _OUT_CODES[native], out_rows, out.stride(0),
            _stream_ptr(a_packed.device),
        ),
        "nvfp4.grouped_mm",
    )
    _trace.end(tok)
    return out if native == out_dtype else out.to(out_dtype)


MAX_GROUPS = 256  # groups per rb_nvfp4_gemm_grouped launch
_BMM_RECORDS: dict[tuple, torch.Tensor] = {}


def bmm(a, b, batch: int, *, out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """Batched NVFP4 GEMM: ``out[i] = a[i] @ b[i].T`` for ``i < batch``, as one grouped launch per
    256 batch entries.

    radiance keeps attention's ``Q @ K^T`` and ``attn @ V`` in bf16 because ``torch._scaled_mm_v2``
    is two-dimensional only (docs/results.md:287-293); the grouped tcgen05 GEMM has no such limit.
    ``a`` and ``b`` are rowblock ``NVFP4Tensor``s of the stacked ``(batch * M, K)`` and
    ``(batch * N, K)`` operands, each quantized as one tensor (one global scale);
    M and N must be multiples of 128 and K of 64.  Returns ``(batch, M, N)``.
    """
    a_packed, b_packed = a.packed.view(torch.uint8), b.packed.view(torch.uint8)
    _require_cuda(a_packed, "nvfp4.bmm")
    rows_a, rows_b = a_packed.shape[0], b_packed.shape[0]
    if batch < 1 or rows_a % batch or rows_b % batch:
        raise ValueError(f"nvfp4.bmm: {rows_a} and {rows_b} rows do not split into {batch} batch entries")
    m, n, k = rows_a // batch, rows_b // batch, a_packed.shape[1] * 2
    if m % 128 or n % 128 or k % 64 or b_packed.shape[1] * 2 != k:
        raise ValueError(f"nvfp4.bmm needs M % 128 == 0, N % 128 == 0 and a shared K % 64 == 0, got M={m}, "
                         f"N={n}, K={k} and {b_packed.shape[1] * 2}")
    dev = a_packed.device
    native = out_dtype if out_dtype in _OUT_CODES else torch.float32
    if out is None:
        out = torch.empty(batch * m, n, dtype=native, device=dev)
    for start in range(0, batch, MAX_GROUPS):
        cnt = min(MAX_GROUPS, batch - start)
        key = (dev, start, cnt, m, n, k)
        recs = _BMM_RECORDS.get(key)
        if recs is None:
            g = torch.arange(start, start + cnt, dtype=torch.int64)
            recs = torch.stack([g * m, g * n, g * m, torch.full_like(g, m), torch.zeros_like(g),
                                torch.full_like(g, k)], dim=1).to(dev)
            _BMM_RECORDS[key] = recs
        grouped_mm((a_packed, a.scale.view(torch.uint8)), (b_packed, b.scale.view(torch.uint8)), recs, n=n,
                   k_total=k, out_rows=batch * m, alpha_a=a.global_scale.reshape(1).expand(cnt),
                   alpha_b=b.global_scale.reshape(1).expand(cnt), out_dtype=native, out=out)
    out = out.view(batch, m, n)
    return out if native == out_dtype else out.to(out_dtype)


def groups_over_rows(offsets: torch.Tensor, b_rows_per_group: int, k: int) -> torch.Tensor:
    """Group records for a forward or dgrad GEMM: group g multiplies token rows
    ``offsets[g]:offsets[g+1]`` by expert operand rows ``g * b_rows_per_group ...`` over the full
    contraction ``k``, writing the same token rows of the output."""
    start, size = offsets[:-1], offsets[1:] - offsets[:-1]
    e = start.numel()
    idx = torch.arange(e, dtype=torch.int64, device=offsets.device)
    zeros = torch.zeros_like(start)
    return torch.stack([start, idx * b_rows_per_group, start, size, zeros, torch.full_like(start, k)], dim=1)


def groups_over_contraction(offsets: torch.Tensor, out_rows_per_group: int) -> torch.Tensor:
    """Group records for a wgrad GEMM: group g contracts over its token range
    ``offsets[g]:offsets[g+1]`` of two colblock operands, writing output rows
    ``g * out_rows_per_group ...`` (that expert's weight gradient)."""
    start, size = offsets[:-1], offsets[1:] - offsets[:-1]
    e = start.numel()
    idx = torch.arange(e, dtype=torch.int64, device=offsets.device)
    zeros = torch.zeros_like(start)
    return torch.stack([zeros, zeros, idx * out_rows_per_group, torch.full_like(start, out_rows_per_group), start,
                        size], dim=1)


_RECORD_CACHE: dict = {}


def _records(kind: str, offsets: torch.Tensor, a: int, b: int) -> torch.Tensor:
    """Group records for ``offsets``, cached per offsets tensor object (held weakly) and its version:
    one step's routing is reused by every expert layer, forward and backward."""
    key = (id(offsets), kind, a, b)
    hit = _RECORD_CACHE.get(key)
    if hit is not None and hit[0]() is offsets and hit[1] == offsets._version:
        return hit[2]
    if len(_RECORD_CACHE) > 64:
        _RECORD_CACHE.clear()
    rec = groups_over_rows(offsets, a, b) if kind == "rows" else groups_over_contraction(offsets, a)
    _RECORD_CACHE[key] = (weakref.ref(offsets), offsets._version, rec)
    return rec


class _FP4GroupedLinearFn(torch.autograd.Function):
    """``y[rows of expert g] = x[rows of g] @ W_g`` for every expert, all three GEMMs in NVFP4.

    ``weight`` is ``(E, in, out)`` (BatchedExperts' storage, ffn.py:117-141).  Per expert this is
    ``_FP4LinearFn`` (linear.py:63-155) with ``W = W_g^T``; the gradients are straight-through, as
    there."""

    @staticmethod
    def forward(ctx, x, offsets, weight, w_fwd_packed, w_fwd_scale, w_dgrad_packed, w_dgrad_scale, w_gs, hadamard,
                seed, recipe):
        e, k, n = weight.shape
        t = x.shape[0]
        gx = global_scale_grouped(x, offsets)
        rot = hadamard if recipe.hadamard and hadamard.numel() else None
        xrow = _row_buffers(t, k, x.device)
        xcol = _col_buffers(t, k, x.device) if recipe.grad_gemms else None
        quantize_grouped_into_(x, offsets, gx, row=xrow, col=xcol, hadamard=rot)
        y = grouped_mm(xrow, (w_fwd_packed, w_fwd_scale), _records("rows", offsets, n, k), n=n, k_total=k,
                       out_rows=t, alpha_a=gx, alpha_b=w_gs, out_dtype=x.dtype)
        if recipe.grad_gemms:
            ctx.save_for_backward(offsets, xcol[0], xcol[1], gx, w_dgrad_packed, w_dgrad_scale, w_gs, hadamard, seed)
        else:
            ctx.save_for_backward(offsets, x, weight)
        ctx.recipe = recipe
        ctx.shape = (e, k, n, t)
        ctx.x_dtype = x.dtype
        return y

    @staticmethod
    def backward(ctx, grad_y):
        recipe: FP4Recipe = ctx.recipe
        e, k, n, t = ctx.shape
        grad_y = grad_y.contiguous()
        if not recipe.grad_gemms:
            offsets, x, weight = ctx.saved_tensors
            raise RuntimeError("FP4GroupedLinear: grad_gemms=False needs a bf16 expert path; use BatchedExperts")
        offsets, xcol_p, xcol_s, gx, wdp, wds, w_gs, hadamard, seed = ctx.saved_tensors
        rot = hadamard if recipe.hadamard and hadamard.numel() else None
        gg = global_scale_grouped(grad_y, offsets)
        grow = _row_buffers(t, n, grad_y.device)
        gcol = _col_buffers(t, n, grad_y.device)
        quantize_grouped_into_(grad_y, offsets, gg, row=grow, col=gcol, hadamard=rot,
                               stochastic=recipe.stochastic_rounding, seed=seed)
        grad_x = grouped_mm(grow, (wdp, wds), _records("rows", offsets, k, n), n=k, k_total=n, out_rows=t,
                            alpha_a=gg, alpha_b=w_gs, out_dtype=ctx.x_dtype)
        # dW_g in (in, out) storage = X_g^T dY_g: rows of the colblock X operand (in) times rows of
        # the colblock dY operand (out), contracted over the expert's tokens.
        grad_w = grouped_mm((xcol_p, xcol_s), gcol, _records("contraction", offsets, k, 0), n=n, k_total=t,
                            out_rows=e * k, alpha_a=gx, alpha_b=gg, out_dtype=torch.float32)
        return grad_x, None, grad_w.view(e, k, n), None, None, None, None, None, None, None, None


class FP4GroupedLinear(nn.Module):
    """E expert linears ``in -> out`` in NVFP4 over expert-sorted tokens.

    ``weight`` is ``(E, in, out)`` as in BatchedExperts (ffn.py:130-141).  The weight cache holds,
    per expert, the forward operand (``W_g^T``, rowblock over ``in``) and the dgrad operand (``W_g``,
    rowblock over ``out``) with one global scale per expert; ``refresh_fp4_cache`` rebuilds it in
    place (call once per optimizer step, like ``refresh_fp4_weights``)."""

    def __init__(self, n_experts: int, in_features: int, out_features: int, recipe: FP4Recipe | None = None,
                 device=None, dtype=None):
        super().__init__()
        if in_features % ALIGN or out_features % ALIGN:
            raise ValueError("FP4GroupedLinear needs in_features and out_features that are multiples of 128")
        self.n_experts, self.in_features, self.out_features = n_experts, in_features, out_features
        self.recipe = recipe or FP4Recipe()
        self.weight = nn.Parameter(torch.empty(n_experts, in_features, out_features, device=device, dtype=dtype))
        nn.init.normal_(self.weight, std=0.02)
        e, k, n = n_experts, in_features, out_features
        dev = self.weight.device
        self.register_buffer("_w_fwd_packed", torch.empty(e * n, k // 2, dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_fwd_scale", torch.empty(e * col_scale_bytes(k, n), dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_dgrad_packed", torch.empty(e * k, n // 2, dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_dgrad_scale", torch.empty(row_scale_bytes(e * k, n), dtype=torch.uint8, device=dev),
                             persistent=False)
        self.register_buffer("_w_gs", torch.ones(e, dtype=torch.float32, device=dev), persistent=False)
        self.register_buffer("_hadamard", hadamard_matrix(BLOCK, device=dev), persistent=False)
        self.register_buffer("_seed", torch.zeros((), dtype=torch.int64, device=dev), persistent=False)
        self._cache_valid = False
        self.register_load_state_dict_post_hook(lambda module, *_: module.invalidate_fp4_cache())

    def invalidate_fp4_cache(self) -> None:
        self._cache_valid = False

    @torch.no_grad()
    def refresh_fp4_cache(self) -> None:
        w = self.weight.detach()
        if not w.is_cuda:
            require_nvfp4("FP4GroupedLinear.refresh_fp4_cache")
            raise RuntimeError("FP4GroupedLinear.refresh_fp4_cache: the weight must be on the CUDA device")
        e, k, n = w.shape
        stacked = w.reshape(e * k, n)
        offs = torch.arange(e + 1, dtype=torch.int64, device=w.device) * k
        global_scale_grouped(stacked, offs, out=self._w_gs)
        # dgrad operand: W_g (in x out) rowblock, all experts in one pass.
        quantize_grouped_into_(stacked, offs, self._w_gs, row=(self._w_dgrad_packed, self._w_dgrad_scale))
        # forward operand: W_g^T = the colblock form of W_g, one launch per expert.
        sb = col_scale_bytes(k, n)
        for g in range(e):
            quantize_into_(w[g], global_scale=self._w_gs[g],
                           col=(self._w_fwd_packed[g * n:(g + 1) * n], self._w_fwd_scale[g * sb:(g + 1) * sb]))
        self._cache_valid = True

    def forward(self, x: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
        """``x``: ``(T, in)`` tokens sorted by expert, ``T % 128 == 0``; ``offsets``: ``(E + 1,)``
        device row offsets (multiples of 128).  Returns ``(T, out)``; rows past ``offsets[E]``
        (a worst-case allocation's tail) are left undefined, and so are their input gradients."""
        if not x.is_cuda:
            require_nvfp4("FP4GroupedLinear")
            raise RuntimeError("FP4GroupedLinear: input must be a CUDA tensor on the sm_100 device (no CPU path)")
        if not self._cache_valid:
            raise RuntimeError("FP4GroupedLinear: call refresh_fp4_cache() after (re)loading or updating weights")
        if x.dim() != 2 or x.shape[1] != self.in_features or x.shape[0] % ALIGN:
            raise ValueError(f"FP4GroupedLinear expects (T, {self.in_features}) with T % 128 == 0, got {tuple(x.shape)}")
        offsets = _check_offsets(offsets, x.device)
        if offsets.numel() != self.n_experts + 1:
            raise ValueError(f"FP4GroupedLinear: expected {self.n_experts + 1} offsets, got {offsets.numel()}")
        return _FP4GroupedLinearFn.apply(
            x.contiguous(), offsets, self.weight, self._w_fwd_packed, self._w_fwd_scale, self._w_dgrad_packed,
            self._w_dgrad_scale, self._w_gs, self._hadamard, self._seed, self.recipe,
        )


class FP4BatchedExperts(nn.Module):
    """``BatchedExperts`` (ffn.py:108-153, ``ffn_depth`` 1) with NVFP4 expert GEMMs: input and
    output ``(n_experts, capacity, d_model)``, ``silu(x W_gate + b_gate) * (x W_up + b_up)``, then
    ``W_down``.  Gate and up run as one fused ``d -> 2 * ffn`` grouped linear.  ``capacity`` must be
    a multiple of 128; ``forward_sorted`` takes expert-sorted tokens with arbitrary 128-aligned
    group sizes instead.  ``F.silu(g) * u`` and its backward run as one kernel each (``swiglu``),
    bit-identical to the eager torch ops."""

    def __init__(self, n_experts: int, d_model: int, ffn_dim: int, recipe: FP4Recipe | None = None, device=None):
        super().__init__()
        self.n_experts, self.d_model, self.ffn_dim = n_experts, d_model, ffn_dim
        self.gate_up = FP4GroupedLinear(n_experts, d_model, 2 * ffn_dim, recipe, device=device)
        self.down = FP4GroupedLinear(n_experts, ffn_dim, d_model, recipe, device=device)
        self.gate_up_b = nn.Parameter(torch.zeros(n_experts, 1, 2 * ffn_dim, device=device))
        self.down_b = nn.Parameter(torch.zeros(n_experts, 1, d_model, device=device))

    def refresh_fp4_cache(self) -> None:
        self.gate_up.refresh_fp4_cache()
        self.down.refresh_fp4_cache()

    def forward_sorted(self, x: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
        return self.down(swiglu(self.gate_up(x, offsets), "split"), offsets)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        e, cap, d = x.shape
        if cap % ALIGN:
            raise ValueError(f"FP4BatchedExperts: capacity must be a multiple of 128, got {cap}")
        offsets = torch.arange(e + 1, dtype=torch.int64, device=x.device) * cap
        h = self.gate_up(x.reshape(e * cap, d), offsets).view(e, cap, -1) + self.gate_up_b.to(x.dtype)
        hidden = swiglu(h.reshape(e * cap, 2 * self.ffn_dim), "split")  # one kernel, eager torch's roundings
        return self.down(hidden, offsets).view(e, cap, d) + self.down_b.to(x.dtype)
