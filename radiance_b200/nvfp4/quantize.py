"""NVFP4 quantization and GEMM: radiance's operator surface on the B200-native CUDA library.

Drop-in for ``radiance.nvfp4``'s quantize module (``src/radiance/nvfp4/quantize.py`` in
jamespa16/radiance): the same names, argument meanings, layouts and error text.  The layer below
it -- two Triton kernels and ``torch._scaled_mm_v2`` in the reference -- is replaced by the C ABI of
``include/radiance_nvfp4.h`` (``radiance_b200/_lib.py``): a TMA-fed quantizer and a tcgen05
block-scaled GEMM for sm_100a.  There is no CPU path: every op raises on a non-CUDA tensor, and if
the library is missing.

The reference's pure-torch format definition (``quantize_reference``, ``ref_quantize_rowblock``,
``ref_quantize_colblock``, ``encode_e2m1``, ``dequantize``, ``ref_to_blocked``, ``_block_scale``) is
re-exported from ``reference.py`` with the same names; nothing here calls it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib
from . import _trace

# Format constants -- quantize.py:16-32.
FP4_VALUES: tuple[float, ...] = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
FP4_MAX = 6.0
E4M3_MAX = 448.0
BLOCK = 16
TINY = 1e-12


# ------------------------------------------------------------------------------------------------
# Capability
# ------------------------------------------------------------------------------------------------


def nvfp4_supported(device: torch.device | str | None = None) -> bool:
    """True when the CUDA library is present and the device is an sm_100 (B200-class) GPU.

    Mirrors quantize.py:43-69, with the capability being this library rather than
    ``torch._scaled_mm_v2``.
    """
    if not torch.cuda.is_available():
        return False
    index = None
    if device is not None:
        device = torch.device(device)
        if device.type != "cuda":
            return False
        index = device.index
    if torch.cuda.get_device_capability(index)[0] != 10:
        return False
    try:
        _lib.load()
    except _lib.LibraryNotAvailable:
        return False
    return True


def require_nvfp4(reason: str) -> None:
    """quantize.py:72-82 -- raise with something actionable when FP4 cannot run here."""
    if nvfp4_supported():
        return
    cap = torch.cuda.get_device_capability() if torch.cuda.is_available() else None
    raise RuntimeError(
        f"{reason} needs NVFP4 support: the radiance_b200 CUDA library and an sm_100 (B200) GPU. "
        f"Got torch {torch.__version__}, device capability {cap}. "
        "Unset model.fp4_linear (or train.dtype: nvfp4) to train in bf16 instead."
    )


_SUPPORT_CACHE: dict[torch.device, bool] = {}


def _supported_cached(device: torch.device) -> bool:
    """quantize.py:739-746 -- memoised per device (hot path: once per linear per forward)."""
    if device not in _SUPPORT_CACHE:
        _SUPPORT_CACHE[device] = nvfp4_supported(device)
    return _SUPPORT_CACHE[device]


# ------------------------------------------------------------------------------------------------
# Layout helpers (pure indexing; quantize.py:142-157, :190-202, :293-305, :647-669)
# ------------------------------------------------------------------------------------------------


def pack_nibbles(code: torch.Tensor) -> torch.Tensor:
    """(..., K) uint8 codes -> (..., K // 2) ``float4_e2m1fn_x2``, element 2i in the low nibble."""
    return (code[..., 1::2] << 4 | code[..., 0::2]).view(torch.float4_e2m1fn_x2)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    raw = packed.view(torch.uint8)
    return torch.stack([raw & 0x0F, raw >> 4], dim=-1).reshape(*raw.shape[:-1], raw.shape[-1] * 2)


def blocked_offset(r: torch.Tensor, c: torch.Tensor, n_col_tiles: int) -> torch.Tensor:
    """Byte offset of scale element (r, c) in the SWIZZLE_32_4_4 layout."""
    tile = (r // 128) * n_col_tiles + (c // 4)
    return tile * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def scale_denominator(global_scale: torch.Tensor) -> torch.Tensor:
    """``6 * global_scale`` (the quantizer computes this same single fp32 multiply on the device)."""
    return FP4_MAX * global_scale


def hadamard_matrix(n: int = BLOCK, *, device=None, seed: int = 0) -> torch.Tensor:
    """Normalised n x n Sylvester Hadamard with a fixed random row-sign diagonal (quantize.py:647-659).

    The signs come from torch's CPU generator exactly as in the reference, so both libraries
    produce the same matrix for the same seed.
    """
    h = torch.ones(1, 1, dtype=torch.float32)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    signs = torch.where(torch.rand(n, 1, generator=gen) < 0.5, -1.0, 1.0)
    return (h / n**0.5 * signs).to(device)


def quantize_supported_shape(rows: int, cols: int) -> bool:
    """The kernels' shape contract (quantize.py:662-669): 128-row tiles, 64-wide column tiles."""
    return rows % 128 == 0 and cols % 64 == 0


def row_scale_bytes(rows: int, cols: int) -> int:
    return (rows // 128) * (cols // 64) * 512


def col_scale_bytes(rows: int, cols: int) -> int:
    return ((cols + 127) // 128) * (rows // 64) * 512


# ------------------------------------------------------------------------------------------------
# Operand type
# ------------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class NVFP4Tensor:
    """One GEMM operand (quantize.py:328-356): rows = output index, columns = contraction index."""

    packed: torch.Tensor  # float4_e2m1fn_x2, (rows, contraction // 2)
    scale: torch.Tensor  # float8_e4m3fn, SWIZZLE_32_4_4, flat
    global_scale: torch.Tensor  # fp32, 0-d

    @property
    def rows(self) -> int:
        return self.packed.shape[0]

    @property
    def contraction(self) -> int:
        return self.packed.shape[1] * 2


# ------------------------------------------------------------------------------------------------
# Device plumbing
# ------------------------------------------------------------------------------------------------

_WORKSPACES: dict[tuple[torch.device, int], torch.Tensor] = {}
_SEED_CACHE: dict[tuple[torch.device, int], torch.Tensor] = {}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _workspace(device: torch.device) -> torch.Tensor:
    """8 bytes of zeroed scratch for the amax reduction, one per (device, stream); every call
    leaves it zeroed again, so calls ordered on one stream can share it."""
    key = (device, _stream_ptr(device))
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = torch.zeros(2, dtype=torch.int32, device=device)
        _WORKSPACES[key] = ws
    return ws


def _default_seed(device: torch.device, value: int) -> torch.Tensor:
    """quantize.py:749-765 -- a cached 0-d device seed, read by the kernel through a pointer."""
    key = (device, value)
    if key not in _SEED_CACHE:
        _SEED_CACHE[key] = torch.tensor(value, device=device, dtype=torch.int64)
    return _SEED_CACHE[key]


def _require_cuda(x: torch.Tensor, what: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(
            f"{what}: expects a CUDA tensor on an sm_100 GPU; radiance_b200 has no CPU implementation"
        )


def _dtype_code(x: torch.Tensor) -> int:
    if x.dtype == torch.bfloat16:
        return _lib.RB_DTYPE_BF16
    if x.dtype == torch.float32:
        return _lib.RB_DTYPE_F32
    raise ValueError(f"nvfp4: unsupported input dtype {x.dtype} (bf16 or fp32)")


def _prep_input(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.to(torch.bfloat16)
    if x.stride(-1) != 1 or (x.stride(0) * x.element_size()) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


# ------------------------------------------------------------------------------------------------
# Global scale and quantization
# ------------------------------------------------------------------------------------------------


def global_scale_of(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-tensor fp32 global scale ``amax / (6 * 448)``, clamped at 1e-12 (quantize.py:205-213).

    One CUDA kernel, no host synchronisation.  ``out`` (a 0-d fp32 CUDA tensor) is written in
    place when given.
    """
    _require_cuda(x, "nvfp4.global_scale_of")
    lib = _lib.load()
    x2 = _prep_input(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x)
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=x.device)
    rows, cols = x2.shape
    tok = _trace.begin("amax", rows * cols * x2.element_size())
    _lib.check(
        lib.rb_nvfp4_global_scale(
            x2.data_ptr(), _dtype_code(x2), rows, cols, x2.stride(0), out.data_ptr(),
            _workspace(x.device).data_ptr(), _stream_ptr(x.device),
        ),
        "nvfp4.global_scale_of",
    )
    _trace.end(tok)
    return out


def update_and_global_scale_(w: torch.Tensor, update: torch.Tensor, alpha: float,
                             out: torch.Tensor | None = None) -> torch.Tensor:
    """``w.add_(update, alpha=alpha)`` and ``global_scale_of(w)`` of the result in one pass.

    The last in-place step of radiance's Muon update (``target.add_(orthogonalize(u),
    alpha=-lr*scale)``, src/radiance/optim.py:518) fused with the amax the weight's cache refresh
    needs (linear.py:193-210).  Each element is one fp32 fused multiply-add of the widened operands,
    rounded once to ``w``'s dtype.  ``w`` (bf16 or fp32) and ``update`` (bf16 or fp32, same shape)
    must be contiguous CUDA tensors; returns the 0-d fp32 global scale (``out`` when given).
    """
    _require_cuda(w, "nvfp4.update_and_global_scale_")
    if update.shape != w.shape:
        raise ValueError(f"nvfp4.update_and_global_scale_: update {tuple(update.shape)} vs weight {tuple(w.shape)}")
    if not w.is_contiguous():
        raise ValueError("nvfp4.update_and_global_scale_: the weight must be contiguous (it is updated in place)")
    lib = _lib.load()
    u = update.contiguous()
    if u.dtype not in (torch.bfloat16, torch.float32):
        u = u.float()
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=w.device)
    _lib.check(
        lib.rb_nvfp4_update_global_scale(
            w.data_ptr(), _dtype_code(w), u.data_ptr(), _dtype_code(u), w.numel(), float(alpha), out.data_ptr(),
            _workspace(w.device).data_ptr(), _stream_ptr(w.device),
        ),
        "nvfp4.update_and_global_scale_",
    )
    return out


_COLSUM_WS: dict[tuple[torch.device, int], torch.Tensor] = {}


def global_scale_and_column_sums(x: torch.Tensor, out: torch.Tensor | None = None,
                                 colsum: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(global_scale_of(x), x.sum(0) in fp32)`` from one read of ``x`` (two kernels, no host
    synchronisation).  The upstream gradient of a linear with a bias needs both: the global scale
    for its quantization and ``grad_y.sum(0)`` for the bias gradient (linear.py:146), which the
    reference computes with a second full pass over ``grad_y``.  The sums are fp32 accumulated in
    a fixed order (deterministic)."""
    _require_cuda(x, "nvfp4.global_scale_and_column_sums")
    lib = _lib.load()
    x2 = _prep_input(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x)
    rows, cols = x2.shape
    dev = x.device
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=dev)
    if colsum is None:
        colsum = torch.empty(cols, dtype=torch.float32, device=dev)
    need = int(lib.rb_nvfp4_global_scale_colsum_workspace(_dtype_code(x2), rows, cols))
    key = (dev, _stream_ptr(dev))
    ws = _COLSUM_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)  # the first 16 bytes start (and stay) zero
        _COLSUM_WS[key] = ws
    tok = _trace.begin("amax", rows * cols * x2.element_size())
    _lib.check(
        lib.rb_nvfp4_global_scale_colsum(
            x2.data_ptr(), _dtype_code(x2), rows, cols, x2.stride(0), out.data_ptr(), colsum.data_ptr(),
            ws.data_ptr(), _stream_ptr(dev),
        ),
        "nvfp4.global_scale_and_column_sums",
    )
    _trace.end(tok)
    return out, colsum


def _quantize_into(
    x: torch.Tensor,
    *,
    global_scale: torch.Tensor,
    hadamard: torch.Tensor | None,
    stochastic: bool,
    seed: torch.Tensor | int,
    row: tuple[torch.Tensor, torch.Tensor] | None,
    col: tuple[torch.Tensor, torch.Tensor] | None,
) -> None:
    lib = _lib.load()
    m, k = x.shape
    seed_t = None
    if stochastic:
        seed_t = seed if isinstance(seed, torch.Tensor) else _default_seed(x.device, int(seed))
        if seed_t.dtype != torch.int64 or not seed_t.is_cuda:
            seed_t = seed_t.to(device=x.device, dtype=torch.int64)
    had = None
    if hadamard is not None and hadamard.numel():
        had = hadamard.to(device=x.device, dtype=torch.float32).contiguous()
        if had.shape != (BLOCK, BLOCK):
            raise ValueError(f"nvfp4.quantize: hadamard must be {BLOCK}x{BLOCK}, got {tuple(had.shape)}")
    gs = global_scale
    if gs.dtype != torch.float32 or not gs.is_cuda:
        gs = gs.to(device=x.device, dtype=torch.float32)
    forms = (row is not None) + (col is not None)
    tok = _trace.begin("quantize", m * k * (x.element_size() + 0.5625 * forms))
    _lib.check(
        lib.rb_nvfp4_quantize(
            x.data_ptr(), _dtype_code(x), m, k, x.stride(0), gs.data_ptr(),
            None if had is None else had.data_ptr(), None if seed_t is None else seed_t.data_ptr(),
            None if row is None else row[0].data_ptr(), None if row is None else row[1].data_ptr(),
            None if col is None else col[0].data_ptr(), None if col is None else col[1].data_ptr(),
            _stream_ptr(x.device),
        ),
        "nvfp4.quantize",
    )
    _trace.end(tok)


_SYNC_WS: dict[tuple[torch.device, int], torch.Tensor] = {}


def _sync_workspace(device: torch.device) -> torch.Tensor:
    """16 bytes of zeroed device memory per (device, stream) for the fused global-scale quantizer's
    grid barrier; every call leaves it ready for the next, so calls ordered on one stream share it."""
    key = (device, _stream_ptr(device))
    ws = _SYNC_WS.get(key)
    if ws is None:
        ws = torch.zeros(4, dtype=torch.int32, device=device)
        _SYNC_WS[key] = ws
    return ws


def _quantize_auto_scale_into(
    x: torch.Tensor,
    *,
    out_scale: torch.Tensor,
    hadamard: torch.Tensor | None,
    stochastic: bool,
    seed: torch.Tensor | int,
    row: tuple[torch.Tensor, torch.Tensor] | None,
    col: tuple[torch.Tensor, torch.Tensor] | None,
) -> None:
    lib = _lib.load()
    m, k = x.shape
    seed_t = None
    if stochastic:
        seed_t = seed if isinstance(seed, torch.Tensor) else _default_seed(x.device, int(seed))
        if seed_t.dtype != torch.int64 or not seed_t.is_cuda:
            seed_t = seed_t.to(device=x.device, dtype=torch.int64)
    had = None
    if hadamard is not None and hadamard.numel():
        had = hadamard.to(device=x.device, dtype=torch.float32).contiguous()
        if had.shape != (BLOCK, BLOCK):
            raise ValueError(f"nvfp4.quantize: hadamard must be {BLOCK}x{BLOCK}, got {tuple(had.shape)}")
    if out_scale.dtype != torch.float32 or not out_scale.is_cuda or out_scale.numel() != 1:
        raise ValueError("nvfp4.quantize: the global-scale output must be a 0-d fp32 CUDA tensor")
    forms = (row is not None) + (col is not None)
    tok = _trace.begin("quantize", m * k * (x.element_size() + 0.5625 * forms))
    _lib.check(
        lib.rb_nvfp4_quantize_auto_scale(
            x.data_ptr(), _dtype_code(x), m, k, x.stride(0), out_scale.data_ptr(),
            None if had is None else had.data_ptr(), None if seed_t is None else seed_t.data_ptr(),
            None if row is None else row[0].data_ptr(), None if row is None else row[1].data_ptr(),
            None if col is None else col[0].data_ptr(), None if col is None else col[1].data_ptr(),
            _sync_workspace(x.device).data_ptr(), _stream_ptr(x.device),
        ),
        "nvfp4.quantize",
    )
    _trace.end(tok)


def quantize_auto_scale_into_(
    x: torch.Tensor,
    *,
    out_scale: torch.Tensor,
    row: tuple[torch.Tensor, torch.Tensor] | None = None,
    col: tuple[torch.Tensor, torch.Tensor] | None = None,
    hadamard: torch.Tensor | None = None,
    stochastic: bool = False,
    seed: torch.Tensor | int = 0,
) -> torch.Tensor:
    """``global_scale_of(x, out=out_scale)`` then ``quantize_into_(x, global_scale=out_scale, ...)`` in
    one kernel (``rb_nvfp4_quantize_auto_scale``): the same global scale and bytes, one launch fewer,
    and the quantizing pass re-reads ``x`` from L2 when it fits there.  Returns ``out_scale``."""
    _require_cuda(x, "nvfp4.quantize_auto_scale_into_")
    _check_shape(x, "rowblock" if col is None else "colblock")
    x = _prep_input(x)
    _quantize_auto_scale_into(x, out_scale=out_scale, hadamard=hadamard, stochastic=stochastic, seed=seed, row=row,
                              col=col)
    return out_scale


def _check_shape(x: torch.Tensor, form: str) -> None:
    if x.dim() != 2:
        raise ValueError(f"nvfp4.quantize expects a 2-D tensor, got shape {tuple(x.shape)}")
    m, k = x.shape
    if not quantize_supported_shape(m, k):
        raise ValueError(f"nvfp4.quantize {form} needs rows % 128 == 0 and cols % 64 == 0, got {(m, k)}")


def _alloc_row(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    return (
        torch.empty(m, k // 2, device=x.device, dtype=torch.uint8),
        torch.empty(row_scale_bytes(m, k), device=x.device, dtype=torch.uint8),
    )


def _alloc_col(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    return (
        torch.empty(k, m // 2, device=x.device, dtype=torch.uint8),
        torch.empty(col_scale_bytes(m, k), device=x.device, dtype=torch.uint8),
    )


def _as_nvfp4(buf: tuple[torch.Tensor, torch.Tensor], gs: torch.Tensor) -> NVFP4Tensor:
    return NVFP4Tensor(
        packed=buf[0].view(torch.float4_e2m1fn_x2), scale=buf[1].view(torch.float8_e4m3fn), global_scale=gs
    )


def quantize(
    x: torch.Tensor,
    axis: int,
    *,
    global_scale: torch.Tensor | None = None,
    hadamard: torch.Tensor | None = None,
    stochastic: bool = False,
    seed: torch.Tensor | int = 0,
) -> NVFP4Tensor:
    """Quantize ``x`` to NVFP4 (quantize.py:672-736).  ``axis=-1`` blocks along the last dim
    (rowblock), ``axis=0`` along the first (colblock, output transposed).

    Bit-identical to the reference's ``quantize_reference`` on codes and scale bytes.
    ``stochastic`` selects stochastic rounding with ``seed`` (a 0-d int64 tensor read on the
    device, or an int).  ``hadamard`` applies to the colblock form only, as in the reference.
    """
    _require_cuda(x, "nvfp4.quantize")
    if x.dim() != 2:
        raise ValueError(f"nvfp4.quantize expects a 2-D tensor, got shape {tuple(x.shape)}")
    if axis in (-1, 1):
        form = "rowblock"
    elif axis == 0:
        form = "colblock"
    else:
        raise ValueError(f"nvfp4.quantize supports axis 0 or -1, got {axis}")
    _check_shape(x, form)
    x = _prep_input(x)
    buf = _alloc_row(x) if form == "rowblock" else _alloc_col(x)
    row, col = (buf, None) if form == "rowblock" else (None, buf)
    had = None if form == "rowblock" else hadamard
    if global_scale is None:  # the global scale and the quantization in one launch
        global_scale = torch.empty((), dtype=torch.float32, device=x.device)
        _quantize_auto_scale_into(x, out_scale=global_scale, hadamard=had, stochastic=stochastic, seed=seed, row=row,
                                  col=col)
    else:
        _quantize_into(x, global_scale=global_scale, hadamard=had, stochastic=stochastic, seed=seed, row=row, col=col)
    return _as_nvfp4(buf, global_scale)


def quantize_both(
    x: torch.Tensor,
    *,
    global_scale: torch.Tensor | None = None,
    hadamard: torch.Tensor | None = None,
    stochastic: bool = False,
    seed: torch.Tensor | int = 0,
) -> tuple[NVFP4Tensor, NVFP4Tensor]:
    """Both forms from one read of ``x``: ``(quantize(x, -1, ...), quantize(x, 0, hadamard=...))``.

    Bit-identical to the two separate calls for round-to-nearest.  Without ``global_scale`` the
    global scale is computed in the same launch (``quantize_auto_scale_into_``).  This is what ``FP4Linear``
    uses: the reference quantizes each activation and each upstream gradient both ways per
    micro-batch (linear.py:80, :99, :129, :133), two full reads of the bf16 tensor.
    """
    _require_cuda(x, "nvfp4.quantize_both")
    _check_shape(x, "rowblock+colblock")
    x = _prep_input(x)
    row, col = _alloc_row(x), _alloc_col(x)
    if global_scale is None:  # the global scale and both forms in one launch
        global_scale = torch.empty((), dtype=torch.float32, device=x.device)
        _quantize_auto_scale_into(x, out_scale=global_scale, hadamard=hadamard, stochastic=stochastic, seed=seed,
                                  row=row, col=col)
    else:
        _quantize_into(
            x, global_scale=global_scale, hadamard=hadamard, stochastic=stochastic, seed=seed, row=row, col=col
        )
    return _as_nvfp4(row, global_scale), _as_nvfp4(col, global_scale)


def quantize_into_(
    x: torch.Tensor,
    *,
    global_scale: torch.Tensor,
    row: tuple[torch.Tensor, torch.Tensor] | None = None,
    col: tuple[torch.Tensor, torch.Tensor] | None = None,
    hadamard: torch.Tensor | None = None,
    stochastic: bool = False,
    seed: torch.Tensor | int = 0,
) -> None:
    """Quantize into caller-owned (packed, scale) uint8 buffers -- the weight-cache refresh writes
    straight into ``FP4Linear``'s buffers this way, keeping their data pointers stable."""
    _require_cuda(x, "nvfp4.quantize_into_")
    _check_shape(x, "rowblock" if col is None else "colblock")
    x = _prep_input(x)
    _quantize_into(x, global_scale=global_scale, hadamard=hadamard, stochastic=stochastic, seed=seed, row=row, col=col)


# ------------------------------------------------------------------------------------------------
# GEMM
# ------------------------------------------------------------------------------------------------

_OUT_CODES = {torch.bfloat16: _lib.RB_OUT_BF16, torch.float32: _lib.RB_OUT_F32}


def _gemm(
    a_packed: torch.Tensor,
    a_scale: torch.Tensor,
    b_packed: torch.Tensor,
    b_scale: torch.Tensor,
    alpha_a: torch.Tensor | None,
    alpha_b: torch.Tensor | None,
    bias: torch.Tensor | None,
    out_dtype: torch.dtype,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    _require_cuda(a_packed, "nvfp4.mm")
    lib = _lib.load()
    m, k2 = a_packed.shape
    n, k2b = b_packed.shape
    if k2 != k2b:
        raise ValueError(f"nvfp4.mm: contraction mismatch {2 * k2} vs {2 * k2b}")
    k = 2 * k2
    native = out_dtype if out_dtype in _OUT_CODES else torch.float32
    if out is None or out.dtype != native:
        out = torch.empty(m, n, device=a_packed.device, dtype=native)
    bias_code = 0
    if bias is not None:
        if bias.dtype not in (torch.bfloat16, torch.float32):
            bias = bias.to(torch.float32)
        bias = bias.contiguous()
        if bias.data_ptr() % 16:  # the epilogue reads the bias in 16-byte vectors
            bias = bias.clone()
        bias_code =_lib.RB_DTYPE_BF16 if bias.dtype == torch.bfloat16 else _lib.RB_DTYPE_F32
    tok = _trace.begin("gemm", 2.0 * m * n * k)
    _lib.check(
        lib.rb_nvfp4_gemm(
            a_packed.data_ptr(), a_scale.data_ptr(), b_packed.data_ptr(), b_scale.data_ptr(), m, n, k,
            None if alpha_a is None else alpha_a.data_ptr(), None if alpha_b is None else alpha_b.data_ptr(),
            None if bias is None else bias.data_ptr(), bias_code, out.data_ptr(), _OUT_CODES[native], out.stride(0),
            _stream_ptr(a_packed.device),
        ),
        "nvfp4.mm",
    )
    _trace.end(tok)
    return out if native == out_dtype else out.to(out_dtype)


def _nvfp4_mm_name() -> str:
    """The reference registers its op as ``radiance::nvfp4_mm`` (quantize.py:359-371) and code that
    swaps this package in finds it under that name.  Should radiance itself be loaded in the same
    process, its registration stands and this one moves to ``radiance_b200::nvfp4_mm``."""
    try:
        torch.ops.radiance.nvfp4_mm  # noqa: B018 -- raises when no such op is registered
    except (AttributeError, RuntimeError):
        return "radiance::nvfp4_mm"
    return "radiance_b200::nvfp4_mm"


@torch.library.custom_op(_nvfp4_mm_name(), mutates_args=())
def nvfp4_mm(
    a_packed: torch.Tensor,
    a_scale: torch.Tensor,
    b_packed: torch.Tensor,
    b_scale: torch.Tensor,
) -> torch.Tensor:
    """``a @ b.T`` in NVFP4 without the global scales: (M, K/2) x (N, K/2) -> (M, N) bf16.

    Same contract as the reference's ``radiance::nvfp4_mm`` (quantize.py:359-387); a custom op so
    ``torch.compile`` keeps it in the graph as an opaque call.
    """
    return _gemm(
        a_packed.view(torch.uint8), a_scale.view(torch.uint8), b_packed.view(torch.uint8), b_scale.view(torch.uint8),
        None, None, None, torch.bfloat16,
    )


@nvfp4_mm.register_fake
def _nvfp4_mm_fake(a_packed, a_scale, b_packed, b_scale):
    return a_packed.new_empty((a_packed.shape[0], b_packed.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("radiance_b200::nvfp4_linear_mm", mutates_args=())
def nvfp4_linear_mm(
    a_packed: torch.Tensor,
    a_scale: torch.Tensor,
    a_gs: torch.Tensor,
    b_packed: torch.Tensor,
    b_scale: torch.Tensor,
    b_gs: torch.Tensor,
    bias: torch.Tensor | None,
    out_dtype: torch.dtype,
) -> torch.Tensor:
    """``(a @ b.T) * (ga * gb) + bias`` in one kernel: the global-scale fold, bias add and output
    cast of quantize.py:400-409 and linear.py:82-83 happen in the GEMM epilogue."""
    return _gemm(
        a_packed.view(torch.uint8), a_scale.view(torch.uint8), b_packed.view(torch.uint8), b_scale.view(torch.uint8),
        a_gs, b_gs, bias, out_dtype,
    )


@nvfp4_linear_mm.register_fake
def _nvfp4_linear_mm_fake(a_packed, a_scale, a_gs, b_packed, b_scale, b_gs, bias, out_dtype):
    return a_packed.new_empty((a_packed.shape[0], b_packed.shape[0]), dtype=out_dtype)


# ------------------------------------------------------------------------------------------------
# SwiGLU producer: the gate/up GEMM whose epilogue also emits h and its global scale
# ------------------------------------------------------------------------------------------------

SWIGLU_GROUP = 32  # hidden units per [gate | up] block of the interleaved layout


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Stack the gate and up projections' rows (weights ``(H, in)`` or biases ``(H,)``) into the
    ``(2H, ...)`` order ``swiglu_mm`` reads: blocks of 64 rows, [32 gate rows | the 32 up rows of
    the same hidden units]."""
    if gate.shape != up.shape or gate.shape[0] % SWIGLU_GROUP:
        raise ValueError(f"interleave_gate_up: gate {tuple(gate.shape)} and up {tuple(up.shape)} must match, "
                         f"with rows % {SWIGLU_GROUP} == 0")
    h, rest = gate.shape[0], gate.shape[1:]
    blocks = (h // SWIGLU_GROUP, SWIGLU_GROUP, *rest)
    return torch.stack([gate.reshape(blocks), up.reshape(blocks)], dim=1).reshape(2 * h, *rest)


def split_gate_up(gu: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The interleaved order along the last dimension -> gate, up ``(..., H)`` (contiguous copies)."""
    two_h = gu.shape[-1]
    v = gu.reshape(*gu.shape[:-1], two_h // (2 * SWIGLU_GROUP), 2, SWIGLU_GROUP)
    return (v[..., 0, :].reshape(*gu.shape[:-1], two_h // 2), v[..., 1, :].reshape(*gu.shape[:-1], two_h // 2))


def merge_gate_up(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """Inverse of ``split_gate_up``: gate and up ``(..., H)`` -> the interleaved ``(..., 2H)``."""
    lead, h = g.shape[:-1], g.shape[-1]
    blocks = (*lead, h // SWIGLU_GROUP, SWIGLU_GROUP)
    return torch.stack([g.reshape(blocks), u.reshape(blocks)], dim=-2).reshape(*lead, 2 * h)


def swiglu_mm(a: NVFP4Tensor, b: NVFP4Tensor, *, bias=None, out: torch.Tensor | None = None,
              h: torch.Tensor | None = None, h_global_scale: torch.Tensor | None = None):
    """The gate/up projection of a SwiGLU FFN and its activation in one GEMM.

    ``b`` holds the gate and up weights interleaved (``interleave_gate_up``).  Returns
    ``(gu, h, gs)``: ``gu = (a @ b.T) * (ga * gb) + bias`` in bf16 (the pre-activations, in the
    interleaved order), ``h = F.silu(g) * u`` in bf16 with the roundings of radiance's eager
    ``F.silu(gate_proj(x)) * up_proj(x)`` (src/radiance/model/ffn.py:32), and
    ``gs = global_scale_of(h)``, all from the GEMM's epilogue -- the next linear's quantizer takes
    ``gs`` and reads ``h`` once.
    """
    _require_cuda(a.packed, "nvfp4.swiglu_mm")
    lib = _lib.load()
    ap, asc = a.packed.view(torch.uint8), a.scale.view(torch.uint8)
    bp, bsc = b.packed.view(torch.uint8), b.scale.view(torch.uint8)
    m, k2 = ap.shape
    n, k2b = bp.shape
    if k2 != k2b:
        raise ValueError(f"nvfp4.swiglu_mm: contraction mismatch {2 * k2} vs {2 * k2b}")
    if n % (2 * SWIGLU_GROUP):
        raise ValueError(f"nvfp4.swiglu_mm: the interleaved gate/up operand needs rows % 64 == 0, got {n}")
    dev = ap.device
    if out is None:
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    if h is None:
        h = torch.empty(m, n // 2, device=dev, dtype=torch.bfloat16)
    if h_global_scale is None:
        h_global_scale = torch.empty((), device=dev, dtype=torch.float32)
    bias_code = 0
    if bias is not None:
        if bias.dtype not in (torch.bfloat16, torch.float32):
            bias = bias.to(torch.float32)
        bias = bias.contiguous()
        if bias.data_ptr() % 16:
            bias = bias.clone()
        bias_code = _lib.RB_DTYPE_BF16 if bias.dtype == torch.bfloat16 else _lib.RB_DTYPE_F32
    tok = _trace.begin("gemm", 2.0 * m * n * 2 * k2)
    _lib.check(
        lib.rb_nvfp4_gemm_swiglu(
            ap.data_ptr(), asc.data_ptr(), bp.data_ptr(), bsc.data_ptr(), m, n, 2 * k2,
            a.global_scale.data_ptr(), b.global_scale.data_ptr(),
            None if bias is None else bias.data_ptr(), bias_code, out.data_ptr(), out.stride(0),
            h.data_ptr(), h.stride(0), _workspace(dev).data_ptr(), h_global_scale.data_ptr(), _stream_ptr(dev),
        ),
        "nvfp4.swiglu_mm",
    )
    _trace.end(tok)
    return out, h, h_global_scale


def swiglu_backward(grad_h: torch.Tensor, gu: torch.Tensor, out: torch.Tensor | None = None,
                    out_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The gradient of ``h = F.silu(g) * u`` with respect to the interleaved pre-activations ``gu``
    (``swiglu_mm``'s layout), and that gradient's global scale, in one kernel.  Bit-identical to
    eager autograd's ``grad_h * F.silu(g)`` and ``aten.silu_backward(grad_h * u, g)`` (ffn.py:32).
    Returns ``(grad_gu, global_scale_of(grad_gu))``."""
    _require_cuda(grad_h, "nvfp4.swiglu_backward")
    lib = _lib.load()
    gh = grad_h.reshape(-1, grad_h.shape[-1])
    if gh.stride(-1) != 1 or gh.data_ptr() % 16 or gh.stride(0) % 8:
        gh = gh.contiguous()
    g2 = gu.reshape(-1, gu.shape[-1])
    if g2.stride(-1) != 1 or g2.data_ptr() % 16 or g2.stride(0) % 8:
        g2 = g2.contiguous()
    if gh.dtype != torch.bfloat16 or g2.dtype != torch.bfloat16:
        raise ValueError("nvfp4.swiglu_backward: bf16 tensors expected")
    rows, hidden = gh.shape
    if g2.shape != (rows, 2 * hidden):
        raise ValueError(f"nvfp4.swiglu_backward: pre-activations {tuple(g2.shape)} vs gradient {tuple(gh.shape)}")
    if out is None:
        out = torch.empty(rows, 2 * hidden, dtype=torch.bfloat16, device=gh.device)
    if out_scale is None:
        out_scale = torch.empty((), dtype=torch.float32, device=gh.device)
    _lib.check(
        lib.rb_nvfp4_swiglu_backward(
            gh.data_ptr(), gh.stride(0), g2.data_ptr(), g2.stride(0), rows, hidden, out.data_ptr(), out.stride(0),
            out_scale.data_ptr(), _workspace(gh.device).data_ptr(), _stream_ptr(gh.device),
        ),
        "nvfp4.swiglu_backward",
    )
    return out, out_scale


def _swiglu_layout(gu: torch.Tensor, layout: str, what: str):
    """(rows x 2*hidden bf16 view, hidden, up offset in elements, group stride) of a gate/up tensor:
    ``"split"`` is radiance's [gate | up] halves (ffn.py:148-153), ``"interleaved"`` the
    [32 gate | 32 up] order of ``swiglu_mm``."""
    _require_cuda(gu, what)
    g2 = gu.reshape(-1, gu.shape[-1])
    if g2.stride(-1) != 1 or g2.data_ptr() % 16 or g2.stride(0) % 8:
        g2 = g2.contiguous()
    if g2.dtype != torch.bfloat16:
        raise ValueError(f"{what}: bf16 pre-activations expected")
    if g2.shape[1] % 64:
        raise ValueError(f"{what}: the gate/up width must be a multiple of 64, got {g2.shape[1]}")
    hidden = g2.shape[1] // 2
    if layout == "split":
        return g2, hidden, hidden, 32
    if layout == "interleaved":
        return g2, hidden, 32, 64
    raise ValueError(f"{what}: layout must be 'split' or 'interleaved', got {layout!r}")


def swiglu_forward(gu: torch.Tensor, layout: str = "split", out: torch.Tensor | None = None,
                   out_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``h = F.silu(g) * u`` from the gate/up pre-activations ``gu`` (``layout`` as in
    ``_swiglu_layout``), bit-identical to the eager bf16 torch ops, and ``global_scale_of(h)``, in
    one kernel.  Returns ``(h, scale)`` with h of shape ``gu.shape[:-1] + (hidden,)``."""
    what = "nvfp4.swiglu_forward"
    g2, hidden, du, blk = _swiglu_layout(gu, layout, what)
    rows = g2.shape[0]
    if out is None:
        out = torch.empty(rows, hidden, dtype=torch.bfloat16, device=g2.device)
    if out_scale is None:
        out_scale = torch.empty((), dtype=torch.float32, device=g2.device)
    lib = _lib.load()
    _lib.check(
        lib.rb_nvfp4_swiglu_forward_strided(
            g2.data_ptr(), g2.data_ptr() + 2 * du, g2.stride(0), blk, rows, hidden, out.data_ptr(), out.stride(0),
            out_scale.data_ptr(), _workspace(g2.device).data_ptr(), _stream_ptr(g2.device),
        ),
        what,
    )
    return out.reshape(*gu.shape[:-1], hidden), out_scale


def swiglu_backward_strided(grad_h: torch.Tensor, gu: torch.Tensor, layout: str = "split",
                            out: torch.Tensor | None = None,
                            out_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The gradient of ``swiglu_forward`` with respect to ``gu``, in ``gu``'s layout, and its global
    scale; bit-identical to eager autograd's backward of ``F.silu(g) * u``."""
    what = "nvfp4.swiglu_backward"
    g2, hidden, du, blk = _swiglu_layout(gu, layout, what)
    gh = grad_h.reshape(-1, hidden)
    if gh.stride(-1) != 1 or gh.data_ptr() % 16 or gh.stride(0) % 8:
        gh = gh.contiguous()
    if gh.dtype != torch.bfloat16 or gh.shape[0] != g2.shape[0]:
        raise ValueError(f"{what}: a bf16 gradient of {g2.shape[0]} x {hidden} expected, got "
                         f"{tuple(grad_h.shape)} {grad_h.dtype}")
    rows = g2.shape[0]
    if out is None:
        out = torch.empty(rows, 2 * hidden, dtype=torch.bfloat16, device=g2.device)
    if out_scale is None:
        out_scale = torch.empty((), dtype=torch.float32, device=g2.device)
    lib = _lib.load()
    _lib.check(
        lib.rb_nvfp4_swiglu_backward_strided(
            gh.data_ptr(), gh.stride(0), g2.data_ptr(), g2.data_ptr() + 2 * du, g2.stride(0), blk, rows, hidden,
            out.data_ptr(), out.data_ptr() + 2 * du, out.stride(0), blk, out_scale.data_ptr(),
            _workspace(g2.device).data_ptr(), _stream_ptr(g2.device),
        ),
        what,
    )
    return out.reshape(gu.shape), out_scale


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu, layout):
        h, _ = swiglu_forward(gu, layout)
        ctx.save_for_backward(gu)
        ctx.layout = layout
        return h

    @staticmethod
    def backward(ctx, grad_h):
        (gu,) = ctx.saved_tensors
        grad_gu, _ = swiglu_backward_strided(grad_h, gu, ctx.layout)
        return grad_gu, None


def swiglu(gu: torch.Tensor, layout: str = "split") -> torch.Tensor:
    """Differentiable ``F.silu(g) * u`` on gate/up pre-activations (``layout`` "split": radiance's
    ``[gate | up]`` halves, ffn.py:148-153; "interleaved": ``swiglu_mm``'s order): one kernel
    forward and one backward, outputs and gradients bit-identical to the eager torch ops."""
    return _SwiGLUFn.apply(gu, layout)


def mm(a: NVFP4Tensor, b: NVFP4Tensor, *, out_dtype: torch.dtype = torch.bfloat16, bias=None) -> torch.Tensor:
    """``a @ b.T`` with the global scales folded back in (quantize.py:400-409).

    The fold, the optional bias and the cast to ``out_dtype`` run in the GEMM's epilogue: one
    rounding to ``out_dtype`` where the reference rounds to bf16 and again after the multiply.
    """
    return nvfp4_linear_mm(a.packed, a.scale, a.global_scale, b.packed, b.scale, b.global_scale, bias, out_dtype)
