"""CPU oracle for the NVFP4 linear path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker (or as the timed CPU baseline).  The product path in
``radiance_b200`` never imports it; the CUDA extension is the only implementation that ships.

This is a numpy restatement of radiance's pure-torch NVFP4 emulation,
``src/radiance/nvfp4/quantize.py`` in jamespa16/radiance.  Each function names the reference lines
it follows.  Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against
vectors produced by the reference itself (``tests/golden/make_golden.py`` imports the reference and
writes ``tests/golden/nvfp4_golden.npz``), bit-exactly on packed nibbles and scale bytes.

Arithmetic is float32 throughout, one IEEE rounding per operation, exactly as torch's CPU kernels
do it: numpy float32 ``/`` and ``*`` are correctly rounded, so ``x / (divisor * gs)`` here is the
same two roundings as the reference's ``xb / (divisor * global_scale)``.
"""

from __future__ import annotations

import numpy as np

# Format constants -- quantize.py:16-32.
FP4_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
FP4_MAX = np.float32(6.0)
E4M3_MAX = np.float32(448.0)
BLOCK = 16
TINY = np.float32(1e-12)

_F32 = np.float32


def _e4m3_table() -> np.ndarray:
    """Value of every non-negative finite e4m3fn byte 0x00..0x7E (0x7F is NaN)."""
    vals = np.zeros(127, dtype=np.float64)
    for b in range(127):
        e, m = b >> 3, b & 7
        vals[b] = (m / 8.0) * 2.0**-6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals.astype(np.float32)


E4M3_VALUES = _e4m3_table()


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (torch's ``.to(torch.bfloat16)``)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def global_scale_of(x: np.ndarray) -> np.float32:
    """quantize.py:205-213 -- ``(|x|.amax().float() / (6 * 448)).clamp(min=1e-12)``, one fp32 divide."""
    amax = np.abs(x.astype(np.float32)).max() if x.size else _F32(0.0)
    return np.maximum(_F32(amax) / _F32(FP4_MAX * E4M3_MAX), TINY)


def scale_denominator(gs) -> np.float32:
    """quantize.py:190-202 -- ``6 * global_scale``, one fp32 multiply."""
    return _F32(FP4_MAX * _F32(gs))


def block_scale(amax: np.ndarray, gs) -> tuple[np.ndarray, np.ndarray]:
    """quantize.py:160-187 -- block amax -> (e4m3 byte, fp32 divisor).

    ``scale = clamp(amax / denom, 1e-12, 448)``; the byte is the smallest e4m3 value >= scale (the
    reference casts round-to-nearest-even and bumps one code up when the cast landed below, never
    onto 0x7F); the divisor is that value, or 1.0 for an all-zero block.
    """
    amax = amax.astype(np.float32)
    scale = np.minimum(np.maximum(amax / scale_denominator(gs), TINY), E4M3_MAX)
    byte = np.searchsorted(E4M3_VALUES, scale, side="left").astype(np.int64)
    byte = np.minimum(byte, 0x7E).astype(np.uint8)
    divisor = np.where(amax > 0, E4M3_VALUES[byte], _F32(1.0)).astype(np.float32)
    return byte, divisor


def encode_e2m1(a: np.ndarray, sign: np.ndarray, u: np.ndarray | None = None) -> np.ndarray:
    """quantize.py:93-139 -- magnitudes in [0, 6] -> 4-bit codes, sign in bit 3.

    Without ``u``: the round-to-nearest-even ladder (``>`` and ``>=`` alternate so ties go to the
    even code).  With ``u`` (uniform [0, 1) per element): stochastic rounding, up with probability
    ``(a - lo) / (hi - lo)``.
    """
    a = a.astype(np.float32)
    if u is None:
        code = (
            (a > 0.25).astype(np.uint8)
            + (a >= 0.75)
            + (a > 1.25)
            + (a >= 1.75)
            + (a > 2.5)
            + (a >= 3.5)
            + (a > 5.0)
        ).astype(np.uint8)
    else:
        lo = (
            (a >= 0.5).astype(np.uint8)
            + (a >= 1.0)
            + (a >= 1.5)
            + (a >= 2.0)
            + (a >= 3.0)
            + (a >= 4.0)
            + (a >= 6.0)
        ).astype(np.uint8)
        levels = np.array(FP4_VALUES + (6.0,), dtype=np.float32)
        lo_v = levels[lo]
        hi_v = levels[lo + 1]
        span = np.maximum(hi_v - lo_v, TINY)
        with np.errstate(invalid="ignore", divide="ignore"):
            frac = np.where(hi_v > lo_v, (a - lo_v) / span, _F32(0.0)).astype(np.float32)
        code = np.minimum(lo + (u.astype(np.float32) < frac), 7).astype(np.uint8)
    return (code | (sign.astype(np.uint8) << 3)).astype(np.uint8)


# --- the device's stochastic-rounding stream -----------------------------------------------------
# radiance draws u = tl.rand(seed, row * K + col) per element (quantize.py:566-567, :622-623) and
# rounds up when u < (a - lo) / (hi - lo).  The B200 kernels keep that rule but round with the
# hardware convert cvt.rs.satfinite.e2m1x4.f32 and their own counter-based generator, restated here
# so the device output can be checked bit for bit.
#
# The convert takes four values and 32 random bits `rbits`.  With R0 = rbits[23:16]:rbits[7:0] and
# R2 = rbits[31:24]:rbits[15:8] (16-bit numbers), element 0 uses R0, element 1 the bit reversal of
# R0, element 2 R2 and element 3 the bit reversal of R2; an element rounds up when
# floor(f * 2^16) + R >= 2^16, f the fraction of the grid step above the level below (so up with
# probability floor(f * 2^16) / 2^16).  This was measured on the B200 for every single-bit rbits
# against fractions on every binade of [0.25, 6] and agrees with the statistics over random rbits.
#
# Each 32-element unit draws from its own stream:
#   S       = mix32(lo32(unit) ^ key(hi32(unit)))          (mix32: the lowbias32 finalizer)
#   r_j     = A^j S + C (A^(j-1) + ... + 1)  mod 2^32      (j = 0..15; a full-period LCG,
#                                                           A = 747796405, C = 2891336453: PCG's
#                                                           32-bit constants)
#   rbits_c = (r_2c >> 16) | (r_2c+1 & 0xFFFF0000)         for the convert of unit elements 4c..4c+3
#   key(0)  = mix32(lo32(seed) ^ 0x9E3779B9) ^ mix32(hi32(seed) + 0x7F4A7C15) for the rowblock
#             form, and mix32(that ^ 0x85EBCA6B) for the colblock form
#   key(h)  = key(0) ^ mix32(h + 0x632BE5AB)                for h != 0
# Rowblock units are numbered row * (K / 32) + col / 32; unit element e is column 32 * (col / 32) + e.
# Colblock units are numbered (col / 2) * (M / 16) + row / 16 (a column pair's 16-row group); unit
# element e is column 2 * (col / 2) + e / 16, row 16 * (row / 16) + e % 16.

_M32 = np.uint64(0xFFFFFFFF)
LCG_A, LCG_C = 747796405, 2891336453
SR_UNIT = 32


def mix32(x) -> np.ndarray:
    """lowbias32 (C. Wellons' hash-prospector finalizer) on uint32 values."""
    x = np.asarray(x, dtype=np.uint64) & _M32
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & _M32
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & _M32
    x ^= x >> np.uint64(16)
    return x.astype(np.uint32)


def sr_key(seed: int) -> np.uint32:
    s = np.uint64(int(seed) & 0xFFFFFFFFFFFFFFFF)
    lo, hi = s & _M32, s >> np.uint64(32)
    return np.uint32(mix32(lo ^ np.uint64(0x9E3779B9)) ^ mix32((hi + np.uint64(0x7F4A7C15)) & _M32))


def sr_key_col(seed: int) -> np.uint32:
    return np.uint32(mix32(np.uint64(sr_key(seed)) ^ np.uint64(0x85EBCA6B)))


def sr_unit_seeds(unit: np.ndarray, key) -> np.ndarray:
    """S of units ``unit`` (uint64 unit indices)."""
    unit = np.asarray(unit, dtype=np.uint64)
    key = np.uint64(key)
    hi = unit >> np.uint64(32)
    keyh = np.where(hi == 0, key, key ^ mix32((hi + np.uint64(0x632BE5AB)) & _M32).astype(np.uint64))
    return mix32((unit & _M32) ^ keyh)


def lcg_jump(s: np.ndarray, j: np.ndarray) -> np.ndarray:
    """r_j = A^j S + C_j mod 2^32, elementwise (j < 16)."""
    mul = np.ones(16, dtype=np.uint64)
    add = np.zeros(16, dtype=np.uint64)
    for i in range(1, 16):
        mul[i] = (mul[i - 1] * np.uint64(LCG_A)) & _M32
        add[i] = (add[i - 1] * np.uint64(LCG_A) + np.uint64(LCG_C)) & _M32
    j = np.asarray(j)
    return ((np.asarray(s, dtype=np.uint64) * mul[j] + add[j]) & _M32).astype(np.uint32)


def sr_rbits(s: np.ndarray, c: np.ndarray) -> np.ndarray:
    """rbits of convert c (0..7) of units with stream seeds s."""
    c = np.asarray(c, dtype=np.int64)
    lo = lcg_jump(s, 2 * c).astype(np.uint64)
    hi = lcg_jump(s, 2 * c + 1).astype(np.uint64)
    return ((lo >> np.uint64(16)) | (hi & np.uint64(0xFFFF0000))).astype(np.uint32)


def _bitrev16(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.uint32)
    out = np.zeros_like(x)
    for b in range(16):
        out |= ((x >> np.uint32(b)) & np.uint32(1)) << np.uint32(15 - b)
    return out


def convert_random16(rbits: np.ndarray, n: np.ndarray) -> np.ndarray:
    """The 16 random bits element n (0..3) of one cvt.rs e2m1x4 convert takes from rbits."""
    rb = np.asarray(rbits, dtype=np.uint32)
    r0 = (((rb >> np.uint32(16)) & np.uint32(0xFF)) << np.uint32(8)) | (rb & np.uint32(0xFF))
    r2 = ((rb >> np.uint32(24)) << np.uint32(8)) | ((rb >> np.uint32(8)) & np.uint32(0xFF))
    n = np.asarray(n)
    return np.where(n == 0, r0, np.where(n == 1, _bitrev16(r0), np.where(n == 2, r2, _bitrev16(r2)))).astype(np.uint32)


def _random16(unit: np.ndarray, e: np.ndarray, key) -> np.ndarray:
    return convert_random16(sr_rbits(sr_unit_seeds(unit, key), e // 4), e % 4)


def sr_stream_row(rows: int, cols: int, seed: int) -> np.ndarray:
    """(rows, cols) 16-bit random numbers of the rowblock form, indexed by element position."""
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(cols, dtype=np.uint64)[None, :]
    unit = r * np.uint64(cols // SR_UNIT) + c // np.uint64(SR_UNIT)
    e = np.broadcast_to((c % np.uint64(SR_UNIT)).astype(np.int64), (rows, cols))
    return _random16(unit, e, sr_key(seed))


def sr_stream_col(rows: int, cols: int, seed: int) -> np.ndarray:
    """(rows, cols) 16-bit random numbers of the colblock form, indexed by the element's (row, col)
    in x."""
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(cols, dtype=np.uint64)[None, :]
    unit = (c >> np.uint64(1)) * np.uint64(rows // BLOCK) + (r >> np.uint64(4))
    e = ((c & np.uint64(1)) * np.uint64(16) + (r & np.uint64(15))).astype(np.int64)
    return _random16(unit, e, sr_key_col(seed))


def sr_nibbles(q: np.ndarray, r16: np.ndarray) -> np.ndarray:
    """The device's stochastic rounding of quotients q (already clamped to +-6) with 16-bit random
    numbers r16: the rule of quantize.py:122-138 with the fraction truncated to 16 bits -- up when
    floor(f * 2^16) + r16 >= 2^16, f = (a - lo) / (hi - lo).  Sign in bit 3 (q < 0).

    The device's quotient here is RN(x * RN(1/d)) rather than the IEEE x / d (one ulp of it moves
    the probability of rounding up by at most 2^-22, below the 2^-16 resolution above);
    ``_quantize_blocks`` forms it that way when given random numbers.  On the Hadamard path the
    device evaluates the same product as (4y) * (RN(1/d) / 4), identical unless RN(1/d) / 4 is
    subnormal (divisors above 2^124)."""
    q = np.asarray(q, dtype=np.float32)
    a = np.minimum(np.abs(q), np.float32(6.0)).astype(np.float64)
    levels = np.array(FP4_VALUES + (6.0,), dtype=np.float64)
    lo = np.clip(np.searchsorted(levels[:8], a, side="right") - 1, 0, 7)
    span = np.where(lo < 7, levels[np.minimum(lo + 1, 7)] - levels[lo], 1.0)
    f16 = np.floor((a - levels[lo]) / span * 65536.0).astype(np.int64)  # exact: a is an fp32 value
    up = (lo < 7) & (f16 + np.asarray(r16, dtype=np.int64) >= 65536)
    code = (lo + up).astype(np.uint8)
    return (code | ((q < 0).astype(np.uint8) << 3)).astype(np.uint8)


def sr_uniform(r16: np.ndarray) -> np.ndarray:
    """The u in [0, 1) of the reference rule (up when u < f) that ``sr_nibbles`` matches exactly for
    every fraction f that is a multiple of 2^-16: u = (2^16 - 1 - r16) / 2^16."""
    return ((np.uint32(65535) - np.asarray(r16, dtype=np.uint32)).astype(np.float64) / 65536.0).astype(np.float32)


def pack_nibbles(code: np.ndarray) -> np.ndarray:
    """quantize.py:142-149 -- element 2i in the low nibble of byte i, 2i+1 in the high nibble."""
    return (code[..., 0::2] | (code[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """quantize.py:152-157."""
    low = packed & 0x0F
    high = packed >> 4
    return np.stack([low, high], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def _quantize_blocks(xb: np.ndarray, gs, axis: int, u: np.ndarray | None, r: np.ndarray | None = None):
    """Shared body of the two quantizers: amax over ``axis`` (the 16-wide block axis), the block
    scale, the IEEE divide by ``divisor * gs``, the +-6 clamp and the encode (``r``: the device's
    stochastic rounding with these random words, see ``sr_nibbles``)."""
    gs = _F32(gs)
    amax = np.abs(xb).max(axis=axis, keepdims=True)
    byte, divisor = block_scale(amax, gs)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        d = (divisor * gs).astype(np.float32)
        # The device's stochastic rounding takes q = RN(x * RN(1/d)), within 1.5 ulp of x / d: see
        # sr_nibbles.  Round-to-nearest uses the IEEE quotient, exactly as the reference.
        q = xb * (_F32(1.0) / d) if r is not None else xb / d
        q = np.clip(q, -FP4_MAX, FP4_MAX).astype(np.float32)
    code = sr_nibbles(q, r) if r is not None else encode_e2m1(np.abs(q), q < 0, u)
    return code, byte


def quantize_rowblock(x: np.ndarray, gs, u: np.ndarray | None = None, r: np.ndarray | None = None):
    """quantize.py:216-232 -- (M, K) -> packed (M, K/2) uint8, unswizzled scale bytes (M, K/16)."""
    m, k = x.shape
    xb = x.astype(np.float32).reshape(m, k // BLOCK, BLOCK)
    ub = None if u is None else u.reshape(m, k // BLOCK, BLOCK)
    rb = None if r is None else r.reshape(m, k // BLOCK, BLOCK)
    code, byte = _quantize_blocks(xb, gs, 2, ub, rb)
    return pack_nibbles(code.reshape(m, k)), byte.reshape(m, k // BLOCK)


def rotate_blocks(xb: np.ndarray, hadamard: np.ndarray) -> np.ndarray:
    """quantize.py:261-262 -- ``einsum("ij,bjk->bik", H.T, xb)`` in float32.

    torch's CPU einsum sums over ``j`` left to right with one rounding per add (checked against the
    reference on bf16 and fp32 inputs by ``tests/test_oracle_golden.py``), so this is the same
    sequential sum.  With the +-0.25 entries of a normalised Hadamard every product is exact.
    """
    ht = hadamard.astype(np.float32).T
    out = np.empty_like(xb)
    for i in range(BLOCK):
        acc = ht[i, 0] * xb[:, 0, :]
        for j in range(1, BLOCK):
            acc = (acc + ht[i, j] * xb[:, j, :]).astype(np.float32)
        out[:, i, :] = acc
    return out


def quantize_colblock(x: np.ndarray, gs, hadamard: np.ndarray | None = None, u: np.ndarray | None = None,
                      r: np.ndarray | None = None):
    """quantize.py:235-268 -- blocks along dim 0, output transposed.

    (M, K) -> packed (K, M/2) uint8, unswizzled scale bytes (K, M/16).  ``u`` (and ``r``) are
    indexed by the original (M, K) position, as in the reference.
    """
    m, k = x.shape
    xb = x.astype(np.float32).reshape(m // BLOCK, BLOCK, k)
    if hadamard is not None:
        xb = rotate_blocks(xb, hadamard)
    ub = None if u is None else u.reshape(m // BLOCK, BLOCK, k)
    rb = None if r is None else r.reshape(m // BLOCK, BLOCK, k)
    code, byte = _quantize_blocks(xb, gs, 1, ub, rb)
    code = code.reshape(m, k).T.copy()
    return pack_nibbles(code), byte.reshape(m // BLOCK, k).T.copy()


def to_blocked(scale: np.ndarray) -> np.ndarray:
    """quantize.py:271-290 -- (rows, cols) scale bytes -> flat SWIZZLE_32_4_4, zero-padded to whole
    128x4 tiles."""
    rows, cols = scale.shape
    nrt, nct = (rows + 127) // 128, (cols + 3) // 4
    padded = np.zeros((nrt * 128, nct * 4), dtype=scale.dtype)
    padded[:rows, :cols] = scale
    tiles = padded.reshape(nrt, 128, nct, 4).transpose(0, 2, 1, 3)
    return tiles.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3).reshape(-1).copy()


def from_blocked(flat: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of ``to_blocked`` (drops the padding)."""
    nrt, nct = (rows + 127) // 128, (cols + 3) // 4
    tiles = flat.reshape(nrt * nct, 32, 4, 4).transpose(0, 2, 1, 3).reshape(nrt, nct, 128, 4)
    return tiles.transpose(0, 2, 1, 3).reshape(nrt * 128, nct * 4)[:rows, :cols].copy()


def blocked_offset(r, c, n_col_tiles: int):
    """quantize.py:293-305 -- byte offset of scale element (r, c) in the SWIZZLE_32_4_4 layout."""
    return ((r // 128) * n_col_tiles + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def hadamard_signs_seed0() -> np.ndarray:
    """Row signs of the reference's ``hadamard_matrix(16, seed=0)`` (quantize.py:647-659), as the
    reference itself produces them (pinned by the golden fixture)."""
    return np.array([-1, 1, -1, -1, -1, 1, -1, 1, -1, 1, -1, -1, -1, -1, -1, 1], dtype=np.float32)


def sylvester(n: int = BLOCK) -> np.ndarray:
    h = np.ones((1, 1), dtype=np.float32)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h.astype(np.float32)


def hadamard_matrix(signs: np.ndarray | None = None) -> np.ndarray:
    """quantize.py:647-659 -- Sylvester Hadamard / sqrt(16) with row signs."""
    s = hadamard_signs_seed0() if signs is None else signs.astype(np.float32)
    return (sylvester(BLOCK) / np.float32(4.0) * s[:, None]).astype(np.float32)


def dequantize(packed: np.ndarray, scale: np.ndarray, gs) -> np.ndarray:
    """quantize.py:308-320 -- packed nibbles + unswizzled scale bytes -> fp32."""
    code = unpack_nibbles(packed)
    values = np.array(FP4_VALUES, dtype=np.float32)
    mag = values[code & 7]
    signed = np.where(code >= 8, -mag, mag).astype(np.float32)
    rows, cols = signed.shape
    blocks = signed.reshape(rows, cols // BLOCK, BLOCK)
    s = (E4M3_VALUES[scale].astype(np.float32) * _F32(gs)).astype(np.float32)
    return (blocks * s[..., None]).reshape(rows, cols).astype(np.float32)


def quantize_supported_shape(rows: int, cols: int) -> bool:
    """quantize.py:662-669."""
    return rows % 128 == 0 and cols % 64 == 0


def quantize(x: np.ndarray, axis: int, gs=None, hadamard=None, u=None, r=None):
    """quantize.py:412-433 (``quantize_reference``) -> (packed, swizzled flat scale, gs).  ``r``
    selects the device's stochastic rounding with those random words (``sr_stream_row`` or
    ``sr_stream_col``)."""
    if gs is None:
        gs = global_scale_of(x)
    if axis in (-1, x.ndim - 1):
        packed, scale = quantize_rowblock(x, gs, u=u, r=r)
    elif axis == 0:
        packed, scale = quantize_colblock(x, gs, hadamard=hadamard, u=u, r=r)
    else:
        raise ValueError(f"nvfp4.quantize supports axis 0 or -1, got {axis}")
    return packed, to_blocked(scale), _F32(gs)


def gemm_reference(a_packed, a_scale_flat, a_gs, b_packed, b_scale_flat, b_gs) -> np.ndarray:
    """The GEMM oracle: dequantize both operands (quantize.py:308-320, global scales included) and
    take ``a @ b.T`` in float64.  The reference's ``mm`` (quantize.py:400-409) computes the same
    product in the tensor cores and rounds to bf16 before multiplying the global scales back in."""
    ra, ka = a_packed.shape[0], a_packed.shape[1] * 2
    rb, kb = b_packed.shape[0], b_packed.shape[1] * 2
    assert ka == kb
    sa = from_blocked(a_scale_flat, ra, ka // BLOCK)
    sb = from_blocked(b_scale_flat, rb, kb // BLOCK)
    da = dequantize(a_packed, sa, a_gs).astype(np.float64)
    db = dequantize(b_packed, sb, b_gs).astype(np.float64)
    return da @ db.T


def linear_forward_reference(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """The reference's CPU emulation of one FP4 linear forward: global scales,
    rowblock quantize of both operands, dequantize, fp32 matmul.  Returns float32."""
    gx, gw = global_scale_of(x), global_scale_of(w)
    xp, xs = quantize_rowblock(x, gx)
    wp, ws = quantize_rowblock(w, gw)
    return (dequantize(xp, xs, gx) @ dequantize(wp, ws, gw).T).astype(np.float32)
