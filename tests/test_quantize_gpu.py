"""The CUDA quantizer against the oracle and the reference's golden vectors, bit-exactly.

Mirrors the reference's kernel tests (tests/test_nvfp4.py:277-395 in jamespa16/radiance): packed
codes and scale bytes at rtol=0, atol=0 across shapes, dtypes, forms (row, col, col+Hadamard),
magnitudes, zero blocks and outlier channels; stochastic rounding seeded, reproducible, within one
level of round-to-nearest and unbiased over 10^4 seeds.
"""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import dequantize_gpu, from_golden, to_numpy_f32, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported(), "needs an sm_100 GPU and the built library"
    return nv


def _status_ok():
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


# --- golden vectors produced by the reference itself ------------------------------------------


def test_global_scale_matches_golden(nv, golden):
    for name in [str(c) for c in golden["cases"]]:
        x = from_golden(golden, name)
        gs = nv.global_scale_of(x)
        assert np.float32(gs.item()).view(np.uint32) == golden[f"{name}/gs"].view(np.uint32), name


@pytest.mark.parametrize("tag", ["row", "col", "colh", "colh1"])
def test_quantize_matches_golden(nv, golden, tag):
    had = {"colh": golden["hadamard_seed0"], "colh1": golden["hadamard_seed1"]}.get(tag)
    for name in [str(c) for c in golden["cases"]]:
        x = from_golden(golden, name)
        gs = torch.tensor(golden[f"{name}/gs"], device="cuda")
        h = None if had is None else torch.from_numpy(had).cuda()
        q = nv.quantize(x, -1 if tag == "row" else 0, global_scale=gs, hadamard=h)
        np.testing.assert_array_equal(u8(q.packed), golden[f"{name}/{tag}_packed"], err_msg=f"{name} {tag} packed")
        np.testing.assert_array_equal(u8(q.scale), golden[f"{name}/{tag}_scale"], err_msg=f"{name} {tag} scale")
    _status_ok()


def test_fused_both_forms_match_golden(nv, golden):
    h = torch.from_numpy(golden["hadamard_seed0"]).cuda()
    for name in [str(c) for c in golden["cases"]]:
        x = from_golden(golden, name)
        gs = torch.tensor(golden[f"{name}/gs"], device="cuda")
        row, col = nv.quantize_both(x, global_scale=gs, hadamard=h)
        np.testing.assert_array_equal(u8(row.packed), golden[f"{name}/row_packed"], err_msg=name)
        np.testing.assert_array_equal(u8(row.scale), golden[f"{name}/row_scale"], err_msg=name)
        np.testing.assert_array_equal(u8(col.packed), golden[f"{name}/colh_packed"], err_msg=name)
        np.testing.assert_array_equal(u8(col.scale), golden[f"{name}/colh_scale"], err_msg=name)


# --- the oracle at larger sizes ------------------------------------------------------------------


def _check_vs_oracle(nv, x, axis, had=None, gs=None):
    xn = to_numpy_f32(x)
    gs_t = nv.global_scale_of(x) if gs is None else gs
    gs_np = np.float32(gs_t.item())
    if gs is None:
        assert gs_np.view(np.uint32) == O.global_scale_of(xn).view(np.uint32)
    q = nv.quantize(x, axis, global_scale=gs_t, hadamard=None if had is None else torch.from_numpy(had).cuda())
    p, s, _ = O.quantize(xn, axis, gs=gs_np, hadamard=had)
    np.testing.assert_array_equal(u8(q.packed), p)
    np.testing.assert_array_equal(u8(q.scale), s)


@pytest.mark.parametrize("shape", [(1024, 512), (256, 128), (4096, 1280), (128, 64), (512, 1408), (384, 192)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("axis,rotate", [(-1, False), (0, False), (0, True)])
def test_matches_oracle_bit_exactly(nv, shape, dtype, axis, rotate):
    torch.manual_seed(hash((shape, str(dtype), axis, rotate)) % 2**31)
    x = torch.randn(*shape, device="cuda", dtype=dtype)
    _check_vs_oracle(nv, x, axis, O.hadamard_matrix() if rotate else None)


@pytest.mark.parametrize("exponent", [-4, -2, 0, 2, 4])
def test_matches_oracle_across_magnitudes(nv, exponent):
    x = (torch.randn(1024, 512, device="cuda") * 10.0**exponent).bfloat16()
    for axis in (-1, 0):
        _check_vs_oracle(nv, x, axis)
    _check_vs_oracle(nv, x, 0, O.hadamard_matrix())


def test_general_rotation_matrix(nv):
    """A rotation that is not a signed Sylvester matrix takes the general multiply-then-add path."""
    g = torch.Generator().manual_seed(3)
    q, _ = torch.linalg.qr(torch.randn(16, 16, generator=g, dtype=torch.float64))
    had = q.float().numpy()
    x = torch.randn(512, 256, device="cuda").bfloat16()
    _check_vs_oracle(nv, x, 0, had)


def test_config2_activation_slice(nv):
    """BASELINE config 2's activation (8192 x 4096 bf16, 0.1% of channels x20): the kernel
    quantizes the full tensor; the first 1024 rows are checked against the oracle with the full
    tensor's global scale (both forms are local to 128-row tiles)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(8192, 4096, device="cuda", generator=g)
    ch = torch.randperm(4096, device="cuda", generator=g)[:4]
    x[:, ch] *= 20.0
    x = x.bfloat16()
    gs = nv.global_scale_of(x)
    assert np.float32(gs.item()).view(np.uint32) == O.global_scale_of(to_numpy_f32(x)).view(np.uint32)
    had = O.hadamard_matrix()
    row, col = nv.quantize_both(x, global_scale=gs, hadamard=torch.from_numpy(had).cuda())
    xs = to_numpy_f32(x[:1024])
    gsn = np.float32(gs.item())
    p, s = O.quantize_rowblock(xs, gsn)
    np.testing.assert_array_equal(u8(row.packed)[:1024], p)
    full_row_scale = O.from_blocked(u8(row.scale), 8192, 4096 // 16)
    np.testing.assert_array_equal(full_row_scale[:1024], s)
    p, s = O.quantize_colblock(xs, gsn, hadamard=had)
    np.testing.assert_array_equal(u8(col.packed)[:, :512], p)
    full_col_scale = O.from_blocked(u8(col.scale), 4096, 8192 // 16)
    np.testing.assert_array_equal(full_col_scale[:, :64], s)
    _status_ok()


def test_both_forms_equal_separate_calls_at_full_size(nv):
    """Size-independent property at BASELINE config 3's largest activation gradient
    (16384 x 11264): the fused pass equals the two single-form passes byte for byte."""
    x = torch.randn(16384, 11264, device="cuda").bfloat16() * 1e-3
    gs = nv.global_scale_of(x)
    h = nv.hadamard_matrix(device="cuda")
    row, col = nv.quantize_both(x, global_scale=gs, hadamard=h)
    r1 = nv.quantize(x, -1, global_scale=gs)
    c1 = nv.quantize(x, 0, global_scale=gs, hadamard=h)
    assert torch.equal(row.packed.view(torch.uint8), r1.packed.view(torch.uint8))
    assert torch.equal(row.scale.view(torch.uint8), r1.scale.view(torch.uint8))
    assert torch.equal(col.packed.view(torch.uint8), c1.packed.view(torch.uint8))
    assert torch.equal(col.scale.view(torch.uint8), c1.scale.view(torch.uint8))
    # Round trip: dequantized values stay within half a grid step of |x| / D <= 6.
    deq = dequantize_gpu(row.packed[:256], row.scale, gs, 256, 11264)
    err = (deq - x[:256].float()).abs()
    blk = x[:256].float().abs().view(256, -1, 16).amax(-1, keepdim=True)
    assert (err.view(256, -1, 16) <= blk * (1.0 / 3.0) + 1e-30).all()


# --- properties the reference tests pin ------------------------------------------------------------


def test_codes_never_exceed_six(nv):
    x = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16)
    gs = nv.global_scale_of(x)
    q = nv.quantize(x, -1, global_scale=gs)
    deq = dequantize_gpu(q.packed, q.scale, gs, 1024, 512)
    s = O.from_blocked(u8(q.scale), 1024, 32).astype(np.int64)
    scale = torch.from_numpy(O.E4M3_VALUES[s]).cuda() * gs
    assert (deq.view(1024, 32, 16).abs() <= 6.0 * scale.unsqueeze(-1) * (1 + 1e-6)).all()
    # ...and the rounded-up scale covers every block's amax (tests/test_nvfp4.py:314-324).
    amax = x.float().abs().view(1024, 32, 16).amax(-1)
    assert (scale * 6.0 >= amax - 1e-6).all()


def test_zero_blocks(nv):
    x = torch.randn(256, 128, device="cuda", dtype=torch.bfloat16)
    x[:, :16] = 0.0
    for axis in (-1, 0):
        _check_vs_oracle(nv, x, axis)
    zeros = torch.zeros(256, 128, device="cuda", dtype=torch.bfloat16)
    gz = nv.global_scale_of(zeros)
    assert gz.item() == np.float32(1e-12)
    q = nv.quantize(zeros, -1, global_scale=gz)
    assert u8(q.packed).max() == 0


def test_ragged_shapes_raise(nv):
    assert nv.quantize_supported_shape(4096, 1280)
    assert not nv.quantize_supported_shape(100, 1280)
    assert not nv.quantize_supported_shape(4096, 100)
    with pytest.raises(ValueError, match="rows % 128"):
        nv.quantize(torch.randn(100, 128, device="cuda"), -1)
    with pytest.raises(ValueError, match="axis 0 or -1"):
        nv.quantize(torch.randn(128, 128, device="cuda"), 2)


def test_non_contiguous_and_strided_inputs(nv):
    base = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    x = base[:, 256:768]  # row stride 1024, 512 columns
    for axis in (-1, 0):
        got = nv.quantize(x, axis)
        ref = nv.quantize(x.contiguous(), axis)
        assert torch.equal(got.packed.view(torch.uint8), ref.packed.view(torch.uint8))
        assert torch.equal(got.scale.view(torch.uint8), ref.scale.view(torch.uint8))
    assert nv.global_scale_of(x).item() == nv.global_scale_of(x.contiguous()).item()


def test_global_scale_shapes_and_workspace_reuse(nv):
    for shape in [(1, 7), (3, 1000), (128, 64), (4096, 4096), (777, 333)]:
        for dtype in (torch.bfloat16, torch.float32):
            x = torch.randn(*shape, device="cuda", dtype=dtype) * 3
            want = O.global_scale_of(to_numpy_f32(x))
            for _ in range(2):  # the workspace must come back zeroed
                assert np.float32(nv.global_scale_of(x).item()).view(np.uint32) == want.view(np.uint32)


def test_global_scale_of_column_slices(nv):
    """Row-strided inputs (an N-split layer's slice of the gradient): 16-byte aligned rows take the
    vectorised strided path, others the element path; both equal the oracle bit for bit."""
    for dtype in (torch.bfloat16, torch.float32):
        base = torch.randn(300, 1536, device="cuda", dtype=dtype)
        base[17, 700] = 55.0  # the maximum sits inside the slice
        for sl in (slice(512, 1024), slice(8, 1032), slice(3, 1000)):
            x = base[:, sl]
            want = O.global_scale_of(to_numpy_f32(x))
            assert np.float32(nv.global_scale_of(x).item()).view(np.uint32) == want.view(np.uint32), (dtype, sl)


# --- stochastic rounding ----------------------------------------------------------------------------


def test_stochastic_rounding_is_seeded_and_reproducible(nv):
    x = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    gs = nv.global_scale_of(x)
    seed = torch.tensor(0, device="cuda", dtype=torch.int64)
    a = nv.quantize(x, -1, global_scale=gs, stochastic=True, seed=seed)
    b = nv.quantize(x, -1, global_scale=gs, stochastic=True, seed=seed)
    assert torch.equal(a.packed.view(torch.uint8), b.packed.view(torch.uint8))
    seed.fill_(1)
    c = nv.quantize(x, -1, global_scale=gs, stochastic=True, seed=seed)
    assert not torch.equal(a.packed.view(torch.uint8), c.packed.view(torch.uint8))
    seed.fill_(0)
    again = nv.quantize(x, -1, global_scale=gs, stochastic=True, seed=seed)
    assert torch.equal(a.packed.view(torch.uint8), again.packed.view(torch.uint8))
    # Scale bytes do not depend on the rounding mode.
    rn = nv.quantize(x, -1, global_scale=gs)
    assert torch.equal(a.scale.view(torch.uint8), rn.scale.view(torch.uint8))
    delta = (nv.unpack_nibbles(a.packed).int() & 7) - (nv.unpack_nibbles(rn.packed).int() & 7)
    assert delta.abs().max().item() <= 1
    assert delta.abs().sum().item() > 0


@pytest.mark.parametrize("form", ["row", "colh"])
def test_stochastic_rounding_unbiased_over_many_seeds(nv, form):
    """E[SR(q)] = q: over 10^4 seeds the mean dequantized value converges on the exact scaled
    value, while round-to-nearest keeps its bias (reference test :132-152, at 50x the draws)."""
    torch.manual_seed(5)
    rows, cols = 128, 128
    x = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
    gs = nv.global_scale_of(x)
    h = nv.hadamard_matrix(device="cuda") if form == "colh" else None
    axis = -1 if form == "row" else 0
    # Target: the exact (rotated) values the codes represent.
    xn = to_numpy_f32(x)
    target = xn if form == "row" else O.rotate_blocks(xn.reshape(rows // 16, 16, cols), O.hadamard_matrix()).reshape(rows, cols).T
    target = torch.from_numpy(np.ascontiguousarray(target)).cuda()
    r, c = target.shape
    seed = torch.zeros((), dtype=torch.int64, device="cuda")
    acc = torch.zeros(r, c, device="cuda", dtype=torch.float64)
    draws = 10_000
    for i in range(draws):
        seed.fill_(i)
        q = nv.quantize(x, axis, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
        acc += dequantize_gpu(q.packed, q.scale, gs, r, c).double()
    mean = acc / draws
    rn = nv.quantize(x, axis, global_scale=gs, hadamard=h)
    rn_deq = dequantize_gpu(rn.packed, rn.scale, gs, r, c).double()
    t = target.double()
    # Per-element grid step D * (0.5, 1 or 2); the SR std per draw is at most half a step.
    s = torch.from_numpy(O.E4M3_VALUES[O.from_blocked(u8(q.scale), r, c // 16)].astype(np.float64)).cuda()
    step = (s * gs.double()).repeat_interleave(16, dim=1) * 2.0
    z = (mean - t) / (step / 2 / draws**0.5)
    assert z.abs().mean().item() < 1.2  # ~0.8 for an unbiased estimator
    assert abs((mean - t).mean().item()) < 0.1 * abs((rn_deq - t).abs().mean().item())
    assert ((mean - t).norm() / t.norm()).item() < 0.25 * ((rn_deq - t).norm() / t.norm()).item()


@pytest.mark.parametrize("shape", [(256, 512), (384, 320), (1024, 1408)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("form", ["row", "col", "colh"])
def test_stochastic_rounding_matches_oracle_stream(nv, shape, dtype, form):
    """Bit-exact against the oracle's restatement of the device streams and rounding
    (``sr_stream_row`` / ``sr_stream_col`` / ``sr_nibbles``), both forms, fused and separate."""
    torch.manual_seed(hash((shape, str(dtype), form)) % 2**31)
    x = torch.randn(*shape, device="cuda", dtype=dtype) * 0.3
    gs = nv.global_scale_of(x)
    gs_np = np.float32(gs.item())
    seed_value = 0x1234_5678_9ABC + len(form)
    seed = torch.tensor(seed_value, device="cuda", dtype=torch.int64)
    had = O.hadamard_matrix() if form == "colh" else None
    h = None if had is None else torch.from_numpy(had).cuda()
    axis = -1 if form == "row" else 0
    r = (O.sr_stream_row if form == "row" else O.sr_stream_col)(*shape, seed_value)
    p, s, _ = O.quantize(to_numpy_f32(x), axis, gs=gs_np, hadamard=had, r=r)
    q = nv.quantize(x, axis, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
    np.testing.assert_array_equal(u8(q.packed), p)
    np.testing.assert_array_equal(u8(q.scale), s)
    if form != "row":
        row, col = nv.quantize_both(x, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
        np.testing.assert_array_equal(u8(col.packed), p)
        pr, sr_, _ = O.quantize(to_numpy_f32(x), -1, gs=gs_np, r=O.sr_stream_row(*shape, seed_value))
        np.testing.assert_array_equal(u8(row.packed), pr)
    _status_ok()


def test_stochastic_both_forms(nv):
    x = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16) * 1e-3
    gs = nv.global_scale_of(x)
    h = nv.hadamard_matrix(device="cuda")
    seed = torch.tensor(7, device="cuda", dtype=torch.int64)
    row, col = nv.quantize_both(x, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
    r1 = nv.quantize(x, -1, global_scale=gs, stochastic=True, seed=seed)
    c1 = nv.quantize(x, 0, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
    assert torch.equal(row.packed.view(torch.uint8), r1.packed.view(torch.uint8))
    assert torch.equal(col.packed.view(torch.uint8), c1.packed.view(torch.uint8))
    _status_ok()


# --- the division identity ------------------------------------------------------------------------


def test_division_matches_ieee(nv):
    """Every positive finite bf16 numerator (as fp32) against divisors e4m3 * gs for a spread of
    global scales, plus random fp32 numerators: the reciprocal-plus-two-corrections quotient equals
    the IEEE quotient bit for bit for 2^-64 <= |q| < 2^64.  (Codes are decided by |q| in
    [0.25, 6]; below ~1e-21 the residual x - q*d underflows and the quotient may differ in its last
    bits, which changes no code: such quotients encode as zero, and the sign of an underflowed zero
    is fixed exactly by the kernel's underflow mask.)"""
    from radiance_b200 import _lib

    lib = _lib.load()
    bits = torch.arange(0x0080, 0x7F80, dtype=torch.int32)  # normal bf16 magnitudes
    num = (bits << 16).view(torch.float32)
    e4 = torch.from_numpy(O.E4M3_VALUES[1:127].astype(np.float32))
    g = torch.Generator().manual_seed(1)
    gss = torch.cat([torch.tensor([1e-12, 1.0, 2.0**-20, 3.7e-5, 0.11]), torch.rand(27, generator=g) * 10.0 ** torch.randint(-12, 6, (27,), generator=g)])
    d = (e4.view(1, -1) * gss.view(-1, 1)).reshape(-1)  # fp32 products, as the kernel forms D
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    for chunk in torch.split(d, 64):
        xx = num.view(1, -1).expand(chunk.numel(), -1).reshape(-1)
        dd = chunk.view(-1, 1).expand(-1, num.numel()).reshape(-1)
        q = xx / dd
        keep = (q.abs() >= 2.0**-64) & (q.abs() < 2.0**64) & (xx.abs() >= 2.0**-90)
        xx, dd = xx[keep].cuda(), dd[keep].cuda()
        _lib.check(lib.rb_nvfp4_selftest_division(xx.data_ptr(), dd.data_ptr(), xx.numel(), mism.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream), "selftest")
    xx = (torch.rand(1 << 22, generator=g) * 12 - 6).cuda()
    dd = (torch.rand(1 << 22, generator=g) * 100 + 1e-3).cuda()
    _lib.check(lib.rb_nvfp4_selftest_division(xx.data_ptr(), dd.data_ptr(), xx.numel(), mism.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream), "selftest")
    assert mism.item() == 0


def test_scale_byte_shortcut_matches_exact(nv):
    """The quantizer's block-scale byte (hardware e4m3 rounding of amax / (6 gs) plus one threshold
    compare) equals the exact evaluation (correctly rounded quotient, clamp, round up to e4m3) for
    every amax near every threshold, for every bf16 magnitude, and for random fp32 amaxes, over a
    spread of global scales."""
    from radiance_b200 import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(3)
    gss = torch.cat([torch.tensor([1e-12, 1.0, 2.0**-20, 3.7e-5, 0.11, 1.5e30]),
                     torch.rand(26, generator=g) * 10.0 ** torch.randint(-12, 8, (26,), generator=g)])
    bf16 = (torch.arange(0, 0x7F81, dtype=torch.int32) << 16).view(torch.float32)  # 0, every bf16, +inf
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for gsv in gss.tolist():
        gs = torch.tensor([gsv], dtype=torch.float32, device="cuda")
        den = np.float32(6.0) * np.float32(gsv)
        # amaxes around value(b) * den for every e4m3 byte b, +-64 ulps
        centers = (O.E4M3_VALUES[:127].astype(np.float32) * den).astype(np.float32).view(np.int32)
        near = (centers[:, None] + np.arange(-64, 65, dtype=np.int32)[None, :]).reshape(-1)
        near = near[(near >= 0) & (near < 0x7F800000)].view(np.float32)
        rnd = (torch.rand(1 << 16, generator=g) * 10.0 ** torch.randint(-40, 38, (1 << 16,), generator=g)).float()
        amax = torch.cat([torch.from_numpy(near.copy()), bf16, rnd]).cuda()
        _lib.check(lib.rb_nvfp4_selftest_scale(amax.data_ptr(), amax.numel(), gs.data_ptr(), mism.data_ptr(), stream),
                   "selftest_scale")
    assert mism.item() == 0


def test_stochastic_rounding_wide_range_matches_oracle(nv):
    """Stochastic rounding against the oracle on inputs spanning 2^-30 .. 2^4 inside each block, so
    that most quotients fall below the first e2m1 level (the convert's subnormal range) and some
    underflow entirely; both forms, fused."""
    torch.manual_seed(11)
    rows, cols = 512, 384
    mag = torch.exp2(torch.rand(rows, cols) * 34.0 - 30.0)
    x = (torch.randn(rows, cols).sign() * mag).to(torch.bfloat16).cuda()
    gs = nv.global_scale_of(x)
    gs_np = np.float32(gs.item())
    seed_value = 99
    seed = torch.tensor(seed_value, device="cuda", dtype=torch.int64)
    had = O.hadamard_matrix()
    h = torch.from_numpy(had).cuda()
    row, col = nv.quantize_both(x, global_scale=gs, hadamard=h, stochastic=True, seed=seed)
    xn = to_numpy_f32(x)
    pr, sr_, _ = O.quantize(xn, -1, gs=gs_np, r=O.sr_stream_row(rows, cols, seed_value))
    pc, sc, _ = O.quantize(xn, 0, gs=gs_np, hadamard=had, r=O.sr_stream_col(rows, cols, seed_value))
    np.testing.assert_array_equal(u8(row.packed), pr)
    np.testing.assert_array_equal(u8(row.scale), sr_)
    np.testing.assert_array_equal(u8(col.packed), pc)
    np.testing.assert_array_equal(u8(col.scale), sc)
    _status_ok()


def test_negative_zeros_stochastic(nv):
    """-0 inputs inside ordinary blocks give nibble 0 under stochastic rounding too (the
    round-to-nearest forms are pinned by the golden case ``negzero``)."""
    torch.manual_seed(12)
    x = torch.randn(256, 384)
    x[0::3, 2::5] = -0.0
    x[16:32, 40:56] = -0.0
    x = x.bfloat16().cuda()
    gs = nv.global_scale_of(x)
    gs_np = np.float32(gs.item())
    seed = torch.tensor(5, device="cuda", dtype=torch.int64)
    had = O.hadamard_matrix()
    row, col = nv.quantize_both(x, global_scale=gs, hadamard=torch.from_numpy(had).cuda(), stochastic=True, seed=seed)
    xn = to_numpy_f32(x)
    pr, _, _ = O.quantize(xn, -1, gs=gs_np, r=O.sr_stream_row(256, 384, 5))
    pc, _, _ = O.quantize(xn, 0, gs=gs_np, hadamard=had, r=O.sr_stream_col(256, 384, 5))
    np.testing.assert_array_equal(u8(row.packed), pr)
    np.testing.assert_array_equal(u8(col.packed), pc)
    _status_ok()
