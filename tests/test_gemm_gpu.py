"""The tcgen05 block-scaled GEMM against the oracle (dequantized operands, float64 matmul).

fp32 output within max relative error 1e-3 (``max|got - ref| / max|ref|``);
bf16 output additionally within one bf16 ulp of the exact value.  Plus the reference's own GEMM
tests (tests/test_nvfp4.py:173-258 in jamespa16/radiance): rel-err < 0.2 against the unquantized
product and *not* equal to a bf16 matmul, all three orientations, the Hadamard identity with its
negative control, and the custom op's fake kernel.
"""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import u8

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3  # written in the north star; the kernel is ~1e-6 in practice


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _rel_err(got, ref):
    return ((got.float() - ref.float()).norm() / ref.float().norm()).item()


def _oracle(a, b, with_gs=True, rows=None):
    """float64 product of the dequantized operands (optionally only `rows` of A)."""
    ap, asc = u8(a.packed), u8(a.scale)
    bp, bsc = u8(b.packed), u8(b.scale)
    ga = np.float32(a.global_scale.item()) if with_gs else np.float32(1.0)
    gb = np.float32(b.global_scale.item()) if with_gs else np.float32(1.0)
    ka = ap.shape[1] * 2
    sa = O.from_blocked(asc, ap.shape[0], ka // 16)
    sb = O.from_blocked(bsc, bp.shape[0], ka // 16)
    if rows is not None:
        ap, sa = ap[rows], sa[rows]
    da = O.dequantize(ap, sa, ga).astype(np.float64)
    db = O.dequantize(bp, sb, gb).astype(np.float64)
    return da @ db.T


def _check_close(got: torch.Tensor, ref: np.ndarray, bf16: bool):
    g = got.double().cpu().numpy()
    scale = np.abs(ref).max()
    err = np.abs(g - ref).max() / max(scale, 1e-300)
    if bf16:
        # bf16's unit roundoff (2^-8) is above 1e-3, so a bf16 output is held to the rounding of
        # the exact value instead: within one bf16 ulp (plus fp32-accumulation noise on sums
        # that cancel).
        assert (np.abs(g - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * scale).all(), f"max rel err {err}"
    else:
        assert err <= REL_TOL, f"max rel err {err}"
        assert err < 1e-5, f"fp32 output error {err} is larger than accumulation noise"


SHAPES = [(128, 128, 64), (128, 256, 256), (256, 256, 256), (128, 384, 320), (512, 640, 1088), (384, 128, 192),
          (1024, 2048, 2048), (256, 1280, 5632)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_matches_oracle(nv, m, n, k, out_dtype):
    torch.manual_seed(m * 7 + n * 3 + k)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    got = nv.mm(a, b, out_dtype=out_dtype)
    assert got.shape == (m, n) and got.dtype == out_dtype
    _check_close(got, _oracle(a, b), out_dtype == torch.bfloat16)
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


def test_nvfp4_mm_has_no_global_scales(nv):
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16) * 3
    w = torch.randn(384, 512, device="cuda", dtype=torch.bfloat16)
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    got = nv.nvfp4_mm(a.packed, a.scale, b.packed, b.scale)
    assert got.dtype == torch.bfloat16
    _check_close(got, _oracle(a, b, with_gs=False), True)


@pytest.mark.parametrize("bias_dtype", [torch.bfloat16, torch.float32])
def test_bias_is_fused(nv, bias_dtype):
    x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(512, device="cuda").to(bias_dtype)
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    got = nv.mm(a, b, out_dtype=torch.float32, bias=bias)
    ref = _oracle(a, b) + bias.double().cpu().numpy()[None, :]
    _check_close(got, ref, False)


def test_three_orientations_at_config_scale(nv):
    """Forward, dgrad and wgrad operands (tests/test_nvfp4.py:196-213): the canonical
    rows x contraction layout holds for all three, including the colblock forms."""
    m, k, n = 4096, 1280, 3840
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
    gy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    y = nv.mm(nv.quantize(x, -1), nv.quantize(w, -1))
    assert y.shape == (m, n) and _rel_err(y, x.float() @ w.float().t()) < 0.2
    assert not torch.allclose(y.float(), (x @ w.t()).float(), rtol=1e-3, atol=1e-3)
    gq, wq = nv.quantize(gy, -1), nv.quantize(w, 0)
    dx = nv.mm(gq, wq)
    assert dx.shape == (m, k) and _rel_err(dx, gy.float() @ w.float()) < 0.2
    _check_close(dx[:128], _oracle(gq, wq, rows=slice(0, 128)), True)
    gqt, xqt = nv.quantize(gy, 0), nv.quantize(x, 0)
    dw = nv.mm(gqt, xqt, out_dtype=torch.float32)
    assert dw.shape == (n, k) and _rel_err(dw, gy.float().t() @ x.float()) < 0.2
    _check_close(dw[-256:], _oracle(gqt, xqt, rows=slice(n - 256, n)), False)


def test_wgrad_hadamard_matched_and_mismatched(nv):
    """(R^T dY)^T (R^T X) = dY^T X needs the same R on both operands; the negative control
    (different sign vectors) must diverge (tests/test_nvfp4.py:216-243)."""
    m, k, n = 2048, 512, 1024
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    gy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    ref = gy.float().t() @ x.float()
    r = nv.hadamard_matrix(device="cuda")
    torch.testing.assert_close(r @ r.t(), torch.eye(16, device="cuda"), rtol=1e-4, atol=1e-4)
    matched = nv.mm(nv.quantize(gy, 0, hadamard=r), nv.quantize(x, 0, hadamard=r))
    assert _rel_err(matched, ref) < 0.2
    other = nv.hadamard_matrix(device="cuda", seed=1)
    mismatched = nv.mm(nv.quantize(gy, 0, hadamard=r), nv.quantize(x, 0, hadamard=other))
    assert _rel_err(mismatched, ref) > 1.0


def test_config2_forward_slices(nv):
    """BASELINE config 2 at full size (M=8192, K=N=4096, outlier channels): the kernel computes
    the whole product; three 128-row tiles are checked against the oracle."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(8192, 4096, device="cuda", generator=g)
    x[:, torch.randperm(4096, device="cuda", generator=g)[:4]] *= 20.0
    x = x.bfloat16()
    w = (torch.randn(4096, 4096, device="cuda", generator=g) / 64.0).bfloat16()
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    y = nv.mm(a, b, out_dtype=torch.float32)
    for r0 in (0, 4096, 8192 - 128):
        _check_close(y[r0:r0 + 128], _oracle(a, b, rows=slice(r0, r0 + 128)), False)


def test_zero_operands(nv):
    zeros = torch.zeros(256, 128, device="cuda", dtype=torch.bfloat16)
    q = nv.quantize(zeros, -1)
    out = nv.mm(q, q)
    assert torch.isfinite(out).all() and out.abs().max().item() == 0.0


def test_shape_contract(nv):
    a = nv.quantize(torch.randn(128, 128, device="cuda"), -1)
    with pytest.raises(ValueError, match="contraction mismatch"):
        nv.mm(a, nv.quantize(torch.randn(128, 256, device="cuda"), -1))


def test_custom_op_fake_kernel(nv):
    x = torch.randn(256, 128, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, 128, device="cuda", dtype=torch.bfloat16)
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    with torch._subclasses.FakeTensorMode(allow_non_fake_inputs=True):
        fake = nv.nvfp4_mm(a.packed, a.scale, b.packed, b.scale)
    assert fake.shape == (256, 512) and fake.dtype == torch.bfloat16
