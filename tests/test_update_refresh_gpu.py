"""The optimizer step fused with the weight-cache refresh: ``rb_nvfp4_update_global_scale`` /
``nvfp4.update_and_global_scale_`` / ``FP4Linear.apply_update_and_refresh_``.

radiance's Muon step ends with ``target.add_(orthogonalize(u), alpha=-lr*scale)``
(src/radiance/optim.py:518), after which ``refresh_fp4_weights`` re-quantizes each FP4 weight,
first reading it for its global scale (src/radiance/nvfp4/linear.py:193-210).
- The fused kernel applies the update as one fp32 fused multiply-add per element and computes the
  global scale in the same pass. The update is checked against the exactly rounded result and
  against torch's own ``add_`` (bit for bit); the global scale must equal ``global_scale_of`` of the
  updated weight bit for bit.
- The refreshed cache must equal ``refresh_fp4_cache()``'s on that weight, bit for bit.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _status_ok():
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


def _ulps(got: torch.Tensor, ref: torch.Tensor) -> np.ndarray:
    """Distance in units in the last place, by bit pattern (finite values of one sign class)."""
    if got.dtype == torch.bfloat16:
        g = got.view(torch.int16).cpu().numpy().astype(np.int64)
        r = ref.view(torch.int16).cpu().numpy().astype(np.int64)
        to_ord = lambda b: np.where(b < 0, -(b & 0x7FFF), b)  # noqa: E731
    else:
        g = got.view(torch.int32).cpu().numpy().astype(np.int64)
        r = ref.view(torch.int32).cpu().numpy().astype(np.int64)
        to_ord = lambda b: np.where(b < 0, -(b & 0x7FFFFFFF), b)  # noqa: E731
    return np.abs(to_ord(g) - to_ord(r))


@pytest.mark.parametrize("w_dtype,u_dtype", [(torch.float32, torch.bfloat16), (torch.float32, torch.float32),
                                             (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("shape", [(2048, 1024), (333, 7)])
def test_update_and_global_scale(nv, w_dtype, u_dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(shape[0] + shape[1])
    w0 = (torch.randn(*shape, device="cuda", generator=g) * 0.02).to(w_dtype)
    u = torch.randn(*shape, device="cuda", generator=g).to(u_dtype)
    alpha = -0.0123
    # The exactly rounded w + alpha * u (float64 holds alpha * u exactly; the sum's own rounding in
    # float64 can differ from the exact one only in rare double-rounding cases, hence the 1-ulp bound).
    exact = (w0.double() + torch.tensor(alpha, dtype=torch.float32).double() * u.double()).to(w_dtype)
    w = w0.clone()
    gs = nv.update_and_global_scale_(w, u, alpha)
    d = _ulps(w, exact)
    assert d.max() <= 1 and (d == 0).mean() > 0.999
    assert gs.view(torch.int32).item() == nv.global_scale_of(w).view(torch.int32).item()
    # The reference's own update, target.add_(u, alpha=...), gives the same bits.
    torch_w = w0.clone().add_(u, alpha=alpha)
    ibits = torch.int16 if w_dtype == torch.bfloat16 else torch.int32
    assert torch.equal(w.view(ibits), torch_w.view(ibits))
    _status_ok()


def test_update_of_an_empty_weight(nv):
    w = torch.empty(0, 64, device="cuda")
    gs = nv.update_and_global_scale_(w, torch.empty(0, 64, device="cuda"), 0.5)
    assert gs.item() == np.float32(1e-12)
    _status_ok()


def test_apply_update_and_refresh_matches_plain_refresh(nv):
    """The fused path leaves the same cache (both layouts, scales, global scale) as updating the
    weight and calling refresh_fp4_cache(), and the same weight as the update kernel alone."""
    torch.manual_seed(9)
    lin = nv.FP4Linear(1024, 768, device="cuda")
    ref = nv.FP4Linear(1024, 768, device="cuda")
    with torch.no_grad():
        ref.weight.copy_(lin.weight)
    u = torch.randn(768, 1024, device="cuda").bfloat16()
    w_expected = lin.weight.detach().clone()
    nv.update_and_global_scale_(w_expected, u, -3e-3)
    lin.apply_update_and_refresh_(u, -3e-3)
    assert torch.equal(lin.weight.detach(), w_expected)
    with torch.no_grad():
        ref.weight.copy_(w_expected)
    ref.refresh_fp4_cache()
    for name in ("_w_fwd_packed", "_w_fwd_scale", "_w_fwd_gs", "_w_dgrad_packed", "_w_dgrad_scale", "_w_dgrad_gs"):
        a, b = getattr(lin, name), getattr(ref, name)
        assert torch.equal(a.view(torch.uint8) if a.dim() else a, b.view(torch.uint8) if b.dim() else b), name
    assert lin._cache_valid
    _status_ok()
