"""The GEMMs of the benchmarked workloads at their full sizes, checked against the oracle on slices.

The kernels compute the whole product; the oracle (dequantized operands, float64 matmul) checks
128-row slices at the start, middle and end of the output -- for the contraction-16384 wgrads that
is every one of the 64 K steps of the longest pipelines.  Tolerance as in ``test_gemm_gpu``: fp32
output within max relative error 1e-3 (the north star's bound) and below fp32 accumulation noise
(1e-5); bf16 output within one bf16 ulp.  Shapes: BASELINE config 3's gate/up forward
(16384 x 11264 x 2048) and its QKV and gate/up wgrads over 16384 tokens, config 5's gate/up forward
(65536 x 28672 x 4096), and config 4's grouped expert linears on its real top-2 routing counts.
"""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import to_numpy_f32, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _deq(t, rows=None):
    """Dequantize an NVFP4Tensor (optionally only `rows`) to float64."""
    p, s = u8(t.packed), u8(t.scale)
    k = p.shape[1] * 2
    sc = O.from_blocked(s, p.shape[0], k // 16)
    if rows is not None:
        p, sc = p[rows], sc[rows]
    return O.dequantize(p, sc, np.float32(t.global_scale.item())).astype(np.float64)


def _check(got: torch.Tensor, ref: np.ndarray, bf16: bool):
    g = got.double().cpu().numpy()
    scale = np.abs(ref).max()
    if bf16:
        assert (np.abs(g - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * scale).all()
    else:
        err = np.abs(g - ref).max() / scale
        assert err <= 1e-3 and err < 1e-5, f"max rel err {err}"


def _status_ok():
    from radiance_b200 import _lib

    assert _lib.device_status() == 0


def test_config3_gate_up_forward_full_size(nv):
    m, k, n = 16384, 2048, 11264
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    y32 = nv.mm(a, b, out_dtype=torch.float32)
    y16 = nv.mm(a, b, out_dtype=torch.bfloat16)
    db = _deq(b)
    for r0 in (0, m // 2, m - 128):
        ref = _deq(a, slice(r0, r0 + 128)) @ db.T
        _check(y32[r0:r0 + 128], ref, False)
        _check(y16[r0:r0 + 128], ref, True)
    _status_ok()


@pytest.mark.parametrize("n", [6144, 11264])
def test_config3_wgrad_over_16384_tokens(nv, n):
    """dW = dY^T X with both operands in the rotated colblock form over all 16384 tokens (64 K
    steps), dY stochastically rounded as the layer's backward does."""
    m, k = 16384, 2048
    g = torch.Generator(device="cuda").manual_seed(12 + n)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    dy = (torch.randn(m, n, device="cuda", generator=g) * 1e-3).bfloat16()
    r = nv.hadamard_matrix(device="cuda")
    gqt = nv.quantize(dy, 0, hadamard=r, stochastic=True, seed=5)
    xqt = nv.quantize(x, 0, hadamard=r)
    dw = nv.mm(gqt, xqt, out_dtype=torch.float32)
    assert dw.shape == (n, k)
    dx = _deq(xqt)
    for r0 in (0, n // 2, n - 128):
        _check(dw[r0:r0 + 128], _deq(gqt, slice(r0, r0 + 128)) @ dx.T, False)
    _status_ok()


def test_config5_gate_up_forward_full_size(nv):
    """65536 x 28672 x 4096 (config 5's largest GEMM, 15.4 TFLOP), bf16 output; slices of rows and
    columns at both ends and the middle."""
    m, k, n = 65536, 4096, 28672
    g = torch.Generator(device="cuda").manual_seed(13)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    del x, w
    y = nv.mm(a, b, out_dtype=torch.bfloat16)
    for c0 in (0, n // 2, n - 256):
        db = _deq(b, slice(c0, c0 + 256))
        for r0 in (0, m // 2 + 128, m - 128):
            _check(y[r0:r0 + 128, c0:c0 + 256], _deq(a, slice(r0, r0 + 128)) @ db.T, True)
    _status_ok()


def _config4_counts(seed: int = 0, tokens: int = 16384, experts: int = 8, top_k: int = 2) -> torch.Tensor:
    """BASELINE config 4's routing: router logits ~N(0,1) (seeded), softmax, top-2 -> rows per expert."""
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(tokens, experts, generator=gen)
    top = logits.softmax(-1).topk(top_k, dim=-1).indices
    return torch.bincount(top.flatten(), minlength=experts)


def test_config4_grouped_linear_on_real_routing_counts():
    """FP4GroupedLinear at config 4's gate+up shape (8 experts, 2048 -> 2816) on the uneven group
    sizes of its top-2 routing (32768 routed rows, padded to 128 per group): forward, dgrad and
    wgrad, per expert against the single-linear oracle on 128-row slices."""
    import radiance_b200.nvfp4.grouped as grp
    from radiance_b200.nvfp4 import FP4Recipe

    e, k, n = 8, 2048, 2816
    counts = _config4_counts()
    assert int(counts.sum()) == 32768 and len(set(counts.tolist())) > 1
    offs = grp.align_offsets(counts.cuda())
    o = offs.tolist()
    t = o[-1]
    lin = grp.FP4GroupedLinear(e, k, n, recipe=FP4Recipe(stochastic_rounding=False), device="cuda")
    lin.refresh_fp4_cache()
    gen = torch.Generator(device="cuda").manual_seed(14)
    x = torch.zeros(t, k, device="cuda", dtype=torch.bfloat16)
    dy = torch.zeros(t, n, device="cuda", dtype=torch.bfloat16)
    for gi in range(e):  # real rows, then zero padding up to the group's 128-row boundary
        c = int(counts[gi])
        x[o[gi]:o[gi] + c] = torch.randn(c, k, device="cuda", generator=gen).bfloat16()
        dy[o[gi]:o[gi] + c] = (torch.randn(c, n, device="cuda", generator=gen) * 1e-3).bfloat16()
    x.requires_grad_(True)
    y = lin(x, offs)
    y.backward(dy)
    xn, dyn = to_numpy_f32(x), to_numpy_f32(dy)
    wn = lin.weight.detach().float().cpu().numpy()
    had = O.hadamard_matrix()
    yg = y.detach().double().cpu().numpy()
    gxg = x.grad.double().cpu().numpy()
    gwg = lin.weight.grad.double().cpu().numpy()
    for gi in range(e):
        a, b = o[gi], o[gi + 1]
        xg, wg, dyg = xn[a:b], wn[gi], dyn[a:b]
        gsx, gsw, gsd = O.global_scale_of(xg), O.global_scale_of(wg), O.global_scale_of(dyg)
        pw, sw = O.quantize_colblock(wg, gsw)  # W_g^T rowblock == W_g colblock
        dw_t = O.dequantize(pw, sw, gsw).astype(np.float64)
        pwd, swd = O.quantize_rowblock(wg, gsw)
        dw_r = O.dequantize(pwd, swd, gsw).astype(np.float64)
        for r0 in (0, (b - a) // 256 * 128, b - a - 128):
            rows = slice(r0, r0 + 128)
            px, sx = O.quantize_rowblock(xg[rows], gsx)
            ref = O.dequantize(px, sx, gsx).astype(np.float64) @ dw_t.T
            got = yg[a + r0:a + r0 + 128]
            assert (np.abs(got - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * np.abs(ref).max()).all(), f"fwd g{gi} r{r0}"
            pd, sd = O.quantize_rowblock(dyg[rows], gsd)
            ref = O.dequantize(pd, sd, gsd).astype(np.float64) @ dw_r.T
            got = gxg[a + r0:a + r0 + 128]
            assert (np.abs(got - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * np.abs(ref).max()).all(), f"dgrad g{gi} r{r0}"
        # wgrad (in, out) storage over the group's own tokens: rows 0..127 and the last 128 of `in`.
        pdc, sdc = O.quantize_colblock(dyg, gsd, hadamard=had)
        ddy = O.dequantize(pdc, sdc, gsd).astype(np.float64)
        for c0 in (0, k - 128):
            pxc, sxc = O.quantize_colblock(xg[:, c0:c0 + 128], gsx, hadamard=had)
            ref = O.dequantize(pxc, sxc, gsx).astype(np.float64) @ ddy.T
            got = gwg[gi, c0:c0 + 128]
            err = np.abs(got - ref).max() / np.abs(ref).max()
            assert err < 1e-5, f"wgrad g{gi} c{c0}: {err}"
    _status_ok()
