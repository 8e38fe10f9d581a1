"""Grouped (mixture-of-experts) NVFP4 path against the oracle.

radiance has no FP4 expert path (transformer.py:204-213 rejects FP4 + MoE) and no tests for one, so
the oracle is a composition: every group is checked against the single-tensor oracle applied to that
group alone (per-group global scale, ``quantize_rowblock`` / ``quantize_colblock``, dequantized
float64 matmul), on the stacked layout of ``radiance_b200.nvfp4.grouped``.
"""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import to_numpy_f32, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def grp():
    import radiance_b200.nvfp4 as nv
    import radiance_b200.nvfp4.grouped as grp

    assert nv.nvfp4_supported()
    return grp


def _status_ok():
    from radiance_b200 import _lib

    assert _lib.device_status() == 0


def _stacked(counts, k, dtype=torch.bfloat16, scales=None, seed=0):
    """Expert-sorted tokens: group g has counts[g] rows (already multiples of 128), its own scale."""
    g = torch.Generator().manual_seed(seed)
    parts = []
    for i, c in enumerate(counts):
        s = 1.0 if scales is None else scales[i]
        parts.append((torch.randn(c, k, generator=g) * s).to(dtype))
    x = torch.cat(parts).cuda()
    offs = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int64, device="cuda")
    return x, offs


COUNTS = [384, 0, 128, 768, 256]  # uneven, one empty group, one single-tile group


def test_align_offsets(grp):
    counts = torch.tensor([5, 0, 128, 129, 300], dtype=torch.int64, device="cuda")
    offs = grp.align_offsets(counts)
    assert offs.tolist() == [0, 128, 128, 256, 512, 896]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_global_scale_grouped_matches_oracle(grp, dtype):
    x, offs = _stacked(COUNTS, 320, dtype, scales=[1.0, 1.0, 1e-3, 40.0, 0.5])
    gs = grp.global_scale_grouped(x, offs).cpu().numpy()
    xn = to_numpy_f32(x)
    o = offs.tolist()
    for gi in range(len(COUNTS)):
        part = xn[o[gi]:o[gi + 1]]
        want = O.global_scale_of(part) if part.size else np.float32(1e-12)
        assert gs[gi].view(np.uint32) == np.float32(want).view(np.uint32), gi
    # the workspace comes back zeroed: a second call agrees
    assert np.array_equal(grp.global_scale_grouped(x, offs).cpu().numpy(), gs)
    _status_ok()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rotate", [False, True])
def test_quantize_grouped_equals_per_group_oracle(grp, dtype, rotate):
    k = 320
    x, offs = _stacked(COUNTS, k, dtype, scales=[1.0, 1.0, 1e-3, 40.0, 0.5], seed=1)
    t = x.shape[0]
    gs = grp.global_scale_grouped(x, offs)
    had = O.hadamard_matrix() if rotate else None
    row = (torch.empty(t, k // 2, dtype=torch.uint8, device="cuda"),
           torch.empty(O.to_blocked(np.zeros((t, k // 16), np.uint8)).size, dtype=torch.uint8, device="cuda"))
    col = (torch.empty(k, t // 2, dtype=torch.uint8, device="cuda"),
           torch.empty(O.to_blocked(np.zeros((k, t // 16), np.uint8)).size, dtype=torch.uint8, device="cuda"))
    grp.quantize_grouped_into_(x, offs, gs, row=row, col=col,
                               hadamard=None if had is None else torch.from_numpy(had).cuda())
    xn = to_numpy_f32(x)
    gsn = gs.cpu().numpy()
    rp, rs = u8(row[0]), O.from_blocked(u8(row[1]), t, k // 16)
    cp, cs = u8(col[0]), O.from_blocked(u8(col[1]), k, t // 16)
    o = offs.tolist()
    for gi in range(len(COUNTS)):
        a, b = o[gi], o[gi + 1]
        if a == b:
            continue
        p, s = O.quantize_rowblock(xn[a:b], gsn[gi])
        np.testing.assert_array_equal(rp[a:b], p, err_msg=f"row packed g{gi}")
        np.testing.assert_array_equal(rs[a:b], s, err_msg=f"row scale g{gi}")
        p, s = O.quantize_colblock(xn[a:b], gsn[gi], hadamard=had)
        np.testing.assert_array_equal(cp[:, a // 2:b // 2], p, err_msg=f"col packed g{gi}")
        np.testing.assert_array_equal(cs[:, a // 16:b // 16], s, err_msg=f"col scale g{gi}")
    _status_ok()


def _quant_rows(grp, x, offs, gs):
    t, k = x.shape
    row = (torch.empty(t, k // 2, dtype=torch.uint8, device="cuda"),
           torch.empty(O.to_blocked(np.zeros((t, k // 16), np.uint8)).size, dtype=torch.uint8, device="cuda"))
    grp.quantize_grouped_into_(x, offs, gs, row=row)
    return row


def _deq_rows(packed, scale_flat, rows, k, gs_per_row):
    p = u8(packed)
    s = O.from_blocked(u8(scale_flat), rows, k // 16)
    out = np.empty((rows, k), np.float64)
    for r0 in range(0, rows, 128):
        out[r0:r0 + 128] = O.dequantize(p[r0:r0 + 128], s[r0:r0 + 128], gs_per_row[r0])
    return out


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_grouped_gemm_over_rows_matches_oracle(grp, out_dtype):
    """Forward/dgrad shape: token groups times per-expert weights (E x n rows), k shared."""
    k, n = 320, 384
    counts = COUNTS
    e = len(counts)
    x, offs = _stacked(counts, k, scales=[1.0, 1.0, 2.0, 0.5, 3.0], seed=2)
    w = (torch.randn(e * n, k, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16).cuda()
    woffs = torch.arange(e + 1, dtype=torch.int64, device="cuda") * n
    gx, gw = grp.global_scale_grouped(x, offs), grp.global_scale_grouped(w, woffs)
    xq, wq = _quant_rows(grp, x, offs, gx), _quant_rows(grp, w, woffs, gw)
    groups = grp.groups_over_rows(offs, n, k)
    t = x.shape[0]
    out = torch.full((t, n), 7.0, dtype=out_dtype, device="cuda")
    grp.grouped_mm(xq, wq, groups, n=n, k_total=k, out_rows=t, alpha_a=gx, alpha_b=gw, out_dtype=out_dtype, out=out)
    o = offs.tolist()
    gxr = np.repeat(gx.cpu().numpy(), np.diff(o))
    gwr = np.repeat(gw.cpu().numpy(), n)
    dx = _deq_rows(xq[0], xq[1], t, k, gxr)
    dw = _deq_rows(wq[0], wq[1], e * n, k, gwr)
    got = out.double().cpu().numpy()
    for gi in range(e):
        a, b = o[gi], o[gi + 1]
        if a == b:
            continue
        ref = dx[a:b] @ dw[gi * n:(gi + 1) * n].T
        g = got[a:b]
        scale = np.abs(ref).max()
        if out_dtype == torch.bfloat16:
            assert (np.abs(g - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * scale).all(), gi
        else:
            assert np.abs(g - ref).max() / scale < 1e-5, gi
    _status_ok()


def test_grouped_gemm_over_contraction_matches_oracle(grp):
    """wgrad shape: each group contracts over its own token range of two colblock operands; an
    empty group writes zeros."""
    k, n = 256, 384
    counts = COUNTS
    e = len(counts)
    x, offs = _stacked(counts, k, scales=[1.0, 1.0, 0.1, 1.0, 4.0], seed=4)
    dy, _ = _stacked(counts, n, scales=[1e-3, 1e-3, 1e-3, 2e-3, 1e-3], seed=5)
    t = x.shape[0]
    gx, gg = grp.global_scale_grouped(x, offs), grp.global_scale_grouped(dy, offs)
    had = torch.from_numpy(O.hadamard_matrix()).cuda()
    xc = (torch.empty(k, t // 2, dtype=torch.uint8, device="cuda"),
          torch.empty(O.to_blocked(np.zeros((k, t // 16), np.uint8)).size, dtype=torch.uint8, device="cuda"))
    gc = (torch.empty(n, t // 2, dtype=torch.uint8, device="cuda"),
          torch.empty(O.to_blocked(np.zeros((n, t // 16), np.uint8)).size, dtype=torch.uint8, device="cuda"))
    grp.quantize_grouped_into_(x, offs, gx, col=xc, hadamard=had)
    grp.quantize_grouped_into_(dy, offs, gg, col=gc, hadamard=had)
    out = torch.full((e * k, n), 5.0, dtype=torch.float32, device="cuda")
    grp.grouped_mm(xc, gc, grp.groups_over_contraction(offs, k), n=n, k_total=t, out_rows=e * k, alpha_a=gx,
                   alpha_b=gg, out_dtype=torch.float32, out=out)
    o = offs.tolist()
    xp, xs = u8(xc[0]), O.from_blocked(u8(xc[1]), k, t // 16)
    gp, gsc = u8(gc[0]), O.from_blocked(u8(gc[1]), n, t // 16)
    got = out.double().cpu().numpy()
    gxn, ggn = gx.cpu().numpy(), gg.cpu().numpy()
    for gi in range(e):
        a, b = o[gi], o[gi + 1]
        blk = got[gi * k:(gi + 1) * k]
        if a == b:
            assert (blk == 0).all(), "an empty contraction must write zeros"
            continue
        da = O.dequantize(xp[:, a // 2:b // 2], xs[:, a // 16:b // 16], gxn[gi]).astype(np.float64)
        db = O.dequantize(gp[:, a // 2:b // 2], gsc[:, a // 16:b // 16], ggn[gi]).astype(np.float64)
        ref = da @ db.T
        assert np.abs(blk - ref).max() / np.abs(ref).max() < 1e-5, gi
    _status_ok()


def test_grouped_gemm_rejects_a_bad_record_and_keeps_the_rest(grp):
    k, n = 256, 256
    x, offs = _stacked([256, 256], k, seed=6)
    w = (torch.randn(2 * n, k) * 0.02).to(torch.bfloat16).cuda()
    woffs = torch.tensor([0, n, 2 * n], dtype=torch.int64, device="cuda")
    gx, gw = grp.global_scale_grouped(x, offs), grp.global_scale_grouped(w, woffs)
    xq, wq = _quant_rows(grp, x, offs, gx), _quant_rows(grp, w, woffs, gw)
    groups = grp.groups_over_rows(offs, n, k).clone()
    groups[1, 3] = 200  # m not a multiple of 128
    out = torch.zeros(512, n, dtype=torch.float32, device="cuda")
    grp.grouped_mm(xq, wq, groups, n=n, k_total=k, out_rows=512, alpha_a=gx, alpha_b=gw, out_dtype=torch.float32,
                   out=out)
    from radiance_b200 import _lib

    assert _lib.device_status() == 5
    assert out[256:].abs().max().item() == 0.0
    assert out[:256].abs().max().item() > 0.0


def test_fp4_grouped_linear_matches_per_expert_oracle(grp):
    """Forward and (round-to-nearest) gradients of FP4GroupedLinear equal, per expert, the
    single-linear oracle: X_g and W_g^T rowblock for the forward, dY_g against W_g rowblock for
    dgrad, rotated colblock operands for wgrad."""
    from radiance_b200.nvfp4 import FP4Recipe

    e, k, n = 3, 256, 384
    counts = [256, 128, 384]
    lin = grp.FP4GroupedLinear(e, k, n, recipe=FP4Recipe(stochastic_rounding=False), device="cuda")
    lin.refresh_fp4_cache()
    x, offs = _stacked(counts, k, seed=7)
    x.requires_grad_(True)
    y = lin(x, offs)
    dy, _ = _stacked(counts, n, scales=[1e-3] * 3, seed=8)
    y.backward(dy)
    xn, wn, dyn = to_numpy_f32(x), lin.weight.detach().float().cpu().numpy(), to_numpy_f32(dy)
    had = O.hadamard_matrix()
    o = offs.tolist()
    yg, gxg, gwg = y.double().detach().cpu().numpy(), x.grad.double().cpu().numpy(), lin.weight.grad.double().cpu().numpy()
    for gi in range(e):
        a, b = o[gi], o[gi + 1]
        xg, wg, dyg = xn[a:b], wn[gi], dyn[a:b]
        gsx, gsw, gsd = O.global_scale_of(xg), O.global_scale_of(wg), O.global_scale_of(dyg)
        # forward: y = deq(X_g rowblock) @ deq(W_g^T rowblock)^T
        px, sx = O.quantize_rowblock(xg, gsx)
        pw, sw = O.quantize_colblock(wg, gsw)  # W_g^T rowblock == W_g colblock
        ref = O.dequantize(px, sx, gsx).astype(np.float64) @ O.dequantize(pw, sw, gsw).astype(np.float64).T
        assert (np.abs(yg[a:b] - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * np.abs(ref).max()).all(), f"fwd g{gi}"
        # dgrad: dX = deq(dY rowblock) @ deq(W_g rowblock)^T
        pd, sd = O.quantize_rowblock(dyg, gsd)
        pwd, swd = O.quantize_rowblock(wg, gsw)
        ref = O.dequantize(pd, sd, gsd).astype(np.float64) @ O.dequantize(pwd, swd, gsw).astype(np.float64).T
        assert (np.abs(gxg[a:b] - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * np.abs(ref).max()).all(), f"dgrad g{gi}"
        # wgrad (in, out) storage: deq(X colblock, R) @ deq(dY colblock, R)^T
        pxc, sxc = O.quantize_colblock(xg, gsx, hadamard=had)
        pdc, sdc = O.quantize_colblock(dyg, gsd, hadamard=had)
        ref = O.dequantize(pxc, sxc, gsx).astype(np.float64) @ O.dequantize(pdc, sdc, gsd).astype(np.float64).T
        assert np.abs(gwg[gi] - ref).max() / np.abs(ref).max() < 1e-5, f"wgrad g{gi}"
    _status_ok()


def test_fp4_batched_experts_tracks_bf16_experts(grp):
    """FP4BatchedExperts on radiance's (experts, capacity, d) layout against the same experts in
    fp32 (BatchedExperts.forward, ffn.py:148-153): outputs and gradients point the same way
    (cosine > 0.95, the reference's FP4 gradient bar, tests/test_nvfp4.py:415-462)."""
    import torch.nn.functional as F

    e, cap, d, f = 4, 256, 256, 384
    moe = grp.FP4BatchedExperts(e, d, f, device="cuda")
    moe.refresh_fp4_cache()
    x = torch.randn(e, cap, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = moe(x)
    g = torch.randn_like(y) * 1e-2
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wgu, wd = moe.gate_up.weight.detach().float().requires_grad_(True), moe.down.weight.detach().float()
    h = torch.bmm(xr, wgu)
    hg, hu = h.split(f, dim=2)
    yr = torch.bmm(F.silu(hg) * hu, wd)
    yr.backward(g.float())

    def cos(a, b):
        return F.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0).item()

    assert cos(y, yr) > 0.95
    assert cos(x.grad, xr.grad) > 0.95
    assert cos(moe.gate_up.weight.grad, wgu.grad) > 0.95
    _status_ok()
