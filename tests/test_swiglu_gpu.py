"""The SwiGLU producer epilogue (``rb_nvfp4_gemm_swiglu`` / ``nvfp4.swiglu_mm``) and the modules
built on it (``FP4SwiGLU``, ``FP4FeedForward``).

radiance's FFN computes ``h = F.silu(gate_proj(x)) * up_proj(x)`` in eager bf16
(src/radiance/model/ffn.py:32) and the next linear takes ``global_scale_of(h)``
(src/radiance/nvfp4/quantize.py:205-213).  The fused epilogue must give, bit for bit:
- the same pre-activations as the plain GEMM;
- the h that torch's own kernels compute from them;
- the global scale of that h.
The fused module must give the same outputs and gradients as the unfused composition of
``FP4Linear``s and torch's SwiGLU.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _status_ok():
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16 if t.dtype == torch.bfloat16 else torch.int32).cpu().numpy()


# (m, k, hidden): two-SM tiles, a 128-row tail tile (m % 256 == 128) with a 128-wide N tail
# (2 * hidden % 256 == 128), the one-SM kernel (m == 128), the config 4 expert hidden size, and a
# small hidden size with an N tail.
SHAPES = [(256, 512, 256), (384, 1024, 320), (128, 256, 128), (4096, 2048, 1408), (512, 640, 192)]


@pytest.mark.parametrize("m,k,hidden", SHAPES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_swiglu_mm_matches_torch(nv, m, k, hidden, with_bias):
    g = torch.Generator(device="cuda").manual_seed(m + 7 * k + hidden)
    x = (torch.randn(m, k, device="cuda", generator=g) * 2.0).bfloat16()
    wg = (torch.randn(hidden, k, device="cuda", generator=g) * 0.05).bfloat16()
    wu = (torch.randn(hidden, k, device="cuda", generator=g) * 0.05).bfloat16()
    w = nv.interleave_gate_up(wg, wu)
    bias = None
    if with_bias:
        bias = nv.interleave_gate_up(torch.randn(hidden, device="cuda", generator=g),
                                     torch.randn(hidden, device="cuda", generator=g)).bfloat16()
    xq, wq = nv.quantize(x, -1), nv.quantize(w, -1)
    gu, h, gs = nv.swiglu_mm(xq, wq, bias=bias)
    ref_gu = nv.mm(xq, wq, out_dtype=torch.bfloat16, bias=bias)
    np.testing.assert_array_equal(_bits(gu), _bits(ref_gu))
    gate, up = nv.split_gate_up(gu)
    np.testing.assert_array_equal(_bits(h), _bits(F.silu(gate) * up))
    assert gs.view(torch.int32).item() == nv.global_scale_of(h).view(torch.int32).item()
    _status_ok()


def test_swiglu_saturating_and_negative_inputs(nv):
    """Large pre-activations: the exact path below -128 (exp(-g) overflows, silu -> -0) and
    silu(g) = g above 128."""
    m, k, hidden = 256, 256, 128
    x = (torch.randn(m, k, device="cuda") * 40.0).bfloat16()
    w = (torch.randn(2 * hidden, k, device="cuda") * 0.5).bfloat16()
    xq, wq = nv.quantize(x, -1), nv.quantize(w, -1)
    gu, h, gs = nv.swiglu_mm(xq, wq)
    gate, up = nv.split_gate_up(gu)
    assert gate.float().max().item() > 128.0 and gate.float().min().item() < -128.0
    np.testing.assert_array_equal(_bits(h), _bits(F.silu(gate) * up))
    assert gs.view(torch.int32).item() == nv.global_scale_of(h).view(torch.int32).item()
    _status_ok()


def test_silu_is_exact_on_every_bf16_input(nv):
    """The epilogue's silu (a table plus closed forms) equals bf16(g / (1 + exp(-g))) bit for bit on
    all 65536 bf16 inputs (its only inputs: g is the bf16-rounded pre-activation)."""
    from radiance_b200 import _lib

    lib = _lib.load()
    bad = torch.zeros(2, dtype=torch.int32, device="cuda")
    _lib.check(lib.rb_nvfp4_selftest_silu(bad.data_ptr(), torch.cuda.current_stream().cuda_stream), "selftest_silu")
    count, last = bad.tolist()
    assert count == 0, f"{count} bf16 inputs differ, e.g. bits {last - 1:#06x}"
    _status_ok()


def test_swiglu_workspace_is_left_zeroed(nv):
    """Back-to-back calls on one stream (and a global scale in between, sharing the workspace)."""
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(512, 512, device="cuda") * 0.05).bfloat16()
    xq, wq = nv.quantize(x, -1), nv.quantize(w, -1)
    _, h1, gs1 = nv.swiglu_mm(xq, wq)
    other = nv.global_scale_of(torch.randn(128, 64, device="cuda") * 1e6)
    _, h2, gs2 = nv.swiglu_mm(nv.quantize(x * 0.5, -1), wq)
    assert gs1.item() == nv.global_scale_of(h1).item()
    assert gs2.item() == nv.global_scale_of(h2).item()
    assert other.item() > 1.0
    _status_ok()


def test_swiglu_shape_contract(nv):
    a = nv.quantize(torch.randn(128, 128, device="cuda"), -1)
    with pytest.raises(ValueError, match="contraction mismatch"):
        nv.swiglu_mm(a, nv.quantize(torch.randn(128, 256, device="cuda"), -1))
    with pytest.raises(ValueError, match="rows % 32"):
        nv.interleave_gate_up(torch.randn(48, 64), torch.randn(48, 64))
    with pytest.raises(ValueError, match="multiple of 32"):
        nv.FP4SwiGLU(64, 48, device="cuda")


class _Unfused(nn.Module):
    """The composition FP4FeedForward replaces: the interleaved gate/up FP4Linear, torch's SwiGLU
    on its output, and down_proj computing its own global scale."""

    def __init__(self, nv, ff):
        super().__init__()
        gu = ff.gate_up
        self.gate_up = nv.FP4Linear(gu.in_features, gu.out_features, bias=gu.bias is not None, device="cuda",
                                    dtype=gu.weight.dtype)
        self.down = nv.FP4Linear(ff.down_proj.in_features, ff.down_proj.out_features,
                                 bias=ff.down_proj.bias is not None, device="cuda", dtype=gu.weight.dtype)
        with torch.no_grad():
            self.gate_up.weight.copy_(gu.weight)
            self.down.weight.copy_(ff.down_proj.weight)
            if gu.bias is not None:
                self.gate_up.bias.copy_(gu.bias)
                self.down.bias.copy_(ff.down_proj.bias)
        self._split = nv.split_gate_up

    def forward(self, x):
        g, u = self._split(self.gate_up(x))
        return self.down(F.silu(g) * u)


@pytest.mark.parametrize("with_bias", [False, True])
def test_feedforward_matches_unfused_composition(nv, with_bias):
    torch.manual_seed(3)
    d, hidden, tokens = 512, 1408, 1024
    ff = nv.FP4FeedForward(d, hidden, bias=with_bias, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        for p in ff.parameters():
            p.normal_(0.0, 0.02)
    ref = _Unfused(nv, ff)
    nv.refresh_fp4_weights(ff)
    nv.refresh_fp4_weights(ref)
    x = torch.randn(tokens, d, device="cuda", dtype=torch.bfloat16)
    dy = (torch.randn(tokens, d, device="cuda") * 1e-3).bfloat16()
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    ya, yb = ff(xa), ref(xb)
    np.testing.assert_array_equal(_bits(ya), _bits(yb))
    ya.backward(dy)
    yb.backward(dy)
    np.testing.assert_array_equal(_bits(xa.grad), _bits(xb.grad))
    np.testing.assert_array_equal(_bits(ff.gate_up.weight.grad), _bits(ref.gate_up.weight.grad))
    np.testing.assert_array_equal(_bits(ff.down_proj.weight.grad), _bits(ref.down.weight.grad))
    if with_bias:
        np.testing.assert_array_equal(_bits(ff.gate_up.bias.grad), _bits(ref.gate_up.bias.grad))
        np.testing.assert_array_equal(_bits(ff.down_proj.bias.grad), _bits(ref.down.bias.grad))
    _status_ok()


def test_feedforward_from_radiance_layers(nv):
    """From gate_proj / up_proj / down_proj nn.Linears (radiance's FeedForward, ffn.py:21-23): the
    NVFP4 forward tracks the bf16 one, and the module falls back to bf16 -- h from torch, no global
    scale -- on a token count the kernels cannot tile.  The bound is looser than the reference's
    single-GEMM 0.2 (tests/test_nvfp4.py:173-213): two quantized GEMMs in a row, with h the product of
    two quantized pre-activations (measured ~0.27); a mis-copied or mis-interleaved weight gives ~1.4.
    Exactness against the unfused NVFP4 path is the test above."""
    torch.manual_seed(5)
    d, hidden = 256, 512
    src = nn.Module()
    src.gate_proj = nn.Linear(d, hidden).cuda().bfloat16()
    src.up_proj = nn.Linear(d, hidden).cuda().bfloat16()
    src.down_proj = nn.Linear(hidden, d).cuda().bfloat16()
    ff = nv.FP4FeedForward.from_feedforward(src)
    g, u = ff.gate_up.gate_up_weights()
    assert torch.equal(g, src.gate_proj.weight) and torch.equal(u, src.up_proj.weight)
    nv.refresh_fp4_weights(ff)
    x = torch.randn(512, d, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        ref = src.down_proj(F.silu(src.gate_proj(x)) * src.up_proj(x)).float()
        got = ff(x).float()
        assert ((got - ref).norm() / ref.norm()).item() < 0.4
        h, gs = ff.gate_up(x[:100])
        assert gs is None
        ref_h = F.silu(src.gate_proj(x[:100])) * src.up_proj(x[:100])
        torch.testing.assert_close(h.float(), ref_h.float(), rtol=2e-2, atol=2e-2)
    _status_ok()


def _torch_swiglu_backward(nv, grad_h, gu):
    """Eager autograd's backward of h = F.silu(g) * u (ffn.py:32), on the interleaved layout."""
    import torch.nn.functional as F

    g, u = nv.split_gate_up(gu)
    grad_u = grad_h * F.silu(g)
    grad_g = torch.ops.aten.silu_backward(grad_h * u, g)
    return nv.merge_gate_up(grad_g, grad_u)


@pytest.mark.parametrize("rows,hidden", [(128, 32), (512, 1408), (2048, 5632)])
def test_swiglu_backward_matches_eager_autograd(nv, rows, hidden):
    gen = torch.Generator(device="cuda").manual_seed(rows + hidden)
    gu = (torch.randn(rows, 2 * hidden, device="cuda", generator=gen) * 3).bfloat16()
    grad_h = (torch.randn(rows, hidden, device="cuda", generator=gen) * 1e-3).bfloat16()
    got, gs = nv.swiglu_backward(grad_h, gu)
    want = _torch_swiglu_backward(nv, grad_h, gu)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert gs.view(torch.int32).item() == nv.global_scale_of(want).view(torch.int32).item()
    got2, gs2 = nv.swiglu_backward(grad_h, gu)  # the workspace came back zeroed
    assert torch.equal(got2, got) and torch.equal(gs2, gs)


def test_swiglu_backward_on_every_bf16_gate_value(nv):
    """Every bf16 bit pattern of g (finite, infinite and NaN), against several gradients and up values."""
    g = torch.arange(0, 65536, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16)
    for dh_val, u_val in ((1.0, 1.0), (-3.5e-3, 0.75), (1e-30, -2.0), (448.0, 1e-3)):
        g2 = g.view(-1, 32)  # 2048 rows of one 32-unit group
        u2 = torch.full_like(g2, u_val)
        gu = nv.merge_gate_up(g2, u2)
        grad_h = torch.full_like(g2, dh_val)
        got, _ = nv.swiglu_backward(grad_h, gu)
        want = _torch_swiglu_backward(nv, grad_h, gu)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (dh_val, u_val)


def _eager_swiglu(gu: torch.Tensor, layout: str) -> torch.Tensor:
    """radiance's eager ``F.silu(g) * u`` (ffn.py:32, :148-153) on either layout."""
    import radiance_b200.nvfp4 as nv

    g, u = gu.chunk(2, dim=-1) if layout == "split" else nv.split_gate_up(gu)
    return F.silu(g) * u


@pytest.mark.parametrize("layout", ["split", "interleaved"])
@pytest.mark.parametrize("rows,hidden", [(128, 32), (640, 1408), (2048, 5632)])
def test_swiglu_forward_matches_eager(nv, layout, rows, hidden):
    gen = torch.Generator(device="cuda").manual_seed(rows + hidden + len(layout))
    gu = (torch.randn(rows, 2 * hidden, device="cuda", generator=gen) * 3).bfloat16()
    h, gs = nv.swiglu_forward(gu, layout)
    want = _eager_swiglu(gu, layout)
    assert torch.equal(h.view(torch.int16), want.view(torch.int16))
    assert gs.view(torch.int32).item() == nv.global_scale_of(want).view(torch.int32).item()
    h2, gs2 = nv.swiglu_forward(gu, layout)  # the workspace came back zeroed
    assert torch.equal(h2, h) and torch.equal(gs2, gs)
    _status_ok()


@pytest.mark.parametrize("layout", ["split", "interleaved"])
def test_swiglu_forward_on_every_bf16_gate_value(nv, layout):
    """Every bf16 bit pattern of g against up values that make normal, subnormal and overflowing
    products."""
    g = torch.arange(0, 65536, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16).view(-1, 32)
    for u_val in (1.0, -0.75, 3e-38, -1e-39, 2e38):
        u = torch.full_like(g, u_val)
        gu = torch.cat([g, u], dim=1) if layout == "split" else nv.merge_gate_up(g, u)
        h, _ = nv.swiglu_forward(gu, layout)
        want = _eager_swiglu(gu, layout)
        same = h.view(torch.int16) == want.view(torch.int16)
        both_nan = torch.isnan(h.float()) & torch.isnan(want.float())
        assert bool((same | both_nan).all()), u_val


@pytest.mark.parametrize("layout", ["split", "interleaved"])
def test_swiglu_autograd_matches_eager(nv, layout):
    gen = torch.Generator(device="cuda").manual_seed(5)
    rows, hidden = 1024, 1408
    gu = (torch.randn(rows, 2 * hidden, device="cuda", generator=gen) * 2).bfloat16()
    dh = (torch.randn(rows, hidden, device="cuda", generator=gen) * 1e-2).bfloat16()
    a = gu.clone().requires_grad_(True)
    b = gu.clone().requires_grad_(True)
    ya = nv.swiglu(a, layout)
    yb = _eager_swiglu(b, layout)
    ya.backward(dh)
    yb.backward(dh)
    assert torch.equal(ya.view(torch.int16), yb.view(torch.int16))
    assert torch.equal(a.grad.view(torch.int16), b.grad.view(torch.int16))
    grad, gs = nv.swiglu_backward_strided(dh, gu, layout)
    assert torch.equal(grad, a.grad)
    assert gs.view(torch.int32).item() == nv.global_scale_of(b.grad).view(torch.int32).item()
    _status_ok()


def test_swiglu_layout_contract(nv):
    gu = torch.zeros(128, 96, dtype=torch.bfloat16, device="cuda")  # width not a multiple of 64
    with pytest.raises(ValueError, match="multiple of 64"):
        nv.swiglu_forward(gu)
    with pytest.raises(ValueError, match="layout"):
        nv.swiglu_forward(torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda"), "rows")
    with pytest.raises(ValueError, match="bf16"):
        nv.swiglu_forward(torch.zeros(128, 128, dtype=torch.float32, device="cuda"))
