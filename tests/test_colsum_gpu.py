"""The global scale and column sums from one read (``global_scale_and_column_sums``, the dbias
fusion): the scale is bit-identical to ``global_scale_of``; the fp32 column sums match a float64
sum to accumulation noise and repeat bit for bit; ``FP4Linear``'s bias gradient equals the
reference's ``grad_y.sum(0)`` (a bf16 sum) to one bf16 rounding."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


@pytest.mark.parametrize("rows,cols,dtype,strided", [
    (256, 512, torch.bfloat16, False), (1001, 136, torch.bfloat16, False), (4096, 6144, torch.bfloat16, False),
    (513, 260, torch.float32, False), (384, 1024, torch.bfloat16, True), (3, 8, torch.bfloat16, False),
])
def test_scale_and_sums(nv, rows, cols, dtype, strided):
    torch.manual_seed(rows + cols)
    base = torch.randn(rows, cols + (256 if strided else 0), device="cuda").to(dtype) * 0.01
    x = base[:, 128:128 + cols] if strided else base
    gs, cs = nv.global_scale_and_column_sums(x)
    assert torch.equal(gs, nv.global_scale_of(x))
    ref = x.double().sum(0)
    noise = x.double().abs().sum(0) * 2.0**-20
    assert ((cs.double() - ref).abs() <= noise + 1e-30).all()
    gs2, cs2 = nv.global_scale_and_column_sums(x)
    assert torch.equal(cs, cs2) and torch.equal(gs, gs2)
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


def test_linear_bias_gradient(nv):
    torch.manual_seed(4)
    layer = nv.FP4Linear(512, 768, bias=True).cuda()
    layer.refresh_fp4_cache()
    x = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(1024, 768, device="cuda", dtype=torch.bfloat16) * 1e-2
    layer(x).backward(gy)
    want = gy.sum(0).float()  # radiance: grad_y.sum(0) in bf16, then .to(weight.dtype)
    got = layer.bias.grad
    assert got.dtype == layer.bias.dtype
    assert ((got - want).abs() <= want.abs() * 2.0**-8 + 1e-6).all()
