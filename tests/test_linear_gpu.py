"""FP4Linear on the B200 library: the reference's layer contract (tests/test_nvfp4.py:406-716 in
jamespa16/radiance) -- the autograd-trap negative control, the stale weight cache and its in-place
refresh, state-dict hygiene, the ragged-shape fallback, grad_gemms off, packed activation saving
(bit-identical, and smaller), and the per-step seed advance -- plus parity of each GEMM of the
layer with the oracle."""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _layer(nv, in_f=256, out_f=512, bias=True, **kw):
    layer = nv.FP4Linear(in_f, out_f, bias=bias, **kw).cuda()
    layer.refresh_fp4_cache()
    return layer


def _cos(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


def test_gradient_is_not_the_autograd_trap(nv):
    torch.manual_seed(0)
    x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
    layer = _layer(nv, 256, 512, bias=False)
    grad_out = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    xr = x.detach().float().requires_grad_(True)
    torch.nn.functional.linear(xr, layer.weight.detach().float()).backward(grad_out.float())
    xg = x.detach().clone().requires_grad_(True)
    layer(xg).backward(grad_out)
    # The trap: quantize/dequantize inside autograd's view (only the amax path has a gradient).
    xb = x.detach().clone().requires_grad_(True)
    gs = (xb.abs().amax().float() / (6 * 448)).clamp(min=1e-12)
    blocks = xb.reshape(256, 16, 16).float()
    scale = (blocks.abs().amax(-1, keepdim=True) / 6.0 / gs).clamp(min=1e-12)
    q = (blocks / (scale * gs)).clamp(-6, 6)
    codes = torch.bucketize(q.abs(), torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device="cuda"))
    fake = torch.where(q < 0, -1.0, 1.0) * codes.float() * (scale * gs)
    torch.nn.functional.linear(fake.reshape(256, 256).bfloat16(), layer.weight.to(torch.bfloat16)).backward(grad_out)
    assert xb.grad.abs().sum() > 0
    assert _cos(xb.grad, xr.grad) < 0.5
    assert _cos(xg.grad, xr.grad) > 0.95
    assert _cos(layer.weight.grad, (grad_out.float().t() @ x.float())) > 0.95


def test_layer_gemms_match_oracle(nv):
    """Forward, dgrad and wgrad of one layer step, each against the oracle GEMM of the exact
    operands the layer quantized (round-to-nearest recipe so the operands are reproducible)."""
    torch.manual_seed(2)
    layer = _layer(nv, 512, 384, bias=False, recipe=nv.FP4Recipe(stochastic_rounding=False))
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
    y = layer(x)
    y.backward(gy)
    h = O.hadamard_matrix()
    xn, gyn = x.detach().float().cpu().numpy(), gy.float().cpu().numpy()
    wn = layer.weight.detach().float().cpu().numpy()
    gx, gg, gw = O.global_scale_of(xn), O.global_scale_of(gyn), O.global_scale_of(wn)
    fwd = O.gemm_reference(*O.quantize(xn, -1, gs=gx), *O.quantize(wn, -1, gs=gw))
    dgr = O.gemm_reference(*O.quantize(gyn, -1, gs=gg), *O.quantize(wn, 0, gs=gw))
    wgr = O.gemm_reference(*O.quantize(gyn, 0, gs=gg, hadamard=h), *O.quantize(xn, 0, gs=gx, hadamard=h))
    for got, ref, bf16 in ((y, fwd, True), (x.grad, dgr, True), (layer.weight.grad, wgr, False)):
        g = got.detach().double().cpu().numpy()
        if bf16:
            assert (np.abs(g - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * np.abs(ref).max()).all()
        else:
            assert np.abs(g - ref).max() / np.abs(ref).max() <= 1e-3


def test_weight_cache_is_stale_until_refreshed(nv):
    layer = _layer(nv, 256, 512)
    x = torch.randn(128, 256, device="cuda", dtype=torch.bfloat16)
    before = layer(x).clone()
    with torch.no_grad():
        layer.weight.mul_(1.5)
    torch.testing.assert_close(layer(x), before, rtol=0, atol=0)
    ptrs = [layer._w_fwd_packed.data_ptr(), layer._w_dgrad_packed.data_ptr(), layer._w_fwd_scale.data_ptr()]
    layer.refresh_fp4_cache()
    assert not torch.equal(layer(x), before)
    assert ptrs == [layer._w_fwd_packed.data_ptr(), layer._w_dgrad_packed.data_ptr(), layer._w_fwd_scale.data_ptr()]


def test_weight_cache_matches_oracle(nv):
    layer = _layer(nv, 640, 384)
    wn = layer.weight.detach().float().cpu().numpy()
    gw = O.global_scale_of(wn)
    assert np.float32(layer._w_fwd_gs.item()) == gw and np.float32(layer._w_dgrad_gs.item()) == gw
    p, s, _ = O.quantize(wn, -1, gs=gw)
    np.testing.assert_array_equal(layer._w_fwd_packed.cpu().numpy(), p)
    np.testing.assert_array_equal(layer._w_fwd_scale.cpu().numpy(), s)
    p, s, _ = O.quantize(wn, 0, gs=gw)
    np.testing.assert_array_equal(layer._w_dgrad_packed.cpu().numpy(), p)
    np.testing.assert_array_equal(layer._w_dgrad_scale.cpu().numpy(), s)


def test_fp4_buffers_stay_out_of_the_state_dict(nv):
    fp4 = nv.FP4Linear(256, 512)
    plain = torch.nn.Linear(256, 512)
    assert set(fp4.state_dict()) == set(plain.state_dict()) == {"weight", "bias"}
    fp4.load_state_dict(plain.state_dict(), strict=True)
    plain.load_state_dict(fp4.state_dict(), strict=True)


def test_loading_a_state_dict_invalidates_the_cache(nv):
    layer = _layer(nv, 256, 512)
    assert layer._cache_valid
    layer.load_state_dict(layer.state_dict())
    assert not layer._cache_valid


def test_falls_back_to_bf16_on_ragged_token_counts(nv):
    layer = _layer(nv, 256, 512)
    x = torch.randn(100, 256, device="cuda", dtype=torch.bfloat16)
    expected = torch.nn.functional.linear(x, layer.weight.to(x.dtype), layer.bias.to(x.dtype))
    torch.testing.assert_close(layer(x), expected, rtol=0, atol=0)


def test_cpu_input_raises(nv):
    layer = nv.FP4Linear(256, 512)
    with pytest.raises(RuntimeError):
        layer(torch.randn(128, 256))


def test_grad_gemms_off_keeps_the_backward_in_bf16(nv):
    torch.manual_seed(0)
    x = torch.randn(128, 256, device="cuda", dtype=torch.bfloat16)
    grad_out = torch.randn(128, 512, device="cuda", dtype=torch.bfloat16)
    grads = {}
    for name, recipe in [("fp4", nv.FP4Recipe(grad_gemms=True)), ("bf16", nv.FP4Recipe(grad_gemms=False))]:
        torch.manual_seed(1)
        layer = _layer(nv, 256, 512, recipe=recipe)
        xg = x.clone().requires_grad_(True)
        layer(xg).backward(grad_out)
        grads[name] = xg.grad.clone()
    assert not torch.equal(grads["fp4"], grads["bf16"])
    assert _cos(grads["fp4"], grads["bf16"]) > 0.9


def test_saving_activations_packed_is_bit_identical(nv):
    torch.manual_seed(0)
    x = torch.randn(512, 1280, device="cuda", dtype=torch.bfloat16)
    grad_out = torch.randn(512, 2560, device="cuda", dtype=torch.bfloat16)
    results = {}
    for save in (False, True):
        torch.manual_seed(1)
        layer = nv.FP4Linear(1280, 2560, recipe=nv.FP4Recipe(save_activations=save, stochastic_rounding=False)).cuda()
        layer.refresh_fp4_cache()
        xg = x.clone().requires_grad_(True)
        layer(xg).backward(grad_out)
        results[save] = (xg.grad.clone(), layer.weight.grad.clone())
    torch.testing.assert_close(results[True][0], results[False][0], rtol=0, atol=0)
    torch.testing.assert_close(results[True][1], results[False][1], rtol=0, atol=0)


def test_saving_activations_packed_uses_less_memory(nv):
    sizes = {}
    for save in (False, True):
        torch.manual_seed(1)
        layer = nv.FP4Linear(1280, 2560, recipe=nv.FP4Recipe(save_activations=save, stochastic_rounding=False)).cuda()
        layer.refresh_fp4_cache()
        x = torch.randn(4096, 1280, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        out = layer(x)
        node = out.grad_fn
        while not hasattr(node, "saved_tensors") or not node.saved_tensors:
            node = node.next_functions[0][0]
        sizes[save] = sum(t.numel() * t.element_size() for t in node.saved_tensors)
    assert sizes[False] - sizes[True] > 0.5 * 4096 * 1280 * 2


def test_grad_gemms_off_keeps_the_bf16_activation(nv):
    torch.manual_seed(1)
    layer = nv.FP4Linear(1280, 2560, recipe=nv.FP4Recipe(grad_gemms=False, save_activations=True)).cuda()
    layer.refresh_fp4_cache()
    x = torch.randn(512, 1280, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    layer(x).backward(torch.randn(512, 2560, device="cuda", dtype=torch.bfloat16))
    assert x.grad is not None and torch.isfinite(x.grad).all()
    assert torch.isfinite(layer.weight.grad).all()


def test_refresh_advances_the_seed(nv):
    model = torch.nn.Sequential(nv.FP4Linear(256, 512), torch.nn.GELU(), nv.FP4Linear(512, 256)).cuda()
    seeds = []
    for _ in range(3):
        nv.refresh_fp4_weights(model)
        seeds.append([m._seed.item() for m in model.modules() if isinstance(m, nv.FP4Linear)])
    assert seeds == [[1, 1], [2, 2], [3, 3]]


def test_stochastic_backward_changes_with_the_seed(nv):
    layer = _layer(nv, 256, 512, bias=False)
    x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
    gy = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)

    def grads():
        xg = x.clone().requires_grad_(True)
        layer.weight.grad = None
        layer(xg).backward(gy)
        return xg.grad.clone()

    a, b = grads(), grads()
    torch.testing.assert_close(a, b, rtol=0, atol=0)  # same seed: reproducible
    layer._seed.add_(1)
    assert not torch.equal(a, grads())


def test_reshaped_3d_inputs(nv):
    layer = _layer(nv, 256, 512)
    x = torch.randn(2, 64, 256, device="cuda", dtype=torch.bfloat16)
    y = layer(x)
    assert y.shape == (2, 64, 512)
    torch.testing.assert_close(y.view(128, 512), layer(x.view(128, 256)), rtol=0, atol=0)


def test_cuda_graph_capture_of_a_layer_step(nv):
    """Global scales, alpha and the seed are device pointers and outputs come from the caching
    allocator, so a forward+backward step replays under a CUDA graph with the same result."""
    layer = _layer(nv, 512, 512, bias=False, recipe=nv.FP4Recipe(stochastic_rounding=False))
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    gy = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)

    def step():
        xg = x.detach().requires_grad_(True)
        y = layer(xg)
        return torch.autograd.grad(y, (xg, layer.weight), gy)

    ref = step()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out[0], ref[0], rtol=0, atol=0)
    torch.testing.assert_close(out[1], ref[1], rtol=0, atol=0)
