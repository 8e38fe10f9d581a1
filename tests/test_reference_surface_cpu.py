"""The ``quantize_reference`` family re-exported by ``radiance_b200.nvfp4`` (radiance's format
definition in plain torch, src/radiance/nvfp4/quantize.py:86-320, :412-433), checked on CPU against
the vectors the reference itself produced (``tests/golden/nvfp4_golden.npz``), bit for bit; plus the
custom op's registered name.  Nothing in the NVFP4 path calls these functions: a CPU tensor given to
``quantize`` still raises."""

import numpy as np
import pytest
import torch

import radiance_b200.nvfp4 as nv
from oracle import nvfp4_oracle as O


def _x(golden, name):
    raw = golden[f"{name}/x"]
    if int(golden[f"{name}/dtype"]) == 0:
        return torch.from_numpy(raw.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(raw.astype(np.float32))


def _u8(t):
    return t.view(torch.uint8).numpy()


def test_surface_names_are_exported():
    for name in ("quantize_reference", "ref_quantize_rowblock", "ref_quantize_colblock", "ref_to_blocked",
                 "encode_e2m1", "dequantize", "_block_scale", "global_scale_of", "scale_denominator",
                 "blocked_offset", "pack_nibbles", "unpack_nibbles", "nvfp4_mm", "mm", "quantize"):
        assert hasattr(nv, name), name
    assert hasattr(torch.ops.radiance, "nvfp4_mm")


@pytest.mark.parametrize("tag", ["row", "col", "colh", "colh1"])
def test_quantize_reference_matches_golden(golden, tag):
    had = {"colh": golden["hadamard_seed0"], "colh1": golden["hadamard_seed1"]}.get(tag)
    for name in [str(c) for c in golden["cases"]]:
        x = _x(golden, name)
        gs = torch.from_numpy(np.array(golden[f"{name}/gs"], dtype=np.float32))
        q = nv.quantize_reference(x, -1 if tag == "row" else 0, global_scale=gs,
                                  hadamard=None if had is None else torch.from_numpy(had))
        np.testing.assert_array_equal(_u8(q.packed), golden[f"{name}/{tag}_packed"], err_msg=f"{name} {tag}")
        np.testing.assert_array_equal(_u8(q.scale), golden[f"{name}/{tag}_scale"], err_msg=f"{name} {tag}")
        if tag == "row":  # the reference-side global scale agrees too
            own = nv.quantize_reference(x, -1)
            assert own.global_scale.view(torch.int32).item() == gs.view(torch.int32).item(), name


def test_stochastic_rounding_for_a_given_draw(golden):
    name = "rand1"
    x = _x(golden, name)
    gs = torch.from_numpy(np.array(golden[f"{name}/gs"], dtype=np.float32))
    u = torch.from_numpy(golden[f"{name}/u"].astype(np.float32))
    p, s = nv.ref_quantize_rowblock(x, gs, u=u)
    np.testing.assert_array_equal(_u8(p), golden[f"{name}/sr_row_packed"])
    np.testing.assert_array_equal(_u8(nv.ref_to_blocked(s)), golden[f"{name}/sr_row_scale"])
    p, s = nv.ref_quantize_colblock(x, gs, hadamard=torch.from_numpy(golden["hadamard_seed0"]), u=u)
    np.testing.assert_array_equal(_u8(p), golden[f"{name}/sr_colh_packed"])
    np.testing.assert_array_equal(_u8(nv.ref_to_blocked(s)), golden[f"{name}/sr_colh_scale"])


def test_encode_ladder_and_ties(golden):
    grid = torch.from_numpy(golden["encode/grid"].astype(np.float32))
    got = nv.encode_e2m1(grid, sign=torch.zeros_like(grid, dtype=torch.bool))
    np.testing.assert_array_equal(got.numpy(), golden["encode/grid_rn"])
    u = torch.from_numpy(golden["encode/grid_u"].astype(np.float32))
    got = nv.encode_e2m1(grid, sign=torch.zeros_like(grid, dtype=torch.bool), u=u)
    np.testing.assert_array_equal(got.numpy(), golden["encode/grid_sr"])
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    assert nv.encode_e2m1(ties, sign=ties < 0).tolist() == [0, 2, 2, 4, 4, 6, 6]
    neg = nv.encode_e2m1(torch.tensor([1.0, 6.0]), sign=torch.tensor([True, True]))
    assert neg.tolist() == [0xA, 0xF]


@pytest.mark.parametrize("shape", ["128x4", "256x8", "4096x80", "100x16", "64x16"])
def test_ref_to_blocked_matches_golden(golden, shape):
    scale = torch.from_numpy(golden[f"blocked/{shape}/scale"])
    np.testing.assert_array_equal(nv.ref_to_blocked(scale).numpy(), golden[f"blocked/{shape}/expected"])


def test_dequantize_and_block_scale(golden):
    x = torch.from_numpy(golden["dequant/x"].view(np.int16).copy()).view(torch.bfloat16)
    gs = (x.float().abs().amax() / 2688.0).clamp(min=1e-12)
    p, s = nv.ref_quantize_rowblock(x, gs)
    np.testing.assert_array_equal(nv.dequantize(p, s, gs).numpy(), golden["dequant/out"])
    amax = torch.tensor([0.0, 1e-30, 1.0, 1e30])
    scale, divisor = nv._block_scale(amax, torch.tensor(1.0 / 2688.0))
    assert scale.view(torch.uint8).tolist()[0] == 0x01 and divisor[0].item() == 1.0
    assert scale.view(torch.uint8).tolist()[-1] == 0x7E and divisor[-1].item() == 448.0
    b, d = O.block_scale(amax.numpy(), np.float32(1.0 / 2688.0))
    np.testing.assert_array_equal(scale.view(torch.uint8).numpy(), b)
    np.testing.assert_array_equal(divisor.numpy(), d)


def test_the_nvfp4_path_still_refuses_cpu_tensors():
    x = torch.randn(128, 64)
    with pytest.raises(RuntimeError, match="no CPU"):
        nv.quantize(x, -1)
    with pytest.raises(ValueError, match="axis 0 or -1"):
        nv.quantize_reference(x, 2)
