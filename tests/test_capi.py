"""The C ABI without a GPU: the library loads, exports every function ``include/*.h`` declares,
and rejects bad arguments on the host with the reference's error text."""

import ctypes
import glob
import os
import re

import pytest

from radiance_b200 import _lib
from tests.conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(rb_\w+)\s*\(", text))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert "rb_nvfp4_quantize" in declared and "rb_nvfp4_gemm" in declared
    for name in declared:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.rb_nvfp4_abi_version() == _lib.ABI_VERSION


def test_shape_contract_is_checked_on_the_host():
    lib = _lib.load()
    buf = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    rc = lib.rb_nvfp4_quantize(buf, 0, 100, 128, 128, buf, None, None, buf, buf, None, None, None)
    assert rc == 1
    assert "rows % 128" in lib.rb_nvfp4_last_error().decode()
    with pytest.raises(ValueError, match="rows % 128"):
        _lib.check(rc, "nvfp4.quantize")
    rc = lib.rb_nvfp4_quantize(buf, 0, 128, 128, 128, buf, None, None, None, None, None, None, None)
    assert rc == 2 and "no output form" in lib.rb_nvfp4_last_error().decode()
    rc = lib.rb_nvfp4_quantize(buf, 7, 128, 128, 128, buf, None, None, buf, buf, None, None, None)
    assert rc == 2 and "dtype" in lib.rb_nvfp4_last_error().decode()
    rc = lib.rb_nvfp4_global_scale(buf, 0, 4, 4, 2, buf, buf, None)
    assert rc == 1


def test_gemm_shape_contract_is_checked_on_the_host():
    lib = _lib.load()
    buf = ctypes.c_void_p(256)
    rc = lib.rb_nvfp4_gemm(buf, buf, buf, buf, 100, 128, 128, None, None, None, 0, buf, 0, 128, None)
    assert rc in (1, 2)
    assert lib.rb_nvfp4_last_error().decode()


def test_ops_refuse_cpu_tensors():
    import torch

    import radiance_b200.nvfp4 as nv

    x = torch.randn(128, 64)
    with pytest.raises(RuntimeError, match="no CPU"):
        nv.quantize(x, -1)
    with pytest.raises(RuntimeError, match="no CPU"):
        nv.global_scale_of(x)
    gu = torch.randn(128, 128).bfloat16()
    with pytest.raises(RuntimeError, match="no CPU"):
        nv.swiglu(gu, "split")
    with pytest.raises(RuntimeError, match="no CPU"):
        nv.swiglu_backward_strided(gu[:, :64], gu, "split")
    assert not nv.nvfp4_supported("cpu")


def test_grouped_record_builders():
    """The group records the grouped linears hand to the kernel (pure torch, CPU)."""
    import torch

    from radiance_b200.nvfp4.grouped import align_offsets, groups_over_contraction, groups_over_rows

    offs = align_offsets(torch.tensor([5, 0, 130]))
    assert offs.tolist() == [0, 128, 128, 384]
    assert groups_over_rows(offs, 64, 320).tolist() == [
        [0, 0, 0, 128, 0, 320], [128, 64, 128, 0, 0, 320], [128, 128, 128, 256, 0, 320]]
    assert groups_over_contraction(offs, 256).tolist() == [
        [0, 0, 0, 256, 0, 128], [0, 0, 256, 256, 128, 0], [0, 0, 512, 256, 128, 256]]


def test_swiglu_gemm_contract_is_checked_on_the_host():
    """rb_nvfp4_gemm_swiglu refuses shapes and outputs it cannot serve before touching memory."""
    lib = _lib.load()
    buf = ctypes.c_void_p(256)
    # n = 192 is not a multiple of 128.
    rc = lib.rb_nvfp4_gemm_swiglu(buf, buf, buf, buf, 256, 192, 128, None, None, None, 0, buf, 192, buf, 96, buf,
                                  buf, None)
    assert rc in (1, 2) and lib.rb_nvfp4_last_error().decode()
    # h row stride shorter than n / 2.
    rc = lib.rb_nvfp4_gemm_swiglu(buf, buf, buf, buf, 256, 256, 128, None, None, None, 0, buf, 256, buf, 64, buf,
                                  buf, None)
    assert rc == 2 and "ldh" in lib.rb_nvfp4_last_error().decode()
    rc = lib.rb_nvfp4_gemm_swiglu(buf, buf, buf, buf, 256, 256, 128, None, None, None, 0, buf, 256, None, 128, buf,
                                  buf, None)
    assert rc == 2


def test_gate_up_interleave_round_trip():
    """The [32 gate | 32 up] row order the SwiGLU epilogue reads (CPU, pure torch)."""
    import torch

    import radiance_b200.nvfp4 as nv

    wg, wu = torch.randn(96, 8), torch.randn(96, 8)
    w = nv.interleave_gate_up(wg, wu)
    assert torch.equal(w[:32], wg[:32]) and torch.equal(w[32:64], wu[:32]) and torch.equal(w[64:96], wg[32:64])
    x = torch.randn(5, 8)
    g, u = nv.split_gate_up(x @ w.t())
    torch.testing.assert_close(g, x @ wg.t())
    torch.testing.assert_close(u, x @ wu.t())
    assert torch.equal(nv.merge_gate_up(g, u), x @ w.t())


def test_swiglu_silu_closed_forms_match_torch():
    """The SwiGLU epilogue takes silu(g), rounded to bf16, as bf16(g / 2) for |g| < 2^-9 and as g
    for g >= 128 (and +inf, NaN), reading a table only in between (rb_nvfp4_selftest_silu checks the
    whole mapping on the GPU).  Here the two closed forms are checked against torch's own bf16
    F.silu on the CPU for every bf16 bit pattern they cover."""
    import torch
    import torch.nn.functional as F

    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    g = bits.view(torch.bfloat16)
    gf = g.float()
    ref = F.silu(g)
    small = gf.abs() < 2.0 ** -9
    big = gf >= 128.0
    assert int(small.sum()) > 30000 and int(big.sum()) > 100
    half = (gf * 0.5).bfloat16()
    assert torch.equal(ref[small].view(torch.int16), half[small].view(torch.int16))
    assert torch.equal(ref[big].view(torch.int16), g[big].view(torch.int16))


def test_feedforward_module_construction_on_cpu():
    """FP4FeedForward.from_feedforward interleaves radiance's gate_proj / up_proj weights and biases
    and copies down_proj; the gate/up pair splits back unchanged; a CPU input is refused (there is no
    CPU path)."""
    import torch
    import torch.nn as nn

    import radiance_b200.nvfp4 as nv

    torch.manual_seed(0)
    src = nn.Module()
    src.gate_proj, src.up_proj, src.down_proj = nn.Linear(64, 96), nn.Linear(64, 96), nn.Linear(96, 64)
    ff = nv.FP4FeedForward.from_feedforward(src)
    assert ff.gate_up.weight.shape == (192, 64) and ff.gate_up.hidden_features == 96
    g, u = ff.gate_up.gate_up_weights()
    assert torch.equal(g, src.gate_proj.weight) and torch.equal(u, src.up_proj.weight)
    assert torch.equal(ff.gate_up.bias, nv.interleave_gate_up(src.gate_proj.bias, src.up_proj.bias))
    assert torch.equal(ff.down_proj.weight, src.down_proj.weight)
    # Without an sm_100 GPU the reference's actionable message comes first; with one, the CPU input.
    with pytest.raises(RuntimeError, match="needs NVFP4 support|no CPU path"):
        ff(torch.randn(128, 64))


def test_update_global_scale_contract_is_checked_on_the_host():
    lib = _lib.load()
    buf = ctypes.c_void_p(256)
    assert lib.rb_nvfp4_update_global_scale(buf, 7, buf, 0, 16, ctypes.c_float(1.0), buf, buf, None) == 2
    assert "dtypes" in lib.rb_nvfp4_last_error().decode()
    assert lib.rb_nvfp4_update_global_scale(None, 0, buf, 0, 16, ctypes.c_float(1.0), buf, buf, None) == 2
    assert lib.rb_nvfp4_update_global_scale(buf, 0, buf, 0, -1, ctypes.c_float(1.0), buf, buf, None) == 2


def test_wait_selftest_rejects_bad_arguments_on_the_host():
    lib = _lib.load()
    buf = ctypes.c_void_p(256)
    assert lib.rb_nvfp4_selftest_wait_timeout(2, 1000, buf, None) == 2
    assert lib.rb_nvfp4_selftest_wait_timeout(0, 0, buf, None) == 2
    assert lib.rb_nvfp4_selftest_wait_timeout(0, 1 << 40, buf, None) == 2
    assert "limit_cycles" in lib.rb_nvfp4_last_error().decode()


def test_strided_swiglu_contract_is_checked_on_the_host():
    """The strided SwiGLU entries refuse layouts they cannot serve before touching memory."""
    lib = _lib.load()
    gate, up, out = ctypes.c_void_p(4096), ctypes.c_void_p(4096 + 2 * 64), ctypes.c_void_p(1 << 20)
    ws = ctypes.c_void_p(256)
    # null workspace
    assert lib.rb_nvfp4_swiglu_forward_strided(gate, up, 128, 32, 16, 64, out, 64, ws, None, None) == 2
    # hidden not a multiple of 32
    assert lib.rb_nvfp4_swiglu_forward_strided(gate, up, 128, 32, 16, 48, out, 64, ws, ws, None) == 1
    # row stride shorter than the split layout's 2 * hidden
    assert lib.rb_nvfp4_swiglu_forward_strided(gate, up, 96, 32, 16, 64, out, 64, ws, ws, None) == 1
    assert "row strides" in lib.rb_nvfp4_last_error().decode()
    # up below gate
    assert lib.rb_nvfp4_swiglu_forward_strided(up, gate, 128, 32, 16, 64, out, 64, ws, ws, None) == 1
    # misaligned gradient output
    bad = ctypes.c_void_p((1 << 20) + 2)
    assert lib.rb_nvfp4_swiglu_backward_strided(out, 64, gate, up, 128, 32, 16, 64, bad, ctypes.c_void_p((1 << 20) + 128),
                                                128, 32, ws, ws, None) == 2
    assert "aligned" in lib.rb_nvfp4_last_error().decode()
