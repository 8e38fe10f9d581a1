"""The fused global-scale quantizer (``rb_nvfp4_quantize_auto_scale``): amax, global scale and
quantization in one cooperative launch.  It must give exactly what ``global_scale_of`` followed by
the quantizer gives -- the same global-scale bits and the same codes and scale bytes -- in every
form, for both input types, with and without the rotation and stochastic rounding, on ragged and
full-size shapes; leave its 16-byte workspace ready for the next call (calls in a row, and replays of
a captured CUDA graph); and the global scale must equal the oracle's."""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import to_numpy_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nv():
    import radiance_b200.nvfp4 as nv

    assert nv.nvfp4_supported()
    return nv


def _bufs(nv, m, k):
    row = (torch.empty(m, k // 2, dtype=torch.uint8, device="cuda"),
           torch.empty(nv.row_scale_bytes(m, k), dtype=torch.uint8, device="cuda"))
    col = (torch.empty(k, m // 2, dtype=torch.uint8, device="cuda"),
           torch.empty(nv.col_scale_bytes(m, k), dtype=torch.uint8, device="cuda"))
    return row, col


SHAPES = [(128, 64), (256, 192), (1024, 1280), (2048, 2048), (4096, 5632), (16384, 2048)]


@pytest.mark.parametrize("m,k", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("form", ["row", "col", "both"])
def test_auto_scale_equals_amax_then_quantize(nv, m, k, dtype, form):
    torch.manual_seed(m + k)
    x = (torch.randn(m, k, device="cuda") * 3.0).to(dtype)
    x[m // 3, k // 5] = 77.0  # the maximum sits in one CTA's slice only
    had = nv.hadamard_matrix(device="cuda")
    for rot, sr in ((None, False), (had, False), (had, True)):
        if form == "row" and rot is not None:
            continue
        seed = torch.tensor(11, device="cuda", dtype=torch.int64)
        want_gs = nv.global_scale_of(x)
        want_r, want_c = _bufs(nv, m, k)
        got_r, got_c = _bufs(nv, m, k)
        kw = dict(hadamard=rot, stochastic=sr, seed=seed)

        def pick(r, c):
            return dict(row=r if form in ("row", "both") else None, col=c if form in ("col", "both") else None)

        nv.quantize_into_(x, global_scale=want_gs, **pick(want_r, want_c), **kw)
        got_gs = torch.full((), -1.0, device="cuda")
        for _ in range(2):  # twice: the workspace must come back ready
            nv.quantize_auto_scale_into_(x, out_scale=got_gs, **pick(got_r, got_c), **kw)
            torch.cuda.synchronize()
            assert got_gs.view(torch.int32).item() == want_gs.view(torch.int32).item()
            if form in ("row", "both"):
                assert torch.equal(got_r[0], want_r[0]) and torch.equal(got_r[1], want_r[1])
            if form in ("col", "both"):
                assert torch.equal(got_c[0], want_c[0]) and torch.equal(got_c[1], want_c[1])
    from radiance_b200 import _lib

    assert _lib.device_status() == 0


def test_auto_scale_global_scale_matches_oracle_and_edge_values(nv):
    for fill in (0.0, 1e-30):
        x = torch.full((256, 128), fill, device="cuda", dtype=torch.float32)
        gs = torch.empty((), device="cuda")
        nv.quantize_auto_scale_into_(x, out_scale=gs, row=_bufs(nv, 256, 128)[0])
        assert gs.view(torch.int32).item() == nv.global_scale_of(x).view(torch.int32).item()
    x = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16) * 1e-3
    gs = torch.empty((), device="cuda")
    nv.quantize_auto_scale_into_(x, out_scale=gs, col=_bufs(nv, 1024, 512)[1])
    want = O.global_scale_of(to_numpy_f32(x))
    assert np.float32(gs.item()).view(np.uint32) == np.float32(want).view(np.uint32)


def test_auto_scale_in_a_cuda_graph(nv):
    """The cooperative launch captured in a graph and replayed: each replay recomputes the scale of
    the current input contents."""
    m, k = 2048, 1024
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    gs = torch.empty((), device="cuda")
    row, col = _bufs(nv, m, k)
    had = nv.hadamard_matrix(device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        nv.quantize_auto_scale_into_(x, out_scale=gs, row=row, col=col, hadamard=had)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        nv.quantize_auto_scale_into_(x, out_scale=gs, row=row, col=col, hadamard=had)
    for scale in (1.0, 5.0, 0.25):
        x.copy_(torch.randn(m, k, device="cuda") * scale)
        g.replay()
        torch.cuda.synchronize()
        want_r, want_c = _bufs(nv, m, k)
        want_gs = nv.global_scale_of(x)
        nv.quantize_into_(x, global_scale=want_gs, row=want_r, col=want_c, hadamard=had)
        assert gs.view(torch.int32).item() == want_gs.view(torch.int32).item()
        assert torch.equal(row[0], want_r[0]) and torch.equal(col[0], want_c[0]) and torch.equal(col[1], want_c[1])


def test_first_call_on_a_new_thread(nv):
    """A thread whose first call into the library encodes a tensor map (autograd runs backward on
    its own thread) gets the device's context bound by the library itself."""
    import threading

    x = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    want = nv.quantize(x, -1, global_scale=nv.global_scale_of(x))
    out = {}

    def work():
        try:
            out["q"] = nv.quantize(x, -1)
            torch.cuda.synchronize()
        except Exception as e:  # reported below
            out["err"] = e

    t = threading.Thread(target=work)
    t.start()
    t.join(timeout=120)
    assert "err" not in out, out.get("err")
    assert torch.equal(out["q"].packed.view(torch.uint8), want.packed.view(torch.uint8))
