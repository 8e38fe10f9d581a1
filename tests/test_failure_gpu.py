"""Failure detection on the GPU without a fault: a device-side wait that runs out.

Every wait in the library's kernels (TMA data, MMA completion, the accumulator hand-off, a free
pipeline stage) is bounded; when one runs out the kernel records a status code and returns, so the
context stays usable and the host learns of it through ``rb_nvfp4_device_status``.  This test makes
such a wait run out on purpose: a self-test kernel waits, with the library's own bounded wait and a
test-only limit of a few milliseconds, on an mbarrier that nothing ever arrives on.  Nothing (no TMA
copy, no MMA, no TMEM allocation) is in flight when it gives up.  The status must read back, clear,
and the next quantize and GEMM launches must run and match the oracle.
"""

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests._nvfp4_helpers import to_numpy_f32, u8

pytestmark = pytest.mark.gpu

LIMIT = 4_000_000  # cycles, about 2 ms at the B200's clock (the production limit is about 1 s)


@pytest.mark.parametrize("which,code", [(0, 1), (1, 2)])
def test_a_wait_that_runs_out_reports_and_the_next_launch_is_clean(which, code):
    import radiance_b200.nvfp4 as nv
    from radiance_b200 import _lib

    assert nv.nvfp4_supported()
    lib = _lib.load()
    assert _lib.device_status(clear=True) == 0, "a status was left set before this test"
    waited = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.rb_nvfp4_selftest_wait_timeout(which, LIMIT, waited.data_ptr(), stream) == 0, \
        lib.rb_nvfp4_last_error()
    assert _lib.device_status(clear=False) == code
    assert int(waited.item()) & 0xFFFFFFFF >= LIMIT  # it really waited the limit out
    assert _lib.device_status(clear=True) == code
    assert _lib.device_status(clear=True) == 0

    # The context is intact: the next launches run and are exact.
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(384, 512, device="cuda") * 0.02).bfloat16()
    a, b = nv.quantize(x, -1), nv.quantize(w, -1)
    y = nv.mm(a, b, out_dtype=torch.float32)
    xn, wn = to_numpy_f32(x), to_numpy_f32(w)
    gx, gw = O.global_scale_of(xn), O.global_scale_of(wn)
    px, sx = O.quantize_rowblock(xn, gx)
    pw, sw = O.quantize_rowblock(wn, gw)
    assert np.array_equal(u8(a.packed), px) and np.array_equal(u8(b.packed), pw)
    ref = O.dequantize(px, sx, gx).astype(np.float64) @ O.dequantize(pw, sw, gw).astype(np.float64).T
    err = np.abs(y.double().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 1e-5
    assert _lib.device_status(clear=True) == 0
