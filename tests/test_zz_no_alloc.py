"""rb_nvfp4_global_scale_noalloc: the global scale for callers that cannot allocate device memory.

Some callers of this library cannot allocate on the call path -- code running where device
allocation is not allowed, plugin hosts that only receive pre-planned buffers, plain C/FFI callers
without an allocator.  For them the library offers a global-scale entry point that needs no
workspace: its scratch is a fixed array inside the library.  This test calls it through the C ABI
twice in a row (the scratch keeps the previous call's contents, so the second call checks that
nothing leaks between calls) and compares each result with the workspace-taking entry point's.
Both compute the exact maximum, so the comparison is bit-exact.  The file name makes pytest
collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(fn, x, out, *extra):
    stream = torch.cuda.current_stream().cuda_stream
    dtype = 0 if x.dtype == torch.bfloat16 else 1
    return fn(x.data_ptr(), dtype, x.shape[0], x.shape[1], x.stride(0), out.data_ptr(), *extra, stream)


def test_noalloc_global_scale_matches_workspace_version_twice():
    from radiance_b200 import _lib

    lib = _lib.load()
    ws = torch.zeros(2, dtype=torch.int32, device="cuda")
    cases = [
        torch.randn(4096, 6144, device="cuda").bfloat16() * 3.0,  # several hundred blocks
        torch.randn(300, 257, device="cuda") * 1e-3,  # fp32, ragged tail, one block
    ]
    for x in cases:
        got = torch.full((), -1.0, device="cuda")
        want = torch.full((), -2.0, device="cuda")
        assert _call(lib.rb_nvfp4_global_scale_noalloc, x, got) == 0, lib.rb_nvfp4_last_error()
        assert _call(lib.rb_nvfp4_global_scale, x, want, ws.data_ptr()) == 0, lib.rb_nvfp4_last_error()
        torch.cuda.synchronize()
        assert np.float32(got.item()).view(np.uint32) == np.float32(want.item()).view(np.uint32)
        assert got.item() == max(x.abs().max().float().item() / 2688.0, 1e-12) or abs(
            got.item() / (x.abs().max().float().item() / 2688.0) - 1
        ) < 1e-6
    strided = cases[0][:, 1024:3072]  # non-contiguous rows take the indexed path
    got, want = torch.empty((), device="cuda"), torch.empty((), device="cuda")
    assert _call(lib.rb_nvfp4_global_scale_noalloc, strided, got) == 0
    assert _call(lib.rb_nvfp4_global_scale, strided, want, ws.data_ptr()) == 0
    torch.cuda.synchronize()
    assert got.item() == want.item()


def test_noalloc_rejects_inputs_beyond_its_scratch():
    from radiance_b200 import _lib

    lib = _lib.load()
    buf = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    rc = lib.rb_nvfp4_global_scale_noalloc(buf, 0, 1 << 16, (1 << 15) + 64, (1 << 15) + 64, buf, None)
    assert rc == 1
    assert "exceed its limit" in lib.rb_nvfp4_last_error().decode()
