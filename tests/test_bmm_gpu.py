"""Batched NVFP4 GEMM (``nvfp4.bmm``, grouped tcgen05 launches) against the oracle: each batch
entry's product equals the float64 product of its dequantized operands, to the GEMM tolerance
(fp32 output: max relative error 1e-3; bf16 output: one bf16 ulp).  Covers more batch entries than
one launch takes (256), and the shape checks."""

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


def _deq(t):
    p, s = u8(t.packed), u8(t.scale)
    k = p.shape[1] * 2
    return O.dequantize(p, O.from_blocked(s, p.shape[0], k // 16), np.float32(t.global_scale.item())).astype(np.float64)


@pytest.mark.parametrize("batch,m,n,k", [(3, 256, 384, 320), (2, 128, 128, 64), (300, 128, 128, 64)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_bmm_matches_oracle(nv, batch, m, n, k, out_dtype):
    torch.manual_seed(batch + m + n + k)
    q = torch.randn(batch * m, k, device="cuda", dtype=torch.bfloat16)
    kk = (torch.randn(batch * n, k, device="cuda") * 0.5).bfloat16()
    a, b = nv.quantize(q, -1), nv.quantize(kk, -1)
    got = nv.bmm(a, b, batch, out_dtype=out_dtype)
    assert got.shape == (batch, m, n) and got.dtype == out_dtype
    da, db = _deq(a), _deq(b)
    g = got.double().cpu().numpy()
    for i in range(0, batch, max(1, batch // 7)):
        ref = da[i * m:(i + 1) * m] @ db[i * n:(i + 1) * n].T
        scale = np.abs(ref).max()
        if out_dtype == torch.bfloat16:
            assert (np.abs(g[i] - ref) <= np.abs(ref) * 2.0**-8 + 1e-6 * scale).all(), i
        else:
            assert np.abs(g[i] - ref).max() / scale <= 1e-3, i
    from radiance_b200 import _lib

    assert _lib.device_status(clear=True) == 0


def test_bmm_rejects_bad_shapes(nv):
    a = nv.quantize(torch.randn(256, 128, device="cuda", dtype=torch.bfloat16), -1)
    b = nv.quantize(torch.randn(384, 128, device="cuda", dtype=torch.bfloat16), -1)
    with pytest.raises(ValueError):
        nv.bmm(a, b, 3)  # 256 rows do not split into 3 entries
    with pytest.raises(ValueError):
        nv.bmm(a, b, 2)  # N = 192 is not a multiple of 128
