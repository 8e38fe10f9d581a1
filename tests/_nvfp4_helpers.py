"""Test-side helpers: torch <-> numpy conversions and a GPU dequantizer for statistics.

Test infrastructure only (the product path never imports ``tests/``)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import nvfp4_oracle as O


def to_numpy_f32(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().numpy()


def from_golden(golden, name: str, device="cuda") -> torch.Tensor:
    raw = golden[f"{name}/x"]
    if int(golden[f"{name}/dtype"]) == 0:
        t = torch.from_numpy(raw.view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(raw.astype(np.float32))
    return t.to(device)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy()


_E4M3 = None
_FP4 = None


def dequantize_gpu(packed: torch.Tensor, scale_flat: torch.Tensor, gs: torch.Tensor, rows: int, cols: int):
    """Packed codes + swizzled scale bytes -> fp32 (rows, cols), on the GPU (test statistics only)."""
    global _E4M3, _FP4
    dev = packed.device
    if _E4M3 is None or _E4M3.device != dev:
        _E4M3 = torch.from_numpy(O.E4M3_VALUES.astype(np.float32)).to(dev)
        _FP4 = torch.tensor(O.FP4_VALUES, dtype=torch.float32, device=dev)
    raw = packed.view(torch.uint8)
    code = torch.stack([raw & 0xF, raw >> 4], dim=-1).reshape(rows, cols)
    mag = _FP4[(code & 7).long()]
    val = torch.where(code >= 8, -mag, mag)
    nct = (cols // 16 + 3) // 4
    r = torch.arange(rows, device=dev).view(-1, 1)
    c = torch.arange(cols // 16, device=dev).view(1, -1)
    off = ((r // 128) * nct + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)
    s = _E4M3[scale_flat.view(torch.uint8)[off].long()] * gs.float()
    return (val.view(rows, cols // 16, 16) * s.unsqueeze(-1)).view(rows, cols)
