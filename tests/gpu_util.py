"""Host<->device helpers for the GPU parity tests (torch is used only for device memory)."""
from __future__ import annotations

import numpy as np


def dev(a: np.ndarray, kind: str, oracle):
    """Uploads an fp32 array as kind 'f32' | 'bf16' | 'f16' (16-bit: RNE-quantised by the oracle codec)."""
    import torch

    a = np.ascontiguousarray(a, np.float32)
    if kind == "f32":
        return torch.from_numpy(a.copy()).cuda()
    bits = oracle.to_bf16(a) if kind == "bf16" else oracle.to_f16(a)
    t = torch.from_numpy(bits.view(np.int16).copy()).cuda()
    return t.view(torch.bfloat16 if kind == "bf16" else torch.float16)


def quantize(a: np.ndarray, kind: str, oracle) -> np.ndarray:
    """The fp32 values the device sees after upload as `kind`."""
    a = np.ascontiguousarray(a, np.float32)
    if kind == "f32":
        return a
    if kind == "bf16":
        return oracle.from_bf16(oracle.to_bf16(a))
    return oracle.from_f16(oracle.to_f16(a))


def host(t, oracle) -> np.ndarray:
    """Downloads a device tensor as fp32."""
    import torch

    t = t.contiguous()
    if t.dtype == torch.float32:
        return t.cpu().numpy()
    bits = t.view(torch.int16).cpu().numpy().view(np.uint16)
    return oracle.from_bf16(bits) if t.dtype == torch.bfloat16 else oracle.from_f16(bits)


def bits(t) -> np.ndarray:
    """Raw 16-bit patterns of a bf16/fp16 device tensor."""
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
