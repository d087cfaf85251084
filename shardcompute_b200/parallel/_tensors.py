"""Host-side tensor plumbing for the layer API: every weight the layers hold
is a CUDA tensor (no CPU path); numpy arrays and CPU tensors are uploaded."""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch


def _device(device: Optional[torch.device]) -> torch.device:
    if device is not None:
        return device
    if not torch.cuda.is_available():
        raise RuntimeError("shardcompute_b200 layers need a CUDA device (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def as_device(a, dtype: torch.dtype, device: Optional[torch.device] = None) -> torch.Tensor:
    dev = _device(device if device is not None else (a.device if isinstance(a, torch.Tensor) and a.is_cuda else None))
    if isinstance(a, torch.Tensor):
        return a.to(device=dev, dtype=dtype).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def as_words(a, device: Optional[torch.device] = None) -> torch.Tensor:
    """Packed uint32 codes as int32 storage (same bytes) on the device."""
    if isinstance(a, torch.Tensor):
        if a.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
            raise ValueError(f"packed weights must be 32-bit integers, got {a.dtype}")
        dev = _device(device if device is not None else (a.device if a.is_cuda else None))
        return a.view(torch.int32).to(dev).contiguous()
    arr = np.ascontiguousarray(a)
    if arr.dtype not in (np.uint32, np.int32):
        raise ValueError(f"packed weights must be uint32, got {arr.dtype}")
    return torch.from_numpy(arr.view(np.int32)).to(_device(device))
