"""Helpers for the GPU parity tests: numpy (oracle layout) <-> CUDA tensors."""

from __future__ import annotations

import numpy as np
import pytest
import torch

requires_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")

TORCH_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16,
                "f64": torch.float64}


def to_device(values: np.ndarray, dtype: str, device: str = "cuda:0") -> torch.Tensor:
    """Oracle-layout values (bf16 as uint16 bits) -> CUDA tensor of that dtype, same bits."""
    arr = np.ascontiguousarray(values)
    if dtype == "bf16":
        return torch.from_numpy(arr.astype(np.uint16).view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(arr).to(device)


def masks_to_device(words: np.ndarray, device: str = "cuda:0") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(words, dtype=np.uint32).view(np.int32)).to(device)


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()
