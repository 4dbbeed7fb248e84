"""Conversions between the oracle's numpy storage form and torch tensors."""

from __future__ import annotations

import numpy as np
import torch


def to_torch(a: np.ndarray, dtype: str, device) -> torch.Tensor:
    """numpy storage form (bf16 as uint16 bits) -> torch tensor on ``device``."""
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """torch tensor -> numpy storage form (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
