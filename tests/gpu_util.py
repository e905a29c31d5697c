"""Helpers shared by the GPU parity tests (tensor <-> oracle conversions)."""

import numpy as np
import torch

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
NAME = {v: k for k, v in TORCH_DT.items()}


def to_dev(arr: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    """float32-held values (or integer arrays) -> CUDA tensor of `dtype`."""
    # np.array (not ascontiguousarray) keeps 0-dim arrays 0-dim: torch type
    # promotion treats 0-dim tensors differently from [1]-shaped ones
    if dtype in TORCH_DT:
        return torch.from_numpy(np.array(arr, dtype=np.float32, copy=True)).to(device).to(TORCH_DT[dtype])
    return torch.from_numpy(np.array(arr, copy=True)).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        t = t.float()
    return t.numpy()


def seeded(shape, seed, scale=1.0, outliers=0, factor=20.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g) * scale
    if outliers:
        idx = torch.randperm(shape[-1], generator=g)[:outliers]
        x[..., idx] *= factor
    return x
