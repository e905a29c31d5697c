"""W4A16 dispatch for QuantizedLinear.forward (filled in with the tensor-core kernel)."""

import torch


def eligible(ql, x: torch.Tensor) -> bool:
    return False


def linear(ql, x: torch.Tensor) -> torch.Tensor:
    raise NotImplementedError
