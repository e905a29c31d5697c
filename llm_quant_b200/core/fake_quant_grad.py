"""Backward of fake_quantize (the reference's autograd gradient) on the GPU."""

from __future__ import annotations

import torch

from .. import _C


def fake_quantize_backward(x: torch.Tensor, grad_out: torch.Tensor, n_bits: int,
                           symmetric: bool, scheme: str, group_size: int) -> torch.Tensor:
    """grad_x of ``fake_quantize(x, n_bits, symmetric, scheme, group_size)``."""
    xc = x.detach().contiguous()
    g = grad_out.detach().to(xc.dtype).contiguous()
    dx = torch.empty_like(xc)
    if scheme == "per_group":
        rows, cols = xc.shape
        group = group_size
    elif scheme == "per_channel":
        rows = xc.shape[0]
        cols = xc.numel() // max(1, rows)
        group = max(1, cols)
    else:
        rows, cols = 1, xc.numel()
        group = max(1, cols)
    _C.call("lq_fake_quant_backward", xc.data_ptr(), g.data_ptr(), _C.dt(xc), rows, cols, group,
            n_bits, int(symmetric), dx.data_ptr(), _C.stream_ptr(xc))
    return dx
