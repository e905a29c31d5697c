"""GPTQLinear -- the int-weight linear layer GPTQ produces (gptq.py:257-325).

Only the layer (storage, ``pack``, ``forward``) is on the hot path; the GPTQ
algorithm itself (Hessian accumulation and the column-by-column solve,
gptq.py:1-256, 327-) is not part of this package.

Buffers match the reference (``weight_int`` int8 [out, in], ``scale`` /
``zero_point`` [out, n_groups] or [out, 1]), so state_dicts are
interchangeable.  ``forward`` computes exactly the reference's fp32
dequantize + ``F.linear`` for fp32 activations; fp16 / bf16 activations
(which the reference rejects: its dequantized weight is fp32) of a layer with
at most 4-bit codes and groups that are multiples of 64 run the fused W4A16
tensor-core kernel, with the same packed operand cache as QuantizedLinear.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .core.quantizer import int_linear_forward, int_weight_fp32, row_group_quantize


class GPTQLinear(nn.Module):
    """A linear layer whose weights are quantized via GPTQ (gptq.py:257-325)."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        n_bits: int = 4,
        symmetric: bool = True,
        group_size: int = 128,
        bias: bool = True,
    ):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.n_bits = n_bits
        self.symmetric = symmetric
        self.group_size = group_size

        self.register_buffer("weight_int", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(out_features, 1))
        self.register_buffer("zero_point", torch.zeros(out_features, 1))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None
        self._w4 = None  # (act_dtype, device, packed operand) for the W4A16 kernel

    @torch.no_grad()
    def pack(self, w_q: torch.Tensor, weight_orig: torch.Tensor) -> None:
        """Keep GPTQ's integer codes ``w_q`` as int8 and take the scale / zero
        point from the weight they were solved for (gptq.py:285-299): one
        qparams-only pass of the row-group kernel over ``weight_orig``, groups
        of ``group_size`` columns (one per row when group_size <= 0)."""
        row_group_quantize(self, weight_orig, self.symmetric, "GPTQLinear.pack", codes=False)
        self.weight_int.copy_(w_q.to(torch.int8).reshape_as(self.weight_int))

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        self._w4 = None
        for name in ("scale", "zero_point"):  # the reference rebinds these in pack
            k = prefix + name
            if k in state_dict and getattr(self, name).shape != state_dict[k].shape:
                setattr(self, name, torch.empty_like(state_dict[k], device=getattr(self, name).device))
        return super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def _apply(self, fn, *args, **kwargs):
        self._w4 = None
        return super()._apply(fn, *args, **kwargs)

    def dequantized_weight(self) -> torch.Tensor:
        """The fp32 weight the reference's forward builds (gptq.py:302-314)."""
        return int_weight_fp32(self, "GPTQLinear")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return int_linear_forward(self, x)

    def extra_repr(self) -> str:
        return (
            f"in={self.in_features}, out={self.out_features}, "
            f"bits={self.n_bits}, group={self.group_size}"
        )
