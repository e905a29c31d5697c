"""SpQRLinear -- int weights plus sparse fp outliers (spqr.py:102-208).

Only the layer (storage, ``pack``, ``forward``, ``sparsity``) is on the hot
path; the SpQR sensitivity / outlier-selection algorithm (spqr.py:1-100,
210-) is not part of this package.

Buffers match the reference (``weight_int``, ``scale``, ``zero_point``,
``outlier_mask`` bool [out, in], ``outlier_vals`` 1-D in mask order).
``forward`` computes exactly the reference's fp32 dequantize, outlier
restore and ``F.linear`` for fp32 activations.  fp16 / bf16 activations (which
the reference rejects) of a layer with at most 4-bit codes and groups that
are multiples of 64 run the fused W4A16 kernel on the int part, then add the
outliers' contribution with a sparse row kernel (``lq_sparse_row_add``): the
correction at a masked (n, k) is the outlier minus the dequantized int
weight there (zero, since pack quantizes the zeroed outliers
symmetrically), kept as CSR over the rows holding outliers and rebuilt when
the mask, the values or the int weight change.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _C
from .core.quantizer import int_weight_fp32, row_group_quantize


class SpQRLinear(nn.Module):
    """Hybrid sparse-FP + quantized-INT linear layer (spqr.py:102-208)."""

    def __init__(self, in_features: int, out_features: int,
                 n_bits: int = 4, group_size: int = 128, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.n_bits = n_bits
        self.group_size = group_size
        self.symmetric = True  # pack() quantizes symmetrically (spqr.py:146)

        self.register_buffer("weight_int", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(out_features, 1))
        self.register_buffer("zero_point", torch.zeros(out_features, 1))
        self.register_buffer("outlier_mask", torch.zeros(out_features, in_features, dtype=torch.bool))
        self.register_buffer("outlier_vals", torch.zeros(0))

        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None
        self._w4 = None    # packed W4A16 operand of the int part
        self._csr = None   # (key, row_ptr, row_ids, cols, vals) of the outlier correction

    @torch.no_grad()
    def pack(self, weight: torch.Tensor, outlier_mask: torch.Tensor) -> None:
        """Split the weight into fp outliers and a symmetric int part
        (spqr.py:128-170).  ``outlier_vals`` takes the masked weights in
        row-major mask order; the int part is the weight with those positions
        set to zero, quantized (qparams and int8 codes) by one pass of the
        row-group kernel."""
        self.outlier_mask.copy_(outlier_mask)
        self.outlier_vals = weight[outlier_mask].clone()
        inliers = torch.where(outlier_mask, torch.zeros((), dtype=weight.dtype, device=weight.device),
                              weight)
        row_group_quantize(self, inliers, True, "SpQRLinear.pack")
        self._csr = None

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        self._w4 = None
        self._csr = None
        for name in ("scale", "zero_point", "outlier_vals"):  # rebound by pack in the reference
            k = prefix + name
            if k in state_dict and getattr(self, name).shape != state_dict[k].shape:
                setattr(self, name, torch.empty_like(state_dict[k], device=getattr(self, name).device))
        return super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def _apply(self, fn, *args, **kwargs):
        self._w4 = None
        self._csr = None
        return super()._apply(fn, *args, **kwargs)

    def dequantized_weight(self) -> torch.Tensor:
        """The fp32 weight the reference's forward builds: int part, then the
        outliers written over the masked positions (spqr.py:172-193)."""
        w = int_weight_fp32(self, "SpQRLinear")
        w[self.outlier_mask] = self.outlier_vals.to(w.dtype)
        return w

    def _outlier_csr(self):
        ts = (self.outlier_mask, self.outlier_vals, self.weight_int, self.scale, self.zero_point)
        key = tuple((t.data_ptr(), t._version) for t in ts)
        if self._csr is not None and self._csr[0] == key:
            return self._csr[1:]
        idx = self.outlier_mask.nonzero()  # row-major: the order of outlier_vals
        rows, cols = idx[:, 0], idx[:, 1]
        deq = int_weight_fp32(self, "SpQRLinear")[rows, cols]
        vals = (self.outlier_vals.float() - deq).contiguous()
        row_ids, counts = torch.unique_consecutive(rows, return_counts=True)
        row_ptr = torch.zeros(row_ids.numel() + 1, dtype=torch.int32, device=rows.device)
        row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
        csr = (row_ptr, row_ids.to(torch.int32).contiguous(), cols.to(torch.int32).contiguous(), vals)
        self._csr = (key,) + csr
        return csr

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .core import w4a16
        if w4a16.eligible(self, x):
            y = w4a16.linear(self, x)
            row_ptr, row_ids, cols, vals = self._outlier_csr()
            if row_ids.numel():
                x2 = x.reshape(-1, self.in_features).contiguous()
                _C.call("lq_sparse_row_add", x2.data_ptr(), _C.dt(x2), x2.shape[0], self.in_features,
                        self.out_features, row_ptr.data_ptr(), row_ids.data_ptr(), row_ids.numel(),
                        cols.data_ptr(), vals.data_ptr(), y.data_ptr(), _C.stream_ptr(x2))
            return y
        return F.linear(x, self.dequantized_weight(), self.bias)

    @property
    def sparsity(self) -> float:
        """Fraction of weights stored as FP outliers (spqr.py:199-202)."""
        return self.outlier_mask.float().mean().item()

    def extra_repr(self) -> str:
        return (
            f"in={self.in_features}, out={self.out_features}, "
            f"bits={self.n_bits}, group={self.group_size}, "
            f"outliers={self.sparsity:.2%}"
        )
