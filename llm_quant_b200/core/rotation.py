"""llm_quant_b200.core.rotation -- the Hadamard part of llm_quant.core.rotation.

``fast_hadamard_transform`` is the reference's hot-path rotation
(core/rotation.py:130-147).  The reference multiplies by the dense
normalised Sylvester matrix (O(d^2) per row); here the same product is a
butterfly in registers / shared memory on the GPU (O(d log d)), scaled once
by the matrix entry round_dtype(1/sqrt(d)).  Results agree with the
reference to float rounding of the summation order (fp32: 1e-5; half
types: 1e-2 relative).
"""

from __future__ import annotations

import math

import torch

from .. import _C


def hadamard_matrix(n: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Sylvester-construction normalised Hadamard matrix of size *n*
    (core/rotation.py:30-43).  A constant built on the CPU, as in the
    reference; entries are ``+-1 / sqrt(n)`` rounded to ``dtype``."""
    assert n > 0 and (n & (n - 1)) == 0, "n must be a power of 2"
    k = n.bit_length() - 1
    idx = torch.arange(n)
    # H[i, j] = (-1)^popcount(i & j)
    par = torch.zeros(n, n, dtype=torch.int64)
    ij = idx[:, None] & idx[None, :]
    for b in range(k):
        par ^= (ij >> b) & 1
    H = (1 - 2 * par).to(dtype)
    return H / math.sqrt(n)


def _fht(x: torch.Tensor, n_bits=None, symmetric=True, want_qparams=False):
    d = x.shape[-1]
    assert d > 0 and (d & (d - 1)) == 0, "last dim must be power of 2"
    _C.require_cuda(x, what="fast_hadamard_transform")
    _C.require_float(x, "fast_hadamard_transform")
    xc = x.detach().contiguous()
    out = torch.empty_like(xc)
    rows = xc.numel() // d if d else 0
    if n_bits is None:
        _C.call("lq_hadamard", xc.data_ptr(), _C.dt(xc), rows, d, out.data_ptr(), _C.stream_ptr(xc))
        return out
    _C.check_clamp_bounds(xc.dtype, n_bits, symmetric)
    s = z = None
    if want_qparams:
        s = torch.empty(rows, 1, dtype=xc.dtype, device=xc.device)
        z = torch.empty_like(s)
    _C.call("lq_hadamard_fake_quant", xc.data_ptr(), _C.dt(xc), rows, d, n_bits, int(symmetric),
            out.data_ptr(), _C.ptr(s), _C.ptr(z), _C.stream_ptr(xc))
    return (out, s, z) if want_qparams else out


def fast_hadamard_transform(x: torch.Tensor, normalize: bool = True) -> torch.Tensor:
    """``x @ hadamard_matrix(d, x.dtype)`` along the last dim (core/rotation.py:130-147).

    Like the reference, the output is always normalised (``normalize`` is
    accepted and ignored)."""
    return _fht(x)


def hadamard_fake_quantize(x: torch.Tensor, n_bits: int = 4, symmetric: bool = True,
                           return_qparams: bool = False):
    """Fused QuaRot activation path: ``fake_quantize(fast_hadamard_transform(x),
    n_bits, symmetric, QScheme.PER_CHANNEL)`` for a 2-D x (quarot.py:168-170
    followed by core/quantizer.py:143-185), in one pass over HBM.  The
    transform is rounded to x's dtype before quantization, as the two
    reference calls would; each row of the [rows, d] view is one channel.

    Not part of the reference's API (it has no fused op); values equal the
    two-call composition applied to this module's transform."""
    return _fht(x, n_bits, symmetric, return_qparams)
