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


# ──────────────────────────────────────────────────────────────────────────────
# Rotation construction and weight-rotation helpers (core/rotation.py:46-207).
# One-off weight preparation for QuaRot / SpinQuant / FlatQuant, off the
# data-parallel hot path: plain eager PyTorch on the inputs' device (CPU
# included), with the reference's names, signatures, defaults and results.
# ──────────────────────────────────────────────────────────────────────────────

def _gen_device(generator):
    return None if generator is None else generator.device


def random_hadamard_matrix(n: int, dtype: torch.dtype = torch.float32,
                           generator: torch.Generator | None = None) -> torch.Tensor:
    """``hadamard_matrix(n) @ diag(s)`` with s_j = +-1 drawn by
    ``torch.randint(0, 2, (n,))`` from ``generator`` (core/rotation.py:46-55):
    column j of the normalised Sylvester matrix is negated when its draw is 0.
    The draw runs on the generator's device, so a seeded CPU generator gives
    the reference's signs wherever the matrix is placed."""
    H = hadamard_matrix(n, dtype)
    draw = torch.randint(0, 2, (n,), generator=generator, dtype=dtype,
                         device=_gen_device(generator))
    return H * (draw.to(H.device) * 2 - 1)


def random_orthogonal(n: int, dtype: torch.dtype = torch.float32,
                      generator: torch.Generator | None = None) -> torch.Tensor:
    """Haar-distributed orthogonal matrix (core/rotation.py:58-66): the Q of
    a QR factorisation of an n x n standard normal matrix, its columns
    signed so that R's diagonal would be non-negative (a zero diagonal entry
    keeps its column)."""
    g = torch.randn(n, n, dtype=dtype, generator=generator, device=_gen_device(generator))
    q, r = torch.linalg.qr(g)
    sign = torch.diagonal(r).sign()
    sign = torch.where(sign == 0, torch.ones_like(sign), sign)
    return q * sign


def cayley_transform(A: torch.Tensor) -> torch.Tensor:
    """Orthogonal ``(I + A)^-1 (I - A)`` of a skew-symmetric A
    (core/rotation.py:73-81), by one linear solve; the two factors commute
    because both are polynomials in A."""
    eye = torch.eye(A.shape[0], dtype=A.dtype, device=A.device)
    return torch.linalg.solve(eye + A, eye - A)


class CayleyRotation(torch.nn.Module):
    """Learnable rotation Q = cayley_transform(A) (core/rotation.py:84-123).

    The free parameters ``params`` (dim (dim - 1) / 2 of them, zero at
    construction, so Q starts at the identity for either ``init``) fill the
    strict upper triangle of A row by row; A = U - U^T is skew-symmetric and
    Q is orthogonal for every value of the parameters."""

    def __init__(self, dim: int, init: str = "identity"):
        super().__init__()
        self.dim = dim
        self.init = init
        self.params = torch.nn.Parameter(torch.zeros(dim * (dim - 1) // 2))

    def _build_skew(self) -> torch.Tensor:
        rows, cols = torch.triu_indices(self.dim, self.dim, offset=1, device=self.params.device)
        upper = torch.zeros(self.dim, self.dim, dtype=self.params.dtype, device=self.params.device)
        upper = upper.index_put((rows, cols), self.params)
        return upper - upper.t()

    def forward(self) -> torch.Tensor:
        return cayley_transform(self._build_skew())

    def extra_repr(self) -> str:
        return f"dim={self.dim}"


def rotate_weight_right(weight: torch.Tensor, R: torch.Tensor) -> torch.Tensor:
    """``weight @ R``: the rotation absorbed into the input dimension."""
    return torch.matmul(weight, R)


def rotate_weight_left(weight: torch.Tensor, R: torch.Tensor) -> torch.Tensor:
    """``R^T @ weight``: the rotation absorbed into the output dimension."""
    return torch.matmul(R.t(), weight)


@torch.no_grad()
def apply_rotation_to_linear(linear: torch.nn.Linear, R: torch.Tensor, side: str = "right") -> None:
    """Replace ``linear.weight.data`` by its rotation (core/rotation.py:189-207):
    ``side='right'`` W R, ``side='left'`` R^T W; any other side raises
    ``ValueError``."""
    rotate = {"right": rotate_weight_right, "left": rotate_weight_left}.get(side)
    if rotate is None:
        raise ValueError(f"side must be 'right' or 'left', got {side!r}")
    linear.weight.data = rotate(linear.weight.data, R)
