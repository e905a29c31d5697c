"""llm_quant_b200.core.quantizer -- B200 implementation of llm_quant.core.quantizer.

Same names, signatures, defaults, return shapes / dtypes and error types as
the reference module (core/quantizer.py of MindIntels/llm_quant); the work is
done by liblq_sm100 kernels on the tensor's CUDA device.  Values are
bit-identical to the reference's PyTorch CPU results on the same inputs:
every elementwise op is computed in fp32 and rounded to the op's dtype,
exactly as torch's CPU kernels do.
"""

from __future__ import annotations

import math
from enum import Enum
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _C


class QScheme(Enum):
    """Quantization scheme (core/quantizer.py:25-29)."""
    PER_TENSOR = "per_tensor"
    PER_CHANNEL = "per_channel"
    PER_GROUP = "per_group"


def _scheme(scheme) -> str:
    """Accept this module's QScheme, the reference's QScheme or a string."""
    v = scheme.value if isinstance(scheme, Enum) else scheme
    if v not in ("per_tensor", "per_channel", "per_group"):
        raise ValueError(f"Unknown scheme: {scheme}")
    return v


def _qrange(n_bits: int, symmetric: bool):
    if symmetric:
        return -(2 ** (n_bits - 1)), 2 ** (n_bits - 1) - 1
    return 0, 2 ** n_bits - 1


# ──────────────────────────────────────────────────────────────────────────────
# ste_round
# ──────────────────────────────────────────────────────────────────────────────

def _ste_forward(x: torch.Tensor) -> torch.Tensor:
    xc = x.detach().contiguous()
    out = torch.empty_like(xc)
    _C.call("lq_ste_round", xc.data_ptr(), _C.dt(xc), xc.numel(), out.data_ptr(), _C.stream_ptr(xc))
    return out


class _SteRound(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return _ste_forward(x)

    @staticmethod
    def backward(ctx, g):
        return g


def ste_round(x: torch.Tensor) -> torch.Tensor:
    """Round with a straight-through gradient (core/quantizer.py:32-34).

    The value is ``x + (round(x) - x)``: round-half-to-even, except that zero
    results are +0.0 and +-inf becomes NaN, as in the reference."""
    _C.require_cuda(x, what="ste_round")
    _C.require_float(x, "ste_round")
    if x.requires_grad and torch.is_grad_enabled():
        return _SteRound.apply(x)
    return _ste_forward(x)


# ──────────────────────────────────────────────────────────────────────────────
# compute_qparams
# ──────────────────────────────────────────────────────────────────────────────

def _tensor_qparams(x: torch.Tensor, n_bits: int, symmetric: bool):
    if x.numel() == 0:
        raise RuntimeError("max(): Expected reduction dim to be specified for input.numel() == 0.")
    ws_bytes = _C.lib().lq_tensor_qparams_workspace_size(x.numel())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=x.dtype, device=x.device)
    zp = torch.empty((1,) if symmetric else (), dtype=x.dtype, device=x.device)
    _C.call("lq_tensor_qparams", x.data_ptr(), _C.dt(x), x.numel(), n_bits, int(symmetric),
            scale.data_ptr(), zp.data_ptr(), ws.data_ptr(), ws_bytes, _C.stream_ptr(x))
    return scale, zp


def _check_reduce_dims(x: torch.Tensor, keep_dim: int, symmetric: bool) -> None:
    """The reference reduces with torch.amin / amax over every dim but the
    channel dim (core/quantizer.py:64-104), which raises IndexError for a
    zero-size reduced dim; an empty x whose reduced dims are all non-empty
    gives empty results instead."""
    for d in range(x.ndim):
        if d != keep_dim and x.shape[d] == 0:
            op = "amax" if symmetric else "amin"
            raise IndexError(f"{op}(): Expected reduction dim {d} to have non-zero size.")


def _group_qparams(x2: torch.Tensor, group: int, n_bits: int, symmetric: bool):
    rows, cols = x2.shape
    ng = math.ceil(cols / group)
    scale = torch.empty(rows, ng, dtype=x2.dtype, device=x2.device)
    zp = torch.empty_like(scale)
    _C.call("lq_group_quant", x2.data_ptr(), _C.dt(x2), rows, cols, group, n_bits,
            int(symmetric), _C.MODE_QPARAMS, None, 0, scale.data_ptr(), zp.data_ptr(),
            _C.stream_ptr(x2))
    return scale, zp


def compute_qparams(
    x: torch.Tensor,
    n_bits: int = 8,
    symmetric: bool = True,
    scheme: QScheme = QScheme.PER_TENSOR,
    group_size: int = 128,
    channel_dim: int = 0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Scale and zero point (core/quantizer.py:41-108), in x's dtype.

    PER_TENSOR: scale 0-dim, zero_point [1] (symmetric) or 0-dim.
    PER_CHANNEL: keepdim shape with ``channel_dim`` kept.
    PER_GROUP: [out, n_groups, 1] for a 2-D x, last group zero-padded.
    """
    sch = _scheme(scheme)
    _C.require_cuda(x, what="compute_qparams")
    _C.require_float(x, "compute_qparams")
    if not symmetric:  # the zero point is clamped to the code range
        _C.check_clamp_bounds(x.dtype, n_bits, symmetric)
    xc = x.detach().contiguous()
    if sch == "per_tensor":
        return _tensor_qparams(xc, n_bits, symmetric)
    if sch == "per_channel":
        assert x.ndim >= 2, "per-channel requires at least 2-D tensor"
        keep = [1] * x.ndim
        if not (0 <= channel_dim < x.ndim):
            # the reference's reduce_dims then covers every dim
            s, z = _tensor_qparams(xc, n_bits, symmetric)
            return s.reshape(keep), z.reshape(keep) if not symmetric else torch.zeros_like(s.reshape(keep))
        keep[channel_dim] = x.shape[channel_dim]
        _check_reduce_dims(x, channel_dim, symmetric)
        if x.numel() == 0:
            s = torch.empty(keep, dtype=x.dtype, device=x.device)
            return s, torch.empty_like(s)
        if channel_dim == 0:
            s, z = _group_qparams(xc.reshape(x.shape[0], -1), max(1, xc[0].numel()), n_bits, symmetric)
            return s.reshape(keep), z.reshape(keep)
        outer = math.prod(x.shape[:channel_dim])
        C = x.shape[channel_dim]
        inner = math.prod(x.shape[channel_dim + 1:])
        ws_bytes = _C.lib().lq_channel_qparams_workspace_size(outer, C, inner)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        s = torch.empty(C, dtype=x.dtype, device=x.device)
        z = torch.empty_like(s)
        _C.call("lq_channel_qparams", xc.data_ptr(), _C.dt(xc), outer, C, inner, n_bits,
                int(symmetric), s.data_ptr(), z.data_ptr(), ws.data_ptr(), ws_bytes,
                _C.stream_ptr(xc))
        return s.reshape(keep), z.reshape(keep)
    # per_group
    assert x.ndim == 2, "per-group requires a 2-D weight matrix"
    s, z = _group_qparams(xc, group_size, n_bits, symmetric)
    return s.unsqueeze(-1), z.unsqueeze(-1)


# ──────────────────────────────────────────────────────────────────────────────
# quantize / dequantize with given qparams (broadcast, type promotion)
# ──────────────────────────────────────────────────────────────────────────────

def _as_tensor(v, device):
    if isinstance(v, torch.Tensor):
        return v
    return torch.tensor(float(v), dtype=torch.float32, device=device)


def _inter(dtype, ndim):
    return torch.empty((1,) * ndim if ndim else (), dtype=dtype, device="meta")


def _coalesce(shape, *strides):
    """Merge adjacent dims that are contiguous for every operand."""
    shape = list(shape)
    strides = [list(s) for s in strides]
    d = len(shape) - 2
    while d >= 0:
        if all(s[d] == s[d + 1] * shape[d + 1] for s in strides):
            shape[d] *= shape[d + 1]
            del shape[d + 1]
            for s in strides:
                s[d] = s[d + 1]
                del s[d + 1]
        d -= 1
    # drop size-1 dims
    keep = [i for i, n in enumerate(shape) if n != 1]
    return [shape[i] for i in keep], [[s[i] for i in keep] for s in strides]


def _affine(op, x, scale, zp, d0, d1, n_bits, symmetric, out_dtype):
    out_shape = torch.broadcast_shapes(x.shape, scale.shape, zp.shape)
    xe, se, ze = (t.expand(out_shape) for t in (x, scale, zp))
    out = torch.empty(out_shape, dtype=out_dtype, device=x.device)
    if out.numel() == 0:
        return out
    shape, (xs, ss, zs) = _coalesce(out_shape, xe.stride(), se.stride(), ze.stride())
    if len(shape) > 6:
        raise ValueError(f"broadcast of {len(shape)} non-mergeable dims is above the 6 supported")
    p_shape, a1 = _C.i64_array(shape)
    p_xs, a2 = _C.i64_array(xs)
    p_ss, a3 = _C.i64_array(ss)
    p_zs, a4 = _C.i64_array(zs)
    p_dts, a5 = _C.int_array([_C.dt(d0), _C.dt(d1)])
    _C.call("lq_affine", op, len(shape), p_shape, xe.data_ptr(), _C.dt(x), p_xs, se.data_ptr(),
            _C.dt(scale), p_ss, ze.data_ptr(), _C.dt(zp), p_zs, p_dts, n_bits, int(symmetric),
            out.data_ptr(), _C.dt(out_dtype), _C.stream_ptr(x))
    return out


def quantize_tensor(
    x: torch.Tensor,
    scale: torch.Tensor,
    zero_point: torch.Tensor,
    n_bits: int = 8,
    symmetric: bool = True,
) -> torch.Tensor:
    """``round(x / scale + zero_point).clamp(qmin, qmax)`` as a float tensor
    (core/quantizer.py:115-131); broadcasting and dtype as torch would give."""
    scale = _as_tensor(scale, x.device)
    zero_point = _as_tensor(zero_point, x.device)
    _C.require_cuda(x, scale, zero_point, what="quantize_tensor")
    d0 = torch.result_type(x, scale)
    nd = len(torch.broadcast_shapes(x.shape, scale.shape))
    d1 = torch.result_type(_inter(d0, nd), zero_point)
    for d in (d0, d1):
        if d not in _C.FLOAT_TYPES:
            raise TypeError(f"quantize_tensor: unsupported result dtype {d}")
    _C.check_clamp_bounds(d1, n_bits, symmetric)
    return _affine(_C.AFFINE_QUANT, x, scale, zero_point, d0, d1, n_bits, symmetric, d1)


def dequantize_tensor(
    q: torch.Tensor,
    scale: torch.Tensor,
    zero_point: torch.Tensor,
) -> torch.Tensor:
    """``(q - zero_point) * scale`` (core/quantizer.py:134-140)."""
    scale = _as_tensor(scale, q.device)
    zero_point = _as_tensor(zero_point, q.device)
    _C.require_cuda(q, scale, zero_point, what="dequantize_tensor")
    d0 = torch.result_type(q, zero_point)
    nd = len(torch.broadcast_shapes(q.shape, zero_point.shape))
    d1 = torch.result_type(_inter(d0, nd), scale)
    for d in (d0, d1):
        if d not in _C.FLOAT_TYPES:
            raise TypeError(f"dequantize_tensor: unsupported result dtype {d}")
    return _affine(_C.AFFINE_DEQUANT, q, scale, zero_point, d0, d1, 8, True, d1)


# ──────────────────────────────────────────────────────────────────────────────
# fake_quantize
# ──────────────────────────────────────────────────────────────────────────────

def _fake_quant_forward(x, n_bits, symmetric, sch, group_size):
    xc = x.detach().contiguous()
    out = torch.empty_like(xc)
    if sch == "per_tensor":
        s, z = _tensor_qparams(xc, n_bits, symmetric)
        return _affine(_C.AFFINE_FAKE, xc, s, z, xc.dtype, xc.dtype, n_bits, symmetric, xc.dtype)
    if sch == "per_channel":
        assert x.ndim >= 2, "per-channel requires at least 2-D tensor"
        _check_reduce_dims(x, 0, symmetric)
        rows = x.shape[0]
        cols = xc.numel() // max(1, rows)
        group = max(1, cols)
    else:
        assert x.ndim == 2, "per-group requires a 2-D weight matrix"
        rows, cols = x.shape
        if rows == 0:  # the reference reshapes to [out_features, -1]
            raise RuntimeError("cannot reshape tensor of 0 elements into shape [0, -1] because the "
                               "unspecified dimension size -1 can be any value and is ambiguous")
        group = group_size
    _C.call("lq_group_quant", xc.data_ptr(), _C.dt(xc), rows, cols, group, n_bits,
            int(symmetric), _C.MODE_FAKE, out.data_ptr(), _C.dt(out), None, None,
            _C.stream_ptr(xc))
    return out


class _FakeQuantFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, n_bits, symmetric, sch, group_size):
        ctx.save_for_backward(x)
        ctx.cfg = (n_bits, symmetric, sch, group_size)
        return _fake_quant_forward(x, n_bits, symmetric, sch, group_size)

    @staticmethod
    def backward(ctx, g):
        from .fake_quant_grad import fake_quantize_backward
        (x,) = ctx.saved_tensors
        return (fake_quantize_backward(x, g, *ctx.cfg), None, None, None, None)


def fake_quantize(
    x: torch.Tensor,
    n_bits: int = 8,
    symmetric: bool = True,
    scheme: QScheme = QScheme.PER_TENSOR,
    group_size: int = 128,
) -> torch.Tensor:
    """Quantize -> dequantize in one pass (core/quantizer.py:143-185).

    Differentiable: the gradient is the reference's (straight-through round,
    clamp mask, and the path through the min/max scale)."""
    sch = _scheme(scheme)
    _C.require_cuda(x, what="fake_quantize")
    _C.require_float(x, "fake_quantize")
    _C.check_clamp_bounds(x.dtype, n_bits, symmetric)
    if x.requires_grad and torch.is_grad_enabled():
        return _FakeQuantFn.apply(x, n_bits, symmetric, sch, group_size)
    return _fake_quant_forward(x, n_bits, symmetric, sch, group_size)


# ──────────────────────────────────────────────────────────────────────────────
# QuantizedLinear
# ──────────────────────────────────────────────────────────────────────────────

def int_weight_fp32(m, what: str) -> torch.Tensor:
    """``(weight_int.float() - zero_point) * scale`` per group of the input dim
    (or per row when group_size <= 0), in fp32 -- the weight the forward of
    QuantizedLinear / GPTQLinear / SpQRLinear builds before F.linear
    (core/quantizer.py:264-279, gptq.py:302-314, spqr.py:172-189)."""
    _C.require_cuda(m.weight_int, m.scale, m.zero_point, what=what)
    N, K = m.out_features, m.in_features
    wi = m.weight_int.contiguous()
    s = m.scale.reshape(N, -1).contiguous()
    z = m.zero_point.reshape(N, -1)
    z = (z.to(s.dtype) if z.dtype != s.dtype else z).contiguous()
    out = torch.empty(N, K, dtype=torch.float32, device=wi.device)
    if m.group_size > 0:
        ng = s.shape[1]
        tg = m.group_size
    else:
        ng, tg = 1, K
    _C.call("lq_kv_dequant", wi.data_ptr(), _C.I8, N, K, 1, K, 2, tg, s.data_ptr(),
            z.data_ptr(), _C.dt(s), ng, out.data_ptr(), _C.stream_ptr(wi))
    return out


def bind_int_qparams(m, scale: torch.Tensor, zp: torch.Tensor) -> None:
    """Store [out, n_groups] qparams on an int-weight layer.  The layer's
    buffers are replaced when the shape changes (its constructor makes them
    [out, 1]; the reference rebinds them then, so state_dicts carry the
    grouped shape) and copied into otherwise.  Drops the packed W4A16
    operand."""
    if scale.shape != m.scale.shape:
        m.scale, m.zero_point = scale, zp
    else:
        m.scale.copy_(scale)
        m.zero_point.copy_(zp)
    m._w4 = None


def row_group_quantize(m, weight: torch.Tensor, symmetric: bool, what: str,
                       codes: bool = True) -> None:
    """One pass of lq_group_quant over a 2-D weight [out, in]: qparams of
    every group of ``m.group_size`` columns (the last group zero-padded; one
    group per row when group_size <= 0) and, with ``codes``, the int8 codes
    written straight into ``m.weight_int``.  Values equal compute_qparams
    PER_GROUP / PER_CHANNEL followed by quantize_tensor on the padded groups
    (core/quantizer.py:231-260)."""
    _C.require_cuda(weight, what=what)
    _C.require_float(weight, what)
    _C.check_clamp_bounds(weight.dtype, m.n_bits, symmetric)
    w = weight.detach().contiguous()
    N, K = w.shape
    G = m.group_size if m.group_size > 0 else K
    scale = torch.empty(N, math.ceil(K / G), dtype=w.dtype, device=w.device)
    zp = torch.empty_like(scale)
    out = None
    if codes:
        direct = (m.weight_int.device == w.device and m.weight_int.is_contiguous()
                  and m.weight_int.shape == (N, K))
        out = m.weight_int if direct else torch.empty(N, K, dtype=torch.int8, device=w.device)
    _C.call("lq_group_quant", w.data_ptr(), _C.dt(w), N, K, G, m.n_bits, int(symmetric),
            _C.MODE_CODES if codes else _C.MODE_QPARAMS, _C.ptr(out), _C.I8, scale.data_ptr(),
            zp.data_ptr(), _C.stream_ptr(w))
    if codes and out is not m.weight_int:
        m.weight_int.copy_(out.reshape_as(m.weight_int))
    bind_int_qparams(m, scale, zp)


def int_linear_forward(m, x: torch.Tensor) -> torch.Tensor:
    """Forward of an int-weight linear: the fused W4A16 kernel for fp16 / bf16
    activations when the layout allows it, else the reference's fp32
    dequantize + F.linear."""
    from . import w4a16
    if w4a16.eligible(m, x):
        return w4a16.linear(m, x)
    return F.linear(x, int_weight_fp32(m, type(m).__name__), m.bias)


class QuantizedLinear(nn.Module):
    """Drop-in ``nn.Linear`` replacement storing INT weights (core/quantizer.py:192-301).

    Buffers match the reference (``weight_int`` int8 [out, in], ``scale`` /
    ``zero_point`` [out, n_groups]), so state_dicts are interchangeable.

    forward:
      * float16 / bfloat16 activations with n_bits <= 4 group quantization
        run the fused W4A16 tensor-core kernel (int4 weights dequantized in
        tensor memory, fp32 accumulation); its packed operand is a derived
        cache rebuilt after every quantize_weights / load_state_dict;
      * otherwise the weight is dequantized to fp32 exactly as the reference
        does (bit-identical) and multiplied with ``F.linear``.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        n_bits: int = 8,
        symmetric: bool = True,
        group_size: int = 0,
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
    def quantize_weights(self, weight: torch.Tensor) -> None:
        """Quantize a float weight and store INT codes + scale / zero point
        (core/quantizer.py:231-260), one fused pass over the weight."""
        row_group_quantize(self, weight, self.symmetric, "QuantizedLinear.quantize_weights")

    def _load_from_state_dict(self, *args, **kwargs):
        self._w4 = None
        return super()._load_from_state_dict(*args, **kwargs)

    def _apply(self, fn, *args, **kwargs):
        self._w4 = None
        return super()._apply(fn, *args, **kwargs)

    def dequantized_weight(self) -> torch.Tensor:
        """The fp32 weight the reference's forward builds (core/quantizer.py:264-279)."""
        return int_weight_fp32(self, "QuantizedLinear")

    def _w4a16_eligible(self, x: torch.Tensor) -> bool:
        from . import w4a16
        return w4a16.eligible(self, x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return int_linear_forward(self, x)

    @classmethod
    def from_linear(cls, linear: nn.Linear, n_bits: int = 8,
                    symmetric: bool = True, group_size: int = 0) -> "QuantizedLinear":
        """Create a QuantizedLinear from an nn.Linear (core/quantizer.py:282-294);
        the new module lives on the linear's device."""
        ql = cls(
            linear.in_features, linear.out_features,
            n_bits=n_bits, symmetric=symmetric, group_size=group_size,
            bias=linear.bias is not None,
        ).to(linear.weight.device)
        ql.quantize_weights(linear.weight.data)
        if linear.bias is not None:
            ql.bias.data.copy_(linear.bias.data)
        return ql

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, "
            f"bits={self.n_bits}, sym={self.symmetric}, "
            f"group_size={self.group_size}, bias={self.bias is not None}"
        )
