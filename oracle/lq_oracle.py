"""CPU oracle for the llm_quant quantization hot path -- TEST INFRASTRUCTURE ONLY.

This module is a plain-numpy restatement of the reference's algorithms
(MindIntels/llm_quant, pure PyTorch).  It exists to check the CUDA product
path; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline legs may import it.  Nothing in ``llm_quant_b200`` calls it.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree) on seeded inputs and stores inputs and
outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
module against every stored case bit for bit.

Numeric model
-------------
Every tensor value is held as a float32 numpy array whose values are exactly
representable in the tensor's dtype ('float32', 'float16' or 'bfloat16').
Every elementwise torch op of the reference is restated as: fp32 IEEE
arithmetic on the exact input values, then one round-to-nearest-even to the
op's result dtype.  That is what torch's CPU kernels do for fp32, fp16 and
bf16 (reduced-precision types compute in float "opmath" and round after each
op), so the restatement is bit-exact (the golden tests prove it).

Reductions (amin/amax) are exact and propagate NaN, like torch's.
"""

from __future__ import annotations

import math
import numpy as np

F32, F16, BF16 = "float32", "float16", "bfloat16"
FLOAT_DTYPES = (F32, F16, BF16)
_RANK = {F16: 1, BF16: 1, F32: 2}


# ─────────────────────────────────────────────────────────────────────────────
# dtype helpers
# ─────────────────────────────────────────────────────────────────────────────

def to_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), kept as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out.reshape(a.shape)


def rnd(a, dt: str) -> np.ndarray:
    """Round float32 values to dtype ``dt``; result stays a float32 array."""
    a = np.asarray(a, dtype=np.float32)
    if dt == F32:
        return a
    if dt == F16:
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    if dt == BF16:
        return to_bf16(a)
    raise TypeError(f"unsupported dtype {dt}")


def promote(*dts: str) -> str:
    """torch.result_type for dimensioned float tensors of the given dtypes."""
    dts = set(dts)
    if F32 in dts:
        return F32
    if dts == {F16}:
        return F16
    if dts == {BF16}:
        return BF16
    return F32  # float16 with bfloat16 promotes to float32


def result_type(*operands) -> str:
    """torch.result_type for float operands given as (array, dtype) pairs.

    Zero-dim tensors only take part when no dimensioned tensor is present
    (all operands here are of the floating category)."""
    dims = [dt for a, dt in operands if np.ndim(a) > 0]
    return promote(*(dims or [dt for _, dt in operands]))


def _op(fn, dt, *args):
    with np.errstate(all="ignore"):
        return rnd(fn(*[np.asarray(a, np.float32) for a in args]), dt)


def div(a, b, dt):
    return _op(lambda x, y: x / y, dt, a, b)


def add(a, b, dt):
    return _op(lambda x, y: x + y, dt, a, b)


def sub(a, b, dt):
    return _op(lambda x, y: x - y, dt, a, b)


def mul(a, b, dt):
    return _op(lambda x, y: x * y, dt, a, b)


def clamp(a, lo, hi, dt=None):
    """torch.clamp semantics: NaN passes through, -0.0 is kept.  With ``dt``
    the tensor is of that dtype, so the result is too: a bound that the dtype
    cannot hold (qmax = 4095 in bf16) acts as its rounded value (4096), as
    observed on the reference for 12-bit codes."""
    if dt is not None:
        lo, hi = rnd(np.float32(lo), dt), rnd(np.float32(hi), dt)
    a = np.asarray(a, np.float32)
    out = np.where(a < np.float32(lo), np.float32(lo), a)
    out = np.where(out > np.float32(hi), np.float32(hi), out)
    return out.astype(np.float32)


def clamp_min(a, lo_value: float, dt: str):
    """``t.clamp(min=v)``: the scalar is first converted to the tensor dtype."""
    lo = rnd(np.float32(lo_value), dt)
    a = np.asarray(a, np.float32)
    return np.where(a < lo, lo, a).astype(np.float32)


def rint(a):
    """torch.round: round half to even, keeps the sign of zero."""
    return np.rint(np.asarray(a, np.float32)).astype(np.float32)


def ste_round(a):
    """Value of ``x + (x.round() - x).detach()`` (core/quantizer.py:32-34).

    Equal to round(x) except that zero results are +0.0 and +-inf becomes NaN.
    """
    a = np.asarray(a, np.float32)
    with np.errstate(invalid="ignore"):
        r = rint(a)
        d = (r - a).astype(np.float32)
        return (a + d).astype(np.float32)


def qrange(n_bits: int, symmetric: bool):
    """core/quantizer.py:56-61 and kv_cache_quant.py:95-100."""
    if symmetric:
        return -(2 ** (n_bits - 1)), 2 ** (n_bits - 1) - 1
    return 0, 2 ** n_bits - 1


def to_int(a, np_dtype):
    """``float_tensor.to(intN)`` on x86: truncate through int32; NaN/inf -> INT_MIN."""
    a = np.asarray(a, np.float32)
    bad = ~np.isfinite(a) | (np.abs(a) >= 2.0 ** 31)
    with np.errstate(invalid="ignore"):
        i32 = np.where(bad, np.int64(-(2 ** 31)), np.trunc(np.where(bad, 0, a)).astype(np.int64))
    return i32.astype(np.int64).astype(np_dtype)


# ─────────────────────────────────────────────────────────────────────────────
# core/quantizer.py
# ─────────────────────────────────────────────────────────────────────────────

def _amax(a, axis, keepdims=True):
    with np.errstate(invalid="ignore"):
        return np.max(a, axis=axis, keepdims=keepdims).astype(np.float32)


def _amin(a, axis, keepdims=True):
    with np.errstate(invalid="ignore"):
        return np.min(a, axis=axis, keepdims=keepdims).astype(np.float32)


def _scale_zp_from_minmax(x_min, x_max, dt, qmin, qmax, symmetric, amax=None):
    """The shared scale / zero-point formulas of core/quantizer.py:64-104."""
    if symmetric:
        a = clamp_min(amax, 1e-12, dt)
        scale = div(a, np.float32(qmax), dt)
        zp = np.zeros_like(scale)
    else:
        rngv = clamp_min(sub(x_max, x_min, dt), 1e-12, dt)
        scale = div(rngv, np.float32(qmax - qmin), dt)
        zp = clamp(rint(div(-x_min, scale, dt)), qmin, qmax, dt)
    return scale, zp


def pad_groups(x, group_size):
    """F.pad of the last dim to a multiple of group_size, then reshape (core/quantizer.py:89-95)."""
    out_f, in_f = x.shape
    n_groups = math.ceil(in_f / group_size)
    padded = in_f % group_size
    if padded != 0:
        x = np.concatenate([x, np.zeros((out_f, group_size - padded), np.float32)], axis=1)
    return x.reshape(out_f, n_groups, group_size)


def compute_qparams(x, dt, n_bits=8, symmetric=True, scheme="per_tensor",
                    group_size=128, channel_dim=0):
    """core/quantizer.py:41-108.  Returns (scale, zero_point) in dtype ``dt``."""
    x = np.asarray(x, np.float32)
    qmin, qmax = qrange(n_bits, symmetric)
    if scheme == "per_tensor":
        if symmetric:
            amax = np.float32(np.max(np.abs(x))) if x.size else None
            scale, _ = _scale_zp_from_minmax(None, None, dt, qmin, qmax, True,
                                             amax=np.asarray(amax, np.float32))
            return np.asarray(scale, np.float32).reshape(()), np.zeros((1,), np.float32)
        mn = np.asarray(np.min(x), np.float32)
        mx = np.asarray(np.max(x), np.float32)
        scale, zp = _scale_zp_from_minmax(mn, mx, dt, qmin, qmax, False)
        return scale.reshape(()), zp.reshape(())
    if scheme == "per_channel":
        assert x.ndim >= 2, "per-channel requires at least 2-D tensor"
        red = tuple(i for i in range(x.ndim) if i != channel_dim)
        if symmetric:
            amax = _amax(np.abs(x), red)
            return _scale_zp_from_minmax(None, None, dt, qmin, qmax, True, amax=amax)
        return _scale_zp_from_minmax(_amin(x, red), _amax(x, red), dt, qmin, qmax, False)
    if scheme == "per_group":
        assert x.ndim == 2, "per-group requires a 2-D weight matrix"
        xg = pad_groups(x, group_size)
        if symmetric:
            amax = _amax(np.abs(xg), -1)
            return _scale_zp_from_minmax(None, None, dt, qmin, qmax, True, amax=amax)
        return _scale_zp_from_minmax(_amin(xg, -1), _amax(xg, -1), dt, qmin, qmax, False)
    raise ValueError(f"Unknown scheme: {scheme}")


def quantize_tensor(x, xdt, scale, sdt, zp, zdt, n_bits=8, symmetric=True):
    """core/quantizer.py:115-131: ``round(x / scale + zp).clamp(qmin, qmax)`` (float result).

    Returns (q, result_dtype)."""
    qmin, qmax = qrange(n_bits, symmetric)
    d1 = result_type((x, xdt), (scale, sdt))
    t = div(x, scale, d1)
    d2 = result_type((t, d1), (zp, zdt))
    t = add(t, zp, d2)
    return clamp(rint(t), qmin, qmax, d2), d2


def dequantize_tensor(q, qdt, scale, sdt, zp, zdt):
    """core/quantizer.py:134-140: ``(q - zp) * scale``.

    ``qdt`` may be an integer kind ('int') which promotes to the other dtype."""
    d1 = zdt if qdt == "int" else result_type((q, qdt), (zp, zdt))
    t = sub(np.asarray(q, np.float32), zp, d1)
    d2 = result_type((t, d1), (scale, sdt))
    return mul(t, scale, d2), d2


def fake_quantize(x, dt, n_bits=8, symmetric=True, scheme="per_tensor", group_size=128):
    """core/quantizer.py:143-185 (forward value)."""
    x = np.asarray(x, np.float32)
    scale, zp = compute_qparams(x, dt, n_bits, symmetric, scheme, group_size)
    qmin, qmax = qrange(n_bits, symmetric)
    if scheme == "per_group" and x.ndim == 2:
        out_f, in_f = x.shape
        xg = pad_groups(x, group_size)
        q = clamp(ste_round(add(div(xg, scale, dt), zp, dt)), qmin, qmax, dt)
        dq = mul(sub(q, zp, dt), scale, dt)
        return dq.reshape(out_f, -1)[:, :in_f]
    q = clamp(ste_round(add(div(x, scale, dt), zp, dt)), qmin, qmax, dt)
    return mul(sub(q, zp, dt), scale, dt)


def quantized_linear_quantize_weights(w, dt, n_bits=8, symmetric=True, group_size=0):
    """QuantizedLinear.quantize_weights (core/quantizer.py:231-260).

    Returns (weight_int int8 [out,in], scale [out, n_groups or 1], zero_point)."""
    w = np.asarray(w, np.float32)
    out_f, in_f = w.shape
    scheme = "per_group" if group_size > 0 else "per_channel"
    scale, zp = compute_qparams(w, dt, n_bits, symmetric, scheme, group_size)
    if scheme == "per_group":
        wg = pad_groups(w, group_size)
        q, _ = quantize_tensor(wg, dt, scale, dt, zp, dt, n_bits, symmetric)
        q = q.reshape(out_f, -1)[:, :in_f]
    else:
        q, _ = quantize_tensor(w, dt, scale, dt, zp, dt, n_bits, symmetric)
    return to_int(q, np.int8), scale.reshape(out_f, -1), zp.reshape(out_f, -1)


def gptq_linear_pack(w_q, w, dt, n_bits=4, symmetric=True, group_size=128):
    """GPTQLinear.pack (gptq.py:285-299): the given codes as int8, the qparams
    of the original weight.  Returns (weight_int, scale, zero_point)."""
    w = np.asarray(w, np.float32)
    out_f = w.shape[0]
    scheme = "per_group" if group_size > 0 else "per_channel"
    scale, zp = compute_qparams(w, dt, n_bits, symmetric, scheme, group_size)
    wi = np.asarray(w_q).astype(np.int64).astype(np.int8)
    return wi, scale.reshape(out_f, -1), zp.reshape(out_f, -1)


def spqr_linear_pack(w, mask, dt, n_bits=4, group_size=128):
    """SpQRLinear.pack (spqr.py:128-170): outliers kept in fp (mask order),
    the rest quantized symmetrically with the outliers zeroed.  Returns
    (weight_int, scale, zero_point, outlier_vals)."""
    w = np.asarray(w, np.float32)
    mask = np.asarray(mask, bool)
    vals = w[mask].astype(np.float32)
    w0 = np.where(mask, np.float32(0.0), w).astype(np.float32)
    wi, scale, zp = quantized_linear_quantize_weights(w0, dt, n_bits, True, group_size)
    return wi, scale, zp, vals


def spqr_linear_dequant_weight(weight_int, scale, sdt, zp, zdt, group_size, in_features, mask, vals):
    """The fp32 weight SpQRLinear.forward builds (spqr.py:172-193)."""
    w = quantized_linear_dequant_weight(weight_int, scale, sdt, zp, zdt, group_size, in_features).copy()
    w[np.asarray(mask, bool)] = np.asarray(vals, np.float32)
    return w


def quantized_linear_dequant_weight(weight_int, scale, sdt, zp, zdt, group_size, in_features):
    """The fp32 weight QuantizedLinear.forward builds (core/quantizer.py:264-279)."""
    wi = np.asarray(weight_int, np.float32)
    out_f = wi.shape[0]
    if group_size > 0:
        n_groups = scale.shape[1]
        padded_in = n_groups * group_size
        if padded_in > in_features:
            wi = np.concatenate([wi, np.zeros((out_f, padded_in - in_features), np.float32)], 1)
        wg = wi.reshape(out_f, n_groups, group_size)
        d1 = promote(F32, zdt)
        t = sub(wg, zp[..., None], d1)
        w = mul(t, scale[..., None], promote(d1, sdt))
        return w.reshape(out_f, -1)[:, :in_features]
    w, _ = dequantize_tensor(wi, F32, scale, sdt, zp, zdt)
    return w


# ─────────────────────────────────────────────────────────────────────────────
# core/rotation.py
# ─────────────────────────────────────────────────────────────────────────────

def hadamard_matrix(n: int, dt: str = F32) -> np.ndarray:
    """core/rotation.py:30-43: Sylvester doubling, then ``H / sqrt(n)`` in dtype."""
    assert n > 0 and (n & (n - 1)) == 0, "n must be a power of 2"
    H = np.ones((1, 1), np.float32)
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]]).astype(np.float32)
    return div(H, np.float32(math.sqrt(n)), dt)


def hadamard_entry(d: int, dt: str) -> np.float32:
    """Magnitude of every entry of ``hadamard_matrix(d, dt)``."""
    return rnd(np.float32(1.0) / np.float32(math.sqrt(d)), dt).reshape(())


def fast_hadamard_transform(x, dt):
    """core/rotation.py:130-147 is ``x @ hadamard_matrix(d, x.dtype)``.

    Restated as an exact float64 butterfly over +-1 followed by the dtype-rounded
    ``1/sqrt(d)`` entry, rounded once to ``dt``.  The reference's matmul rounds
    in its own order, so comparisons with it use a tolerance."""
    x = np.asarray(x, np.float64)
    d = x.shape[-1]
    assert d > 0 and (d & (d - 1)) == 0, "last dim must be power of 2"
    y = x.reshape(-1, d).copy()
    h = 1
    while h < d:
        y = y.reshape(-1, d // (2 * h), 2, h)
        a = y[:, :, 0, :].copy()
        b = y[:, :, 1, :].copy()
        y[:, :, 0, :] = a + b
        y[:, :, 1, :] = a - b
        y = y.reshape(-1, d)
        h *= 2
    y = y * np.float64(hadamard_entry(d, dt))
    return rnd(y.astype(np.float32), dt).reshape(x.shape) if dt != F32 else \
        y.astype(np.float32).reshape(x.shape)


# ─────────────────────────────────────────────────────────────────────────────
# qlora.py
# ─────────────────────────────────────────────────────────────────────────────

NF4_TABLE = np.array([
    -1.0000, -0.6962, -0.5251, -0.3949,
    -0.2844, -0.1848, -0.0911, 0.0000,
    0.0796, 0.1609, 0.2461, 0.3379,
    0.4407, 0.5626, 0.7230, 1.0000,
], dtype=np.float32)  # qlora.py:50-55 (float32 literals)


def _flat_groups(x, group_size):
    x = np.asarray(x, np.float32).reshape(-1)
    n = x.size
    pad = (group_size - n % group_size) % group_size
    if pad:
        x = np.concatenate([x, np.zeros(pad, np.float32)])
    return x.reshape(-1, group_size), n


def nf4_encode(x_norm):
    """``argmin |x_norm - NF4_TABLE|`` computed in fp32, first minimum (qlora.py:103-104).

    NaN rows give code 0 (torch.argmin returns the first NaN)."""
    xn = np.asarray(x_norm, np.float32)
    with np.errstate(invalid="ignore"):
        diffs = np.abs((xn[..., None] - NF4_TABLE).astype(np.float32))
    codes = np.argmin(diffs, axis=-1)  # numpy argmin: first min; NaN -> first NaN
    return codes.astype(np.int64)


def nf4_quantize(x, dt, group_size=64):
    """qlora.py:66-110.  Returns (codes int64 in x's shape, scales [n_groups] in dt)."""
    shape = np.shape(x)
    xg, n = _flat_groups(x, group_size)
    scales = clamp_min(_amax(np.abs(xg), -1), 1e-12, dt)
    x_norm = div(xg, scales, dt)
    codes = nf4_encode(x_norm).reshape(-1)[:n].reshape(shape)
    return codes, scales.reshape(-1)


def nf4_dequantize(codes, scales, sdt, group_size=64, orig_shape=None):
    """qlora.py:113-157: ``NF4_TABLE.to(scales.dtype)[codes] * scales``."""
    codes = np.asarray(codes)
    shape = codes.shape
    table = rnd(NF4_TABLE, sdt)
    cflat = codes.reshape(-1)
    n = cflat.size
    pad = (group_size - n % group_size) % group_size
    if pad:
        cflat = np.concatenate([cflat, np.zeros(pad, cflat.dtype)])
    vals = table[cflat.reshape(-1, group_size)]
    x = mul(vals, np.asarray(scales, np.float32)[:, None], sdt).reshape(-1)[:n]
    return x.reshape(orig_shape if orig_shape is not None else shape)


def double_quantize(scales, sdt, dq_group_size=256):
    """qlora.py:164-196.  Returns (q_scales [n] in sdt, dq_scales [n_dq] in sdt)."""
    sg, n = _flat_groups(scales, dq_group_size)
    dq = clamp_min(_amax(np.abs(sg), -1, keepdims=False), 1e-12, sdt)
    s_norm = div(sg, dq[:, None], sdt)
    q = clamp(rint(mul(s_norm, np.float32(127.0), sdt)), -127, 127)
    return q.reshape(-1)[:n], dq


def double_dequantize(q_scales, dq_scales, sdt, dq_group_size=256):
    """qlora.py:199-223: ``(q / 127) * dq`` in the scales' dtype."""
    qg, n = _flat_groups(q_scales, dq_group_size)
    s = mul(div(qg, np.float32(127.0), sdt), np.asarray(dq_scales, np.float32)[:, None], sdt)
    return s.reshape(-1)[:n]


# ─────────────────────────────────────────────────────────────────────────────
# kv_cache_quant.py
# ─────────────────────────────────────────────────────────────────────────────

PER_TOKEN, PER_CHANNEL, PER_GROUP = "per_token", "per_channel", "per_group"


def kv_qparams(x, dt, n_bits=8, symmetric=True, granularity=PER_TOKEN, group_size=32):
    """KVCacheQuantizer._compute_qparams / _compute_qparams_grouped (kv_cache_quant.py:102-166).

    PER_GROUP returns [B,H,ng,1,D] (before the squeeze done by quantize)."""
    x = np.asarray(x, np.float32)
    qmin, qmax = qrange(n_bits, symmetric)
    if granularity == PER_GROUP:
        B, H, T, D = x.shape
        ng = math.ceil(T / group_size)
        pad = ng * group_size - T
        if pad:
            x = np.concatenate([x, np.zeros((B, H, pad, D), np.float32)], axis=2)
        x = x.reshape(B, H, ng, group_size, D)
        ax = 3
    elif granularity == PER_TOKEN:
        ax = -1
    elif granularity == PER_CHANNEL:
        ax = -2
    else:
        raise ValueError(f"Unknown granularity: {granularity}")
    if symmetric:
        return _scale_zp_from_minmax(None, None, dt, qmin, qmax, True, amax=_amax(np.abs(x), ax))
    return _scale_zp_from_minmax(_amin(x, ax), _amax(x, ax), dt, qmin, qmax, False)


def kv_quantize(x, dt, n_bits=8, symmetric=True, granularity=PER_TOKEN, group_size=32):
    """KVCacheQuantizer.quantize (kv_cache_quant.py:168-219).  Returns (q, scale, zp)."""
    x = np.asarray(x, np.float32)
    qmin, qmax = qrange(n_bits, symmetric)
    idt = np.int8 if symmetric else np.int16
    scale, zp = kv_qparams(x, dt, n_bits, symmetric, granularity, group_size)
    if granularity == PER_GROUP:
        B, H, T, D = x.shape
        ng = scale.shape[2]
        pad = ng * group_size - T
        xp = np.concatenate([x, np.zeros((B, H, pad, D), np.float32)], 2) if pad else x
        xg = xp.reshape(B, H, ng, group_size, D)
        q = clamp(rint(add(div(xg, scale, dt), zp, dt)), qmin, qmax, dt)
        q = q.reshape(B, H, ng * group_size, D)[:, :, :T, :]
        return to_int(q, idt), scale[:, :, :, 0, :], zp[:, :, :, 0, :]
    q = clamp(rint(add(div(x, scale, dt), zp, dt)), qmin, qmax, dt)
    return to_int(q, idt), scale, zp


def kv_dequantize(q, scale, sdt, zp, zdt, granularity=PER_TOKEN, group_size=32):
    """KVCacheQuantizer.dequantize (kv_cache_quant.py:221-267): fp32 ``(q.float() - zp) * scale``."""
    qf = np.asarray(q).astype(np.float32)
    if granularity == PER_GROUP:
        B, H, T, D = qf.shape
        ng = scale.shape[2]
        pT = ng * group_size
        if pT > T:
            qf = np.concatenate([qf, np.zeros((B, H, pT - T, D), np.float32)], 2)
        qg = qf.reshape(B, H, ng, group_size, D)
        x = mul(sub(qg, zp[:, :, :, None, :], F32), scale[:, :, :, None, :], F32)
        return x.reshape(B, H, pT, D)[:, :, :T, :]
    return mul(sub(qf, zp, F32), scale, F32)


class QuantizedKVCacheOracle:
    """QuantizedKVCache (kv_cache_quant.py:312-426), with an optional separate
    value quantizer (the reference uses one quantizer for K and V)."""

    def __init__(self, num_layers, dt, key_q, value_q=None):
        # key_q / value_q: dicts(n_bits, symmetric, granularity, group_size)
        self.num_layers = num_layers
        self.dt = dt
        self.kq = key_q
        self.vq = value_q or key_q
        self._cache = [None] * num_layers

    def _merge(self, old, new, gran):
        if gran == PER_CHANNEL:
            with np.errstate(invalid="ignore"):
                return np.where(np.isnan(old) | np.isnan(new), np.float32("nan"),
                                np.maximum(old, new)).astype(np.float32)
        return np.concatenate([old, new], axis=2)

    def update(self, layer, key, value):
        kq, ks, kz = kv_quantize(key, self.dt, **self.kq)
        vq, vs, vz = kv_quantize(value, self.dt, **self.vq)
        if self._cache[layer] is None:
            self._cache[layer] = (kq, ks, kz, vq, vs, vz)
        else:
            o = self._cache[layer]
            gk, gv = self.kq["granularity"], self.vq["granularity"]
            self._cache[layer] = (
                np.concatenate([o[0], kq], 2), self._merge(o[1], ks, gk), self._merge(o[2], kz, gk),
                np.concatenate([o[3], vq], 2), self._merge(o[4], vs, gv), self._merge(o[5], vz, gv),
            )
        return self.get(layer)

    def get(self, layer):
        c = self._cache[layer]
        if c is None:
            return None
        fk = kv_dequantize(c[0], c[1], self.dt, c[2], self.dt, self.kq["granularity"],
                           self.kq.get("group_size", 32))
        fv = kv_dequantize(c[3], c[4], self.dt, c[5], self.dt, self.vq["granularity"],
                           self.vq.get("group_size", 32))
        return fk, fv


def kv_attention(q, k, v, sm_scale=None, causal=False):
    """Decode attention over a layer's dequantized cache, in float64.

    k, v: the fp32 [B, H, T, D] tensors QuantizedKVCache.update / get return
    (kv_cache_quant.py:336-382, 408-415; ``QuantizedKVCacheOracle.get``).
    q: [B, Hq, Sq, D], Hq a multiple of H; query head h reads kv head
    h // (Hq // H).  out = softmax(q k^T * sm_scale) v, sm_scale defaulting to
    D ** -0.5; causal: query i of Sq sees tokens t <= T - Sq + i.  The
    reference stops at the dequantized K, V; this is the standard attention
    its caller computes with them."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Hq, Sq, D = q.shape
    H, T = k.shape[1], k.shape[2]
    G = Hq // H
    sm = D ** -0.5 if sm_scale is None else float(sm_scale)
    kk = np.repeat(k, G, axis=1)
    vv = np.repeat(v, G, axis=1)
    s = np.einsum("bhid,bhtd->bhit", q, kk) * sm
    if causal:
        t = np.arange(T)[None, :]
        i = np.arange(Sq)[:, None]
        s = np.where(t <= T - Sq + i, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhit,bhtd->bhid", p, vv)
