"""Fused NF4 base product for QLoRALinear.forward (qlora.py:306-312).

The reference's forward dequantizes the whole NF4 base weight
(``_dequantize_base``, qlora.py:294-304) and calls ``F.linear``; with a bf16 or
fp16 base that call fails, because the bias and the LoRA factors stay fp32.
Here, for fp16 / bf16 activations of the base weight's dtype, the base product
runs in one kernel that looks the NF4 codes up and applies the block scale on
the fly (``lq_nf4_linear``: tensor cores, fp32 accumulation, the fp32 bias
added before the one rounding), with the weights exactly those
``_dequantize_base`` returns.  fp32 activations keep the reference's
computation.

The kernel operand (codes re-tiled + one restored scale per row and 64-wide K
step) is built on first use and cached on the module, keyed on the storage
and version counter of every buffer it is built from, so ``pack_base``, a
state-dict load or an in-place edit of the scales rebuilds it.
"""

from __future__ import annotations

import torch

from . import _C
from .core.w4a16 import _err_flag


def _use_dq(ql) -> bool:
    return ql.double_quant and hasattr(ql, "dq_q_scales")


def base_dtype(ql) -> torch.dtype:
    return (ql.dq_q_scales if _use_dq(ql) else ql.nf4_scales).dtype


def eligible(ql, x: torch.Tensor) -> bool:
    K, N, G = ql.in_features, ql.out_features, ql.group_size
    return (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and x.dtype == base_dtype(ql)
            and x.shape[-1] == K and ql.nf4_codes_packed.is_cuda
            and N % 128 == 0 and K % 64 == 0 and G % 64 == 0 and K % G == 0)


def _sources(ql):
    ts = [ql.nf4_codes_packed]
    ts += [ql.dq_q_scales, ql.dq_scales] if _use_dq(ql) else [ql.nf4_scales]
    return ts


def packed_operand(ql, act_dtype: torch.dtype) -> torch.Tensor:
    """Build (or fetch the cached) kernel operand for `act_dtype`."""
    src = _sources(ql)
    key = (act_dtype, src[0].device) + tuple((t.data_ptr(), t._version) for t in src)
    cached = getattr(ql, "_nf4lin", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    N, K, G = ql.out_features, ql.in_features, ql.group_size
    codes = ql.nf4_codes_packed
    packed = torch.empty(_C.lib().lq_nf4_linear_packed_bytes(N, K), dtype=torch.uint8,
                         device=codes.device)
    if _use_dq(ql):
        qs = ql.dq_q_scales.contiguous()
        dq = ql.dq_scales.to(qs.dtype).contiguous()
        _C.call("lq_nf4_linear_pack", codes.data_ptr(), None, qs.data_ptr(), dq.data_ptr(),
                _C.dt(qs), N, K, G, ql._dq_gs, _C.dt(act_dtype), packed.data_ptr(),
                _C.stream_ptr(codes))
    else:
        s = ql.nf4_scales.contiguous()
        _C.call("lq_nf4_linear_pack", codes.data_ptr(), s.data_ptr(), None, None, _C.dt(s), N, K,
                G, 0, _C.dt(act_dtype), packed.data_ptr(), _C.stream_ptr(codes))
    ql._nf4lin = (key, packed)
    return packed


def _forward(ql, x: torch.Tensor, bias) -> torch.Tensor:
    packed = packed_operand(ql, x.dtype)
    N, K = ql.out_features, ql.in_features
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty(M, N, dtype=x.dtype, device=x.device)
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != torch.float32 or not b.is_contiguous():
            b = b.float().contiguous()
    _C.call("lq_nf4_linear", x2.data_ptr(), _C.dt(x2), M, N, K, packed.data_ptr(), _C.ptr(b),
            y.data_ptr(), _err_flag(x.device).data_ptr(), _C.stream_ptr(x2))
    return y.reshape(*x.shape[:-1], N)


class _BaseLinear(torch.autograd.Function):
    """y = x @ W_base^T + bias; the base is frozen, so the backward returns
    the gradients of x (through the dequantized base) and of the bias."""

    @staticmethod
    def forward(ctx, x, bias, ql):
        ctx.ql = ql
        return _forward(ql, x, bias)

    @staticmethod
    def backward(ctx, gy):
        ql = ctx.ql
        N, K = ql.out_features, ql.in_features
        g2 = gy.reshape(-1, N)
        gx = gb = None
        if ctx.needs_input_grad[0]:
            gx = (g2 @ ql._dequantize_base().to(gy.dtype)).reshape(*gy.shape[:-1], K)
        if ctx.needs_input_grad[1]:
            gb = g2.float().sum(0)
        return gx, gb, None


def base_linear(ql, x: torch.Tensor) -> torch.Tensor:
    """The fused base product (+ bias) of QLoRALinear for eligible x."""
    if torch.is_grad_enabled() and (x.requires_grad or (ql.bias is not None and ql.bias.requires_grad)):
        return _BaseLinear.apply(x, ql.bias, ql)
    return _forward(ql, x, ql.bias)


# ──────────────────────────────────────────────────────────────────────────────
# LoRA fused into the base product (qlora.py:306-312) and merge_lora
# (qlora.py:314-317)
# ──────────────────────────────────────────────────────────────────────────────

def lora_fusable(ql, x: torch.Tensor) -> bool:
    """The kernels take the LoRA term for an even rank up to 16 (tensor-core
    path, more than 8 tokens) or 64 (weight-streaming path, up to 8)."""
    r = ql.rank
    m = x.numel() // ql.in_features if ql.in_features else 0
    return r >= 2 and r % 2 == 0 and r <= (64 if m <= 8 else 16)


def _lora_u(ql, x2: torch.Tensor, lora_a: torch.Tensor) -> torch.Tensor:
    """u = scaling * x @ lora_A^T in the activations' dtype, rows padded with
    zeros to 64 columns (the kernels' row pitch): one lq_lora_u launch on
    lora_A cast to the activations' dtype (cached while lora_A is unchanged)."""
    a = _cast_cached(ql, "_lora_a_cast", lora_a, x2.dtype)
    u = torch.empty(x2.shape[0], 64, dtype=x2.dtype, device=x2.device)
    _C.call("lq_lora_u", x2.data_ptr(), _C.dt(x2), x2.shape[0], ql.in_features, a.data_ptr(), _C.dt(a),
            ql.rank, float(ql.scaling), u.data_ptr(), _C.stream_ptr(x2))
    return u


def _cast_cached(ql, slot: str, src: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """src in `dtype`, contiguous and 16-byte aligned: cast once and kept
    while src is unchanged (same storage, same in-place version counter; the
    cache holds the source, so its address cannot be reused meanwhile)."""
    if src.dtype == dtype and src.is_contiguous() and src.data_ptr() % 16 == 0:
        return src
    key = (src.data_ptr(), src._version, dtype, tuple(src.shape), src.stride())
    cached = getattr(ql, slot, None)
    if cached is not None and cached[0] == key:
        return cached[2]
    t = src.to(dtype).contiguous()
    setattr(ql, slot, (key, src, t))
    return t


def _lora_b(ql, lora_b: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """lora_B in the activations' dtype (the kernels' A operand of the LoRA step)."""
    return _cast_cached(ql, "_lora_b_cast", lora_b, dtype)


def _lora_forward(ql, x: torch.Tensor, lora_a, lora_b, bias) -> torch.Tensor:
    packed = packed_operand(ql, x.dtype)
    N, K = ql.out_features, ql.in_features
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty(M, N, dtype=x.dtype, device=x.device)
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != torch.float32 or not b.is_contiguous():
            b = b.float().contiguous()
    # u = scaling * x @ lora_A^T and the fused kernel, the second started
    # behind the first (lq_nf4_qlora_forward)
    a = _cast_cached(ql, "_lora_a_cast", lora_a.detach(), x2.dtype)
    lb = _lora_b(ql, lora_b.detach(), x.dtype)
    u = torch.empty(M, 64, dtype=x2.dtype, device=x2.device)
    _C.call("lq_nf4_qlora_forward", x2.data_ptr(), _C.dt(x2), M, N, K, packed.data_ptr(), _C.ptr(b),
            a.data_ptr(), _C.dt(a), lb.data_ptr(), ql.rank, float(ql.scaling), u.data_ptr(), y.data_ptr(),
            _err_flag(x.device).data_ptr(), _C.stream_ptr(x2))
    return y.reshape(*x.shape[:-1], N)


class _QLoRAFused(torch.autograd.Function):
    """y = x @ W_base^T + bias + scaling * (x @ A^T) @ B^T in one kernel; the
    backward (frozen base) gives the gradients of x, lora_A, lora_B, bias."""

    @staticmethod
    def forward(ctx, x, lora_a, lora_b, bias, ql):
        ctx.ql = ql
        ctx.save_for_backward(x, lora_a, lora_b)
        ctx.has_bias = bias is not None
        return _lora_forward(ql, x, lora_a, lora_b, bias)

    @staticmethod
    def backward(ctx, gy):
        x, lora_a, lora_b = ctx.saved_tensors
        ql = ctx.ql
        N, K, s = ql.out_features, ql.in_features, ql.scaling
        g2 = gy.reshape(-1, N)
        x2 = x.reshape(-1, K)
        a = lora_a.to(gy.dtype)
        b = lora_b.to(gy.dtype)
        gbp = g2 @ b  # [M, r]
        gx = ga = gb = gbias = None
        if ctx.needs_input_grad[0]:
            gx = (g2 @ ql._dequantize_base().to(gy.dtype) + (gbp @ a) * s).reshape(*gy.shape[:-1], K)
        if ctx.needs_input_grad[1]:
            ga = ((gbp * s).t() @ x2).to(lora_a.dtype)
        if ctx.needs_input_grad[2]:
            gb = ((g2.t() @ (x2 @ a.t())) * s).to(lora_b.dtype)
        if ctx.has_bias and ctx.needs_input_grad[3]:
            gbias = g2.float().sum(0)
        return gx, ga, gb, gbias, None


def qlora_forward(ql, x: torch.Tensor) -> torch.Tensor:
    """QLoRALinear.forward for eligible x with the LoRA term fused."""
    if (torch.is_grad_enabled() and (x.requires_grad or ql.lora_A.requires_grad
                                     or ql.lora_B.requires_grad
                                     or (ql.bias is not None and ql.bias.requires_grad))):
        return _QLoRAFused.apply(x, ql.lora_A, ql.lora_B, ql.bias, ql)
    return _lora_forward(ql, x, ql.lora_A, ql.lora_B, ql.bias)


def merge_fusable(ql) -> bool:
    a, b = ql.lora_A, ql.lora_B
    return (ql.nf4_codes_packed.is_cuda and a.is_cuda and b.is_cuda and a.dtype == b.dtype
            and a.dtype in (torch.float32, torch.float16, torch.bfloat16)
            and 1 <= ql.rank <= 64 and ql.in_features % 8 == 0
            and ql.nf4_codes_packed.data_ptr() % 4 == 0)


def _merge(ql, lora_a, lora_b) -> torch.Tensor:
    N, K = ql.out_features, ql.in_features
    codes = ql.nf4_codes_packed
    ref = ql.dq_q_scales if _use_dq(ql) else ql.nf4_scales
    out_dtype = torch.promote_types(ref.dtype, lora_a.dtype)
    out = torch.empty(N, K, dtype=out_dtype, device=codes.device)
    a = lora_a.detach().contiguous()
    b = lora_b.detach().contiguous()
    if _use_dq(ql):
        qs = ql.dq_q_scales.contiguous()
        dq = ql.dq_scales.to(qs.dtype).contiguous()
        _C.call("lq_nf4_merge_lora", codes.data_ptr(), N, K, ql.group_size, ql._dq_gs, None,
                qs.data_ptr(), dq.data_ptr(), _C.dt(qs), a.data_ptr(), b.data_ptr(), _C.dt(a),
                ql.rank, ql.scaling, out.data_ptr(), _C.dt(out), _C.stream_ptr(codes))
    else:
        s = ql.nf4_scales.contiguous()
        _C.call("lq_nf4_merge_lora", codes.data_ptr(), N, K, ql.group_size, 0, s.data_ptr(), None,
                None, _C.dt(s), a.data_ptr(), b.data_ptr(), _C.dt(a), ql.rank, ql.scaling,
                out.data_ptr(), _C.dt(out), _C.stream_ptr(codes))
    return out


class _MergeLora(torch.autograd.Function):
    """W_base + scaling * B @ A in one pass; gradients reach lora_A / lora_B."""

    @staticmethod
    def forward(ctx, lora_a, lora_b, ql):
        ctx.save_for_backward(lora_a, lora_b)
        ctx.scaling = ql.scaling
        return _merge(ql, lora_a, lora_b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        s = ctx.scaling
        ga = gb = None
        if ctx.needs_input_grad[0]:
            ga = ((b.t().to(g.dtype) @ g) * s).to(a.dtype)
        if ctx.needs_input_grad[1]:
            gb = ((g @ a.t().to(g.dtype)) * s).to(b.dtype)
        return ga, gb, None


def merge_lora(ql) -> torch.Tensor:
    if torch.is_grad_enabled() and (ql.lora_A.requires_grad or ql.lora_B.requires_grad):
        return _MergeLora.apply(ql.lora_A, ql.lora_B, ql)
    return _merge(ql, ql.lora_A, ql.lora_B)
