"""llm_quant_b200.qlora -- NF4 quantization behind QLoRA, on B200.

Same API as llm_quant.qlora (qlora.py of MindIntels/llm_quant).  The NF4
encoder reproduces the reference's ``argmin |x/scale - NF4_TABLE|`` (fp32
differences, first minimum) bit for bit.

QLoRALinear keeps its frozen base weight as packed 4-bit codes on the device
(``nf4_codes_packed``, two codes per byte) -- 16x less memory than the
reference's int64 ``nf4_codes`` buffer.  ``nf4_codes`` is still available as
an int64 tensor (unpacked on access) and is what ``state_dict()`` saves and
``load_state_dict()`` accepts, so checkpoints are interchangeable.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _C

# 16-level NormalFloat table (qlora.py:43-59), float32.
NF4_TABLE = torch.tensor([
    -1.0000, -0.6962, -0.5251, -0.3949,
    -0.2844, -0.1848, -0.0911, 0.0000,
    0.0796, 0.1609, 0.2461, 0.3379,
    0.4407, 0.5626, 0.7230, 1.0000,
])


def _n_groups(n: int, g: int) -> int:
    return (n + g - 1) // g


def nf4_quantize(x: torch.Tensor, group_size: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """NF4 codes (int64, x's shape) and per-block absmax scales [n_groups] in
    x's dtype (qlora.py:66-110).  Blocks run over the flattened tensor; the
    last block is zero-padded."""
    _C.require_cuda(x, what="nf4_quantize")
    _C.require_float(x, "nf4_quantize")
    xc = x.detach().contiguous()
    n = xc.numel()
    codes = torch.empty(x.shape, dtype=torch.int64, device=x.device)
    scales = torch.empty(_n_groups(n, group_size), dtype=x.dtype, device=x.device)
    _C.call("lq_nf4_quantize", xc.data_ptr(), _C.dt(xc), n, group_size, codes.data_ptr(),
            _C.I64, scales.data_ptr(), _C.stream_ptr(xc))
    return codes, scales


def nf4_dequantize(
    codes: torch.Tensor,
    scales: torch.Tensor,
    group_size: int = 64,
    orig_shape: Optional[tuple] = None,
) -> torch.Tensor:
    """``NF4_TABLE.to(scales.dtype)[codes] * scales`` per block (qlora.py:113-157)."""
    _C.require_cuda(codes, scales, what="nf4_dequantize")
    _C.require_float(scales, "nf4_dequantize")
    c = codes.detach()
    if c.dtype not in (torch.int64, torch.uint8):
        c = c.to(torch.int64)
    c = c.contiguous()
    s = scales.detach().contiguous()
    n = c.numel()
    if _n_groups(n, group_size) > s.numel():
        raise IndexError(f"nf4_dequantize: {s.numel()} scales for {_n_groups(n, group_size)} blocks")
    out = torch.empty(orig_shape if orig_shape is not None else codes.shape, dtype=s.dtype,
                      device=s.device)
    if out.numel() != n:
        raise RuntimeError(f"shape '{list(out.shape)}' is invalid for input of size {n}")
    _C.call("lq_nf4_dequantize", c.data_ptr(), _C.dt(c), n, group_size, s.data_ptr(), _C.dt(s),
            out.data_ptr(), _C.stream_ptr(s))
    return out


def double_quantize(
    scales: torch.Tensor,
    dq_group_size: int = 256,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Second-level 8-bit quantization of the block scales (qlora.py:164-196):
    ``q = round(s / absmax * 127).clamp(-127, 127)`` stored in the scales' dtype,
    plus the per-group absmax [ceil(n / dq_group_size)]."""
    _C.require_cuda(scales, what="double_quantize")
    _C.require_float(scales, "double_quantize")
    s = scales.detach().contiguous().reshape(-1)
    n = s.numel()
    q = torch.empty(n, dtype=s.dtype, device=s.device)
    dq = torch.empty(_n_groups(n, dq_group_size), dtype=s.dtype, device=s.device)
    _C.call("lq_double_quantize", s.data_ptr(), _C.dt(s), n, dq_group_size, q.data_ptr(),
            dq.data_ptr(), _C.stream_ptr(s))
    return q, dq


def double_dequantize(
    q_scales: torch.Tensor,
    dq_scales: torch.Tensor,
    dq_group_size: int = 256,
) -> torch.Tensor:
    """``(q / 127) * dq`` per group of scales (qlora.py:199-223)."""
    _C.require_cuda(q_scales, dq_scales, what="double_dequantize")
    _C.require_float(q_scales, "double_dequantize")
    q = q_scales.detach().contiguous().reshape(-1)
    d = dq_scales.detach().to(q.dtype).contiguous().reshape(-1)
    n = q.numel()
    out = torch.empty(n, dtype=q.dtype, device=q.device)
    _C.call("lq_double_dequantize", q.data_ptr(), d.data_ptr(), _C.dt(q), n, dq_group_size,
            out.data_ptr(), _C.stream_ptr(q))
    return out


def codes_to(codes: torch.Tensor, n: int, container: str, packed_src: bool = False) -> torch.Tensor:
    """Convert n NF4 codes between int64 ('i64'), uint8 ('u8') and packed
    ('u4', two per byte) containers; ``packed_src`` marks a packed source."""
    if packed_src:
        src_dt = _C.U4X2
    elif codes.dtype in (torch.int64, torch.uint8):
        src_dt = _C.dt(codes)
    else:
        codes = codes.to(torch.int64)
        src_dt = _C.I64
    src = codes.detach().contiguous()
    if container == "u4":
        out = torch.empty((n + 1) // 2, dtype=torch.uint8, device=codes.device)
        ddt = _C.U4X2
    elif container == "u8":
        out = torch.empty(n, dtype=torch.uint8, device=codes.device)
        ddt = _C.U8
    else:
        out = torch.empty(n, dtype=torch.int64, device=codes.device)
        ddt = _C.I64
    _C.call("lq_codes_convert", src.data_ptr(), src_dt, n, out.data_ptr(), ddt, _C.stream_ptr(src))
    return out


class QLoRALinear(nn.Module):
    """Frozen NF4 base weight + trainable LoRA adapters (qlora.py:230-324).

    ``forward(x) = x @ W_base^T + bias + (x @ A^T @ B^T) * alpha / rank``.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        rank: int = 16,
        alpha: float = 16.0,
        group_size: int = 64,
        double_quant: bool = True,
        bias: bool = True,
    ):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.rank = rank
        self.alpha = alpha
        self.group_size = group_size
        self.double_quant = double_quant
        self.scaling = alpha / rank

        n = out_features * in_features
        # packed NF4 codes, element 2i in the low nibble (not in state_dict:
        # the int64 ``nf4_codes`` entry is written / read by the hooks below)
        self.register_buffer("nf4_codes_packed", torch.zeros((n + 1) // 2, dtype=torch.uint8),
                             persistent=False)
        self.register_buffer("nf4_scales", torch.ones(1))
        if double_quant:
            self.register_buffer("dq_q_scales", torch.ones(1))
            self.register_buffer("dq_scales", torch.ones(1))
            self.register_buffer("dq_group_size_val", torch.tensor(256, dtype=torch.long))
            self._dq_gs = 256

        self.lora_A = nn.Parameter(torch.empty(rank, in_features))
        self.lora_B = nn.Parameter(torch.zeros(out_features, rank))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))

        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None

    # -- int64 view of the codes (state_dict compatible) ----------------------
    @property
    def nf4_codes(self) -> torch.Tensor:
        n = self.out_features * self.in_features
        return codes_to(self.nf4_codes_packed, n, "i64", packed_src=True).reshape(
            self.out_features, self.in_features)

    @nf4_codes.setter
    def nf4_codes(self, codes: torch.Tensor) -> None:
        n = self.out_features * self.in_features
        self.nf4_codes_packed = codes_to(codes.reshape(-1), n, "u4")

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        destination[prefix + "nf4_codes"] = self.nf4_codes

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        key = prefix + "nf4_codes"
        codes = state_dict.pop(key, None) if key in state_dict else None
        # the reference rebinds these buffers in pack_base, so their shapes
        # follow the weight: resize ours before the default copy
        for name in ("nf4_scales", "dq_q_scales", "dq_scales"):
            k = prefix + name
            if k in state_dict and hasattr(self, name):
                cur = getattr(self, name)
                v = state_dict[k]
                if cur.shape != v.shape or cur.dtype != v.dtype:
                    setattr(self, name, torch.empty(v.shape, dtype=v.dtype, device=cur.device))
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)
        if codes is not None:
            state_dict[key] = codes
            dev = self.nf4_codes_packed.device
            self.nf4_codes = codes.to(dev)
        elif strict:
            missing_keys.append(key)
        if self.double_quant and hasattr(self, "dq_group_size_val"):
            self._dq_gs = int(self.dq_group_size_val.item())

    @torch.no_grad()
    def pack_base(self, weight: torch.Tensor) -> None:
        """NF4-quantize and store the base weight (qlora.py:281-292): codes,
        block scales and (double_quant) q_scales / dq_scales in one pass."""
        _C.require_cuda(weight, what="QLoRALinear.pack_base")
        _C.require_float(weight, "QLoRALinear.pack_base")
        w = weight.detach().contiguous()
        n = w.numel()
        gs = self.group_size
        ng = _n_groups(n, gs)
        packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=w.device)
        scales = torch.empty(ng, dtype=w.dtype, device=w.device)
        if self.double_quant:
            dq_gs = self._dq_gs
            q_scales = torch.empty(ng, dtype=w.dtype, device=w.device)
            dq_scales = torch.empty(_n_groups(ng, dq_gs), dtype=w.dtype, device=w.device)
            try:
                _C.call("lq_nf4_pack", w.data_ptr(), _C.dt(w), n, gs, dq_gs, packed.data_ptr(),
                        scales.data_ptr(), q_scales.data_ptr(), dq_scales.data_ptr(),
                        _C.stream_ptr(w))
            except (ValueError, _C.LQError) as e:
                if isinstance(e, _C.LQError) and e.status != _C.EALIGN:
                    raise
                # group sizes / alignments the fused kernel does not tile: two passes
                _C.call("lq_nf4_quantize", w.data_ptr(), _C.dt(w), n, gs, packed.data_ptr(),
                        _C.U4X2, scales.data_ptr(), _C.stream_ptr(w))
                q_scales, dq_scales = double_quantize(scales, dq_gs)
            self.dq_q_scales = q_scales
            self.dq_scales = dq_scales
        else:
            _C.call("lq_nf4_quantize", w.data_ptr(), _C.dt(w), n, gs, packed.data_ptr(), _C.U4X2,
                    scales.data_ptr(), _C.stream_ptr(w))
        self.nf4_codes_packed = packed
        self.nf4_scales = scales

    def _dequantize_base(self) -> torch.Tensor:
        """The base weight in the scales' dtype (qlora.py:294-304); double
        dequantization of the scales is fused into the same pass."""
        n = self.out_features * self.in_features
        codes = self.nf4_codes_packed
        _C.require_cuda(codes, what="QLoRALinear._dequantize_base")
        use_dq = self.double_quant and hasattr(self, "dq_q_scales")
        ref = self.dq_q_scales if use_dq else self.nf4_scales
        out = torch.empty(self.out_features, self.in_features, dtype=ref.dtype, device=codes.device)
        if use_dq:
            dq = self.dq_scales.to(ref.dtype).contiguous()
            _C.call("lq_nf4_unpack", codes.data_ptr(), n, self.group_size, self._dq_gs, None,
                    self.dq_q_scales.contiguous().data_ptr(), dq.data_ptr(), _C.dt(ref),
                    out.data_ptr(), _C.stream_ptr(codes))
        else:
            _C.call("lq_nf4_unpack", codes.data_ptr(), n, self.group_size, 0,
                    self.nf4_scales.contiguous().data_ptr(), None, None, _C.dt(ref),
                    out.data_ptr(), _C.stream_ptr(codes))
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """qlora.py:306-312.  fp16 / bf16 activations of the base weight's dtype
        take the fused NF4 kernel for the base product (the reference fails
        there: its bias and LoRA factors stay fp32), with the LoRA path in the
        activations' dtype; other inputs follow the reference exactly."""
        from . import nf4_linear
        if nf4_linear.eligible(self, x):
            if nf4_linear.lora_fusable(self, x):
                # base product, bias and the rank-r LoRA term in one kernel
                return nf4_linear.qlora_forward(self, x)
            out = nf4_linear.base_linear(self, x)
            lora = F.linear(F.linear(x, self.lora_A.to(x.dtype)), self.lora_B.to(x.dtype))
            return out + lora * self.scaling
        w_base = self._dequantize_base()
        out = F.linear(x, w_base, self.bias)
        out = out + F.linear(F.linear(x, self.lora_A), self.lora_B) * self.scaling
        return out

    def merge_lora(self) -> torch.Tensor:
        """W_eff = W_base + scaling * B @ A (qlora.py:314-317): one kernel that
        dequantizes the base and adds the rank-r update (in the promoted dtype,
        each op rounded as torch does); gradients still reach lora_A / lora_B."""
        from . import nf4_linear
        if nf4_linear.merge_fusable(self):
            return nf4_linear.merge_lora(self)
        w_base = self._dequantize_base()
        return w_base + self.scaling * (self.lora_B @ self.lora_A)

    def extra_repr(self) -> str:
        return (
            f"in={self.in_features}, out={self.out_features}, "
            f"rank={self.rank}, alpha={self.alpha}, "
            f"group={self.group_size}, double_quant={self.double_quant}"
        )


class QLoRA:
    """High-level QLoRA pipeline (qlora.py:331-372)."""

    def __init__(
        self,
        rank: int = 16,
        alpha: float = 16.0,
        group_size: int = 64,
        double_quant: bool = True,
    ):
        self.rank = rank
        self.alpha = alpha
        self.group_size = group_size
        self.double_quant = double_quant

    def wrap_linear(self, linear: nn.Linear) -> QLoRALinear:
        """Wrap an nn.Linear as a QLoRALinear on the linear's device."""
        ql = QLoRALinear(
            linear.in_features,
            linear.out_features,
            rank=self.rank,
            alpha=self.alpha,
            group_size=self.group_size,
            double_quant=self.double_quant,
            bias=linear.bias is not None,
        ).to(linear.weight.device)
        ql.pack_base(linear.weight.data)
        if linear.bias is not None:
            ql.bias.data.copy_(linear.bias.data)
        return ql

    def trainable_params(self, module: nn.Module) -> list[nn.Parameter]:
        """Only the trainable (LoRA) parameters."""
        return [p for p in module.parameters() if p.requires_grad]
