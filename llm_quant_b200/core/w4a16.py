"""W4A16 dispatch for QuantizedLinear.forward on the tensor cores.

Used when the activations are float16 / bfloat16 and the layer holds
group-quantized codes of at most 4 bits with a group size that is a multiple
of 64, in_features % 64 == 0 and out_features % 128 == 0 (the Llama-style
projection shapes).  The packed operand (4-bit codes in the kernel's tile
order + per-group (zero, scale) pairs) is built once per activation dtype
and cached on the module; it is dropped whenever the weights change.
"""

from __future__ import annotations

import torch

from .. import _C

_ERR = {}


def _err_flag(device) -> torch.Tensor:
    t = _ERR.get(device)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[device] = t
    return t


def check_error_flag(device) -> int:
    """Non-zero if a W4A16 launch on `device` hit a device-side wait timeout
    (reads the flag: synchronizes the device)."""
    t = _ERR.get(device)
    return 0 if t is None else int(t.item())


def eligible(ql, x: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)
            and ql.weight_int.is_cuda and ql.n_bits <= 4 and ql.group_size > 0
            and ql.group_size % 64 == 0 and ql.in_features % ql.group_size == 0
            and ql.in_features % 64 == 0 and ql.out_features % 128 == 0
            and x.shape[-1] == ql.in_features
            and ql.scale.dim() == 2 and ql.scale.shape[1] == ql.in_features // ql.group_size)


def packed_operand(ql, act_dtype: torch.dtype) -> torch.Tensor:
    """Build (or fetch the cached) packed weight operand for `act_dtype`."""
    dev = ql.weight_int.device
    cached = ql._w4
    if cached is not None and cached[0] == act_dtype and cached[1] == dev:
        return cached[2]
    N, K, G = ql.out_features, ql.in_features, ql.group_size
    nbytes = _C.lib().lq_w4a16_packed_bytes(N, K, G)
    packed = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    wi = ql.weight_int.contiguous()
    s = ql.scale.contiguous()
    z = ql.zero_point.to(s.dtype).contiguous()
    _C.call("lq_w4a16_pack", wi.data_ptr(), s.data_ptr(), z.data_ptr(), _C.dt(s), N, K, G,
            int(ql.symmetric), _C.dt(act_dtype), packed.data_ptr(), _C.stream_ptr(wi))
    ql._w4 = (act_dtype, dev, packed)
    return packed


def fp32_bias(ql):
    """The layer's bias as the kernels take it (fp32, contiguous), converted
    once and kept while the bias is unchanged (same storage, same in-place
    version counter; the cache holds the source, so its address cannot be
    reused meanwhile).  None without a bias."""
    b = ql.bias
    if b is None:
        return None
    b = b.detach()
    if b.dtype == torch.float32 and b.is_contiguous():
        return b
    key = (b.data_ptr(), b._version, tuple(b.shape), b.stride())
    cached = getattr(ql, "_bias_f32", None)
    if cached is not None and cached[0] == key:
        return cached[2]
    t = b.float().contiguous()
    ql._bias_f32 = (key, b, t)
    return t


def linear(ql, x: torch.Tensor) -> torch.Tensor:
    """y = x @ dequant(W)^T + bias with the fused W4A16 kernel."""
    packed = packed_operand(ql, x.dtype)
    N, K = ql.out_features, ql.in_features
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty(M, N, dtype=x.dtype, device=x.device)
    bias = fp32_bias(ql)
    _C.call("lq_w4a16_linear", x2.data_ptr(), _C.dt(x2), M, N, K, ql.group_size,
            packed.data_ptr(), _C.ptr(bias), y.data_ptr(), _err_flag(x.device).data_ptr(),
            _C.stream_ptr(x2))
    return y.reshape(*x.shape[:-1], N)
