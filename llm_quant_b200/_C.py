"""ctypes binding of liblq_sm100.so (the C ABI in include/lq_sm100.h).

There is no CPU or pure-PyTorch fallback: if the library is missing, or a
tensor given to a hot-path function is not on a CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "liblq_sm100.so")

# lq_dtype codes
F32, F16, BF16, I8, I16, I32, I64, U8, U4X2 = range(9)
# lq_mode
MODE_QPARAMS, MODE_FAKE, MODE_CODES = 0, 1, 2
# lq_affine_op
AFFINE_QUANT, AFFINE_DEQUANT, AFFINE_FAKE = 0, 1, 2
# status
OK, EINVAL, EDTYPE, ECUDA, ETIMEOUT, EALIGN, ERANGE = 0, -1, -2, -3, -4, -5, -6

TORCH_TO_LQ = {
    torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int8: I8,
    torch.int16: I16, torch.int32: I32, torch.int64: I64, torch.uint8: U8,
}
FLOAT_TYPES = (torch.float32, torch.float16, torch.bfloat16)


class LQError(RuntimeError):
    """A CUDA-side failure reported by liblq_sm100 (status code + message)."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: {msg} (status {status})")
        self.status = status


_V = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_PL = ctypes.POINTER(ctypes.c_int64)
_PI = ctypes.POINTER(ctypes.c_int)

_SIGS = {
    "lq_group_quant": [_V, _I, _L, _L, _L, _I, _I, _I, _V, _I, _V, _V, _V],
    "lq_token_group_quant": [_V, _I, _L, _L, _L, _L, _I, _I, _I, _V, _I, _V, _V, _V],
    "lq_kv_dequant": [_V, _I, _L, _L, _L, _L, _I, _L, _V, _V, _I, _L, _V, _V],
    "lq_kv_append": [_V, _I, _L, _L, _L, _I, _L, _I, _I, _V, _I, _L, _L, _V, _V, _L, _L, _I, _V],
    "lq_tensor_qparams": [_V, _I, _L, _I, _I, _V, _V, _V, ctypes.c_size_t, _V],
    "lq_channel_qparams": [_V, _I, _L, _L, _L, _I, _I, _V, _V, _V, ctypes.c_size_t, _V],
    "lq_affine": [_I, _I, _PL, _V, _I, _PL, _V, _I, _PL, _V, _I, _PL, _PI, _I, _I, _V, _I, _V],
    "lq_ste_round": [_V, _I, _L, _V, _V],
    "lq_fake_quant_backward": [_V, _V, _I, _L, _L, _L, _I, _I, _V, _V],
    "lq_nf4_quantize": [_V, _I, _L, _L, _V, _I, _V, _V],
    "lq_nf4_dequantize": [_V, _I, _L, _L, _V, _I, _V, _V],
    "lq_double_quantize": [_V, _I, _L, _L, _V, _V, _V],
    "lq_double_dequantize": [_V, _V, _I, _L, _L, _V, _V],
    "lq_codes_convert": [_V, _I, _L, _V, _I, _V],
    "lq_nf4_pack": [_V, _I, _L, _L, _L, _V, _V, _V, _V, _V],
    "lq_nf4_unpack": [_V, _L, _L, _L, _V, _V, _V, _I, _V, _V],
    "lq_hadamard": [_V, _I, _L, _L, _V, _V],
    "lq_hadamard_fake_quant": [_V, _I, _L, _L, _I, _I, _V, _V, _V, _V],
    "lq_w4a16_pack": [_V, _V, _V, _I, _L, _L, _L, _I, _I, _V, _V],
    "lq_w4a16_linear": [_V, _I, _L, _L, _L, _L, _V, _V, _V, _V, _V],
    "lq_nf4_linear_pack": [_V, _V, _V, _V, _I, _L, _L, _L, _L, _I, _V, _V],
    "lq_nf4_linear": [_V, _I, _L, _L, _L, _V, _V, _V, _V, _V],
    "lq_nf4_linear_lora": [_V, _I, _L, _L, _L, _V, _V, _V, _V, _L, _V, _V, _V],
    "lq_lora_u": [_V, _I, _L, _L, _V, _I, _L, ctypes.c_float, _V, _V],
    "lq_nf4_qlora_forward": [_V, _I, _L, _L, _L, _V, _V, _V, _I, _V, _L, ctypes.c_float, _V, _V, _V, _V],
    "lq_nf4_merge_lora": [_V, _L, _L, _L, _L, _V, _V, _V, _I, _V, _V, _I, _L, ctypes.c_float,
                          _V, _I, _V],
    "lq_sparse_row_add": [_V, _I, _L, _L, _L, _V, _V, _L, _V, _V, _V, _V],
    "lq_wait_probe": [_L, _I, _V, _V],
    "lq_kv_attention": [_V, _I, _L, _L, _L, _L, _L, _L, _L, _I,
                        _V, _I, _L, _V, _V, _L,
                        _V, _I, _L, _V, _V, _L,
                        _I, ctypes.c_float, _I, _V, _V, ctypes.c_size_t, _V],
}
_SIZE_SIGS = {
    "lq_tensor_qparams_workspace_size": [_L],
    "lq_channel_qparams_workspace_size": [_L, _L, _L],
    "lq_w4a16_packed_bytes": [_L, _L, _L],
    "lq_nf4_linear_packed_bytes": [_L, _L],
    "lq_kv_attention_workspace_bytes": [_L, _L, _L, _L, _L, _L],
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load liblq_sm100.so once; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python -m llm_quant_b200.build` "
                    "(there is no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, args in _SIGS.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.argtypes = args
                fn.restype = ctypes.c_int
            for name, args in _SIZE_SIGS.items():
                fn = getattr(L, name, None)
                if fn is not None:
                    fn.argtypes = args
                    fn.restype = ctypes.c_size_t
            L.lq_last_error.restype = ctypes.c_char_p
            L.lq_status_string.restype = ctypes.c_char_p
            L.lq_launch_count.restype = ctypes.c_uint64
            _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point and turn a non-zero status into an exception."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        msg = lib().lq_last_error().decode(errors="replace")
        if rc in (EINVAL, ERANGE):
            raise ValueError(f"{name}: {msg}")
        if rc == EDTYPE:
            raise TypeError(f"{name}: {msg}")
        raise LQError(name, rc, msg)


def launch_count() -> int:
    return int(lib().lq_launch_count())


def stream_ptr(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def dt(t_or_dtype) -> int:
    d = t_or_dtype.dtype if isinstance(t_or_dtype, torch.Tensor) else t_or_dtype
    try:
        return TORCH_TO_LQ[d]
    except KeyError:
        raise TypeError(f"unsupported dtype {d}") from None


def require_cuda(*tensors: torch.Tensor, what: str = "llm_quant_b200") -> None:
    """The hot path runs only on CUDA tensors; there is no CPU fallback."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{what}: expected a CUDA tensor, got device {t.device} "
                "(llm_quant_b200 has no CPU implementation)")


def check_clamp_bounds(dtype: torch.dtype, n_bits: int, symmetric: bool) -> None:
    """torch.clamp converts its scalar bounds to the tensor's dtype and raises
    when a bound overflows it, which for the code range means an fp16 tensor
    with qmax = 2^16 - 1 (asymmetric 16-bit); the reference fails there, so
    this layer does too, with torch's message."""
    if dtype != torch.float16:
        return
    qmin, qmax = (-(2 ** (n_bits - 1)), 2 ** (n_bits - 1) - 1) if symmetric else (0, 2 ** n_bits - 1)
    if max(abs(qmin), abs(qmax)) > 65519:
        raise RuntimeError("value cannot be converted to type c10::Half without overflow")


def require_float(t: torch.Tensor, what: str) -> None:
    if t.dtype not in FLOAT_TYPES:
        raise TypeError(f"{what}: unsupported dtype {t.dtype} (float32, float16, bfloat16)")


def i64_array(vals):
    arr = (ctypes.c_int64 * max(1, len(vals)))(*vals)
    return ctypes.cast(arr, _PL), arr


def int_array(vals):
    arr = (ctypes.c_int * max(1, len(vals)))(*vals)
    return ctypes.cast(arr, _PI), arr
