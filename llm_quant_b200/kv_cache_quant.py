"""llm_quant_b200.kv_cache_quant -- KV-cache quantization on B200.

Same API as llm_quant.kv_cache_quant (kv_cache_quant.py of
MindIntels/llm_quant): codes, scales, zero points and dequantized values are
bit-identical to the reference on the same inputs.

QuantizedKVCache stores each layer's codes in device buffers with spare
capacity (grown geometrically, or sized once by ``max_seq_len``), so an
``update`` quantizes only the new chunk straight into place (one kernel per
K / V) instead of concatenating the whole cache; the full dequantized K and
V it returns are written by one more kernel each.  Semantics follow the
reference, including its PER_CHANNEL scale merge with ``torch.maximum``
that does not requantize earlier codes (kv_cache_quant.py:395-402).

Beyond the reference: ``QuantizedKVCache.append`` stores a chunk without
returning the dequantized cache, and ``QuantizedKVCache.attend`` computes
decode attention straight from the stored codes (``lq_kv_attention``), so a
decode step reads the cache once, in its quantized size.
"""

from __future__ import annotations

import math
from enum import Enum
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import _C


class KVQuantGranularity(Enum):
    """Quantization granularity for KV cache (kv_cache_quant.py:55-59)."""
    PER_TOKEN = "per_token"
    PER_CHANNEL = "per_channel"
    PER_GROUP = "per_group"


_GRAN_CODE = {"per_token": 0, "per_channel": 1, "per_group": 2}


def _gran(g) -> str:
    v = g.value if isinstance(g, Enum) else g
    if v not in _GRAN_CODE:
        raise ValueError(f"Unknown granularity: {g}")
    return v


class KVCacheQuantizer:
    """Stateless INT4 / INT8 quantizer for [B, H, T, D] cache tensors
    (kv_cache_quant.py:66-276)."""

    def __init__(
        self,
        n_bits: int = 8,
        symmetric: bool = True,
        granularity: KVQuantGranularity = KVQuantGranularity.PER_TOKEN,
        group_size: int = 32,
    ):
        self.n_bits = n_bits
        self.symmetric = symmetric
        self.granularity = granularity
        self.group_size = group_size
        if symmetric:
            self.qmin = -(2 ** (n_bits - 1))
            self.qmax = 2 ** (n_bits - 1) - 1
        else:
            self.qmin = 0
            self.qmax = 2 ** n_bits - 1

    # -- helpers ---------------------------------------------------------------
    @property
    def _code_dtype(self):
        return torch.int8 if self.symmetric else torch.int16

    def _prep(self, x: torch.Tensor, what: str) -> torch.Tensor:
        _C.require_cuda(x, what=what)
        _C.require_float(x, what)
        _C.check_clamp_bounds(x.dtype, self.n_bits, self.symmetric)
        return x.detach().contiguous()

    def _token_groups(self, x, tgroup, mode, out_dtype):
        """Run the token-axis kernel on x [..., T, D]; tgroup 0 = whole T."""
        P = math.prod(x.shape[:-2])
        T, D = x.shape[-2], x.shape[-1]
        ngt = 1 if tgroup == 0 else math.ceil(T / tgroup)
        scale = torch.empty(*x.shape[:-2], ngt, D, dtype=x.dtype, device=x.device)
        zp = torch.empty_like(scale)
        out = None
        if mode != _C.MODE_QPARAMS:
            out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
        _C.call("lq_token_group_quant", x.data_ptr(), _C.dt(x), P, T, D, tgroup, self.n_bits,
                int(self.symmetric), mode, _C.ptr(out), _C.dt(out_dtype) if out is not None else 0,
                scale.data_ptr(), zp.data_ptr(), _C.stream_ptr(x))
        return out, scale, zp

    def _per_token(self, x, mode, out_dtype):
        D = x.shape[-1]
        rows = x.numel() // max(1, D)
        scale = torch.empty(*x.shape[:-1], 1, dtype=x.dtype, device=x.device)
        zp = torch.empty_like(scale)
        out = None
        if mode != _C.MODE_QPARAMS:
            out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
        _C.call("lq_group_quant", x.data_ptr(), _C.dt(x), rows, D, max(1, D), self.n_bits,
                int(self.symmetric), mode, _C.ptr(out), _C.dt(out_dtype) if out is not None else 0,
                scale.data_ptr(), zp.data_ptr(), _C.stream_ptr(x))
        return out, scale, zp

    def _check_reduce(self, x: torch.Tensor, g: str) -> None:
        """The reference reduces with torch.amin / amax over the head dim
        (per-token) or the token dim (per-channel), which raises IndexError when
        that dim has size zero."""
        if g == "per_group":
            return
        d = -1 if g == "per_token" else -2
        if x.ndim >= 2 and x.shape[d] == 0:
            op = "amax" if self.symmetric else "amin"
            raise IndexError(f"{op}(): Expected reduction dim {d} to have non-zero size.")

    # -- reference API -----------------------------------------------------------
    def _compute_qparams(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Scale / zero point broadcastable to x (kv_cache_quant.py:102-139)."""
        g = _gran(self.granularity)
        if g == "per_group":
            return self._compute_qparams_grouped(x)
        self._check_reduce(x, g)
        xc = self._prep(x, "KVCacheQuantizer")
        if g == "per_token":
            _, s, z = self._per_token(xc, _C.MODE_QPARAMS, None)
        else:
            _, s, z = self._token_groups(xc, 0, _C.MODE_QPARAMS, None)
        return s, z

    def _compute_qparams_grouped(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """[B, H, n_groups, 1, D] qparams over zero-padded token groups (kv_cache_quant.py:141-166)."""
        B, H, T, D = x.shape
        xc = self._prep(x, "KVCacheQuantizer")
        _, s, z = self._token_groups(xc, self.group_size, _C.MODE_QPARAMS, None)
        return s.unsqueeze(3), z.unsqueeze(3)

    @torch.no_grad()
    def quantize(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(codes int8 | int16, scale, zero_point) (kv_cache_quant.py:168-193)."""
        g = _gran(self.granularity)
        if g == "per_group":
            return self._quantize_grouped(x)
        self._check_reduce(x, g)
        xc = self._prep(x, "KVCacheQuantizer.quantize")
        if g == "per_token":
            return self._per_token(xc, _C.MODE_CODES, self._code_dtype)
        return self._token_groups(xc, 0, _C.MODE_CODES, self._code_dtype)

    def _quantize_grouped(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Per-group codes and [B, H, n_groups, D] qparams (kv_cache_quant.py:195-219)."""
        B, H, T, D = x.shape
        xc = self._prep(x, "KVCacheQuantizer.quantize")
        return self._token_groups(xc, self.group_size, _C.MODE_CODES, self._code_dtype)

    @torch.no_grad()
    def dequantize(self, q: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor) -> torch.Tensor:
        """fp32 ``(q.float() - zp) * scale`` (kv_cache_quant.py:221-243)."""
        g = _gran(self.granularity)
        if g == "per_group":
            return self._dequantize_grouped(q, scale, zp)
        _C.require_cuda(q, scale, zp, what="KVCacheQuantizer.dequantize")
        if q.ndim >= 2 and q.dtype in (torch.int8, torch.int16) and scale.dtype == zp.dtype \
                and scale.dtype in _C.FLOAT_TYPES:
            T, D = q.shape[-2], q.shape[-1]
            lead = tuple(q.shape[:-2])
            gran = None
            if scale.shape == lead + (T, 1) and zp.shape == scale.shape:
                gran, pitch = 0, T
            elif scale.shape == lead + (1, D) and zp.shape == scale.shape:
                gran, pitch = 1, 1
            if gran is not None:
                qc, sc, zc = q.contiguous(), scale.contiguous(), zp.contiguous()
                out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
                _C.call("lq_kv_dequant", qc.data_ptr(), _C.dt(qc), math.prod(lead), T, D, T, gran,
                        1, sc.data_ptr(), zc.data_ptr(), _C.dt(sc), pitch, out.data_ptr(),
                        _C.stream_ptr(qc))
                return out
        # any other broadcast: (q.float() - zp) * scale, fp32 throughout
        from .core.quantizer import _affine
        d0 = torch.result_type(torch.empty(1, dtype=torch.float32, device="meta"), zp)
        nd = len(torch.broadcast_shapes(q.shape, zp.shape))
        d1 = torch.result_type(torch.empty((1,) * nd, dtype=d0, device="meta"), scale)
        return _affine(_C.AFFINE_DEQUANT, q, scale, zp, d0, d1, 8, True, d1)

    def _dequantize_grouped(self, q: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor) -> torch.Tensor:
        """Per-group dequantization (kv_cache_quant.py:245-267): token t uses
        scale group t // group_size."""
        _C.require_cuda(q, scale, zp, what="KVCacheQuantizer.dequantize")
        B, H, T, D = q.shape
        ng = scale.shape[2]
        if ng * self.group_size < T:
            raise RuntimeError(f"shape mismatch: {ng} groups of {self.group_size} < {T} tokens")
        qc = q.contiguous() if q.dtype in (torch.int8, torch.int16) else q.to(torch.int16).contiguous()
        sc = scale.contiguous()
        zc = zp.to(sc.dtype).contiguous()
        out = torch.empty(B, H, T, D, dtype=torch.float32, device=q.device)
        _C.call("lq_kv_dequant", qc.data_ptr(), _C.dt(qc), B * H, T, D, T, 2, self.group_size,
                sc.data_ptr(), zc.data_ptr(), _C.dt(sc), ng, out.data_ptr(), _C.stream_ptr(qc))
        return out

    def fake_quantize(self, x: torch.Tensor) -> torch.Tensor:
        """dequantize(quantize(x)) as fp32 (kv_cache_quant.py:269-276); one pass
        for per-channel / per-group."""
        g = _gran(self.granularity)
        if g == "per_token":
            q, s, z = self.quantize(x)
            return self.dequantize(q, s, z)
        xc = self._prep(x, "KVCacheQuantizer.fake_quantize")
        if self.symmetric and self.n_bits > 8:
            q, s, z = self.quantize(x)
            return self.dequantize(q, s, z)
        out, _, _ = self._token_groups(xc, self.group_size if g == "per_group" else 0,
                                       _C.MODE_FAKE, torch.float32)
        return out


class PerTokenKVCacheQuantizer(KVCacheQuantizer):
    """Per-token granularity (kv_cache_quant.py:283-288)."""

    def __init__(self, n_bits: int = 8, symmetric: bool = True):
        super().__init__(n_bits=n_bits, symmetric=symmetric,
                         granularity=KVQuantGranularity.PER_TOKEN)


class PerChannelKVCacheQuantizer(KVCacheQuantizer):
    """Per-channel granularity (kv_cache_quant.py:291-296)."""

    def __init__(self, n_bits: int = 8, symmetric: bool = True):
        super().__init__(n_bits=n_bits, symmetric=symmetric,
                         granularity=KVQuantGranularity.PER_CHANNEL)


class PerGroupKVCacheQuantizer(KVCacheQuantizer):
    """Per-group-of-tokens granularity (kv_cache_quant.py:299-305)."""

    def __init__(self, n_bits: int = 8, symmetric: bool = True, group_size: int = 32):
        super().__init__(n_bits=n_bits, symmetric=symmetric,
                         granularity=KVQuantGranularity.PER_GROUP,
                         group_size=group_size)


class _CacheSide:
    """Device storage of one side (K or V) of one layer: codes [B, H, cap, D]
    plus scales / zero points laid out for the quantizer's granularity."""

    def __init__(self, qz: KVCacheQuantizer, x: torch.Tensor, reserve: int):
        self.qz = qz
        self.gran = _gran(qz.granularity)
        self.B, self.H, _, self.D = x.shape
        self.dtype, self.device = x.dtype, x.device
        self.code_dtype = qz._code_dtype
        self.T = 0   # tokens stored
        self.ng = 0  # scale rows stored (per-group)
        self.cap = 0
        self.gcap = 0
        self.codes = self.scale = self.zp = None
        self._grow(max(reserve, x.shape[2]), self._groups_for(x.shape[2]))

    def _groups_for(self, tn: int) -> int:
        return math.ceil(tn / self.qz.group_size) if self.gran == "per_group" else 0

    def _grow(self, need_t: int, need_g: int):
        B, H, D = self.B, self.H, self.D
        if need_t > self.cap or self.codes is None:  # storage exists from the first chunk on
            cap = max(need_t, 2 * self.cap, 64)
            cap = (cap + 15) // 16 * 16  # whole 16-token tiles for lq_kv_attention
            codes = torch.empty(B, H, cap, D, dtype=self.code_dtype, device=self.device)
            if self.T:
                codes[:, :, :self.T].copy_(self.codes[:, :, :self.T])
            self.codes = codes
            if self.gran == "per_token":
                s = torch.empty(B, H, cap, 1, dtype=self.dtype, device=self.device)
                z = torch.empty_like(s)
                if self.T:
                    s[:, :, :self.T].copy_(self.scale[:, :, :self.T])
                    z[:, :, :self.T].copy_(self.zp[:, :, :self.T])
                self.scale, self.zp = s, z
            self.cap = cap
        if self.gran == "per_channel" and self.scale is None:
            self.scale = torch.empty(B, H, 1, D, dtype=self.dtype, device=self.device)
            self.zp = torch.empty_like(self.scale)
        if self.gran == "per_group" and need_g > self.gcap:
            gcap = max(need_g, 2 * self.gcap, 4)
            s = torch.empty(B, H, gcap, D, dtype=self.dtype, device=self.device)
            z = torch.empty_like(s)
            if self.ng:
                s[:, :, :self.ng].copy_(self.scale[:, :, :self.ng])
                z[:, :, :self.ng].copy_(self.zp[:, :, :self.ng])
            self.scale, self.zp, self.gcap = s, z, gcap

    def append(self, x: torch.Tensor) -> None:
        _C.require_cuda(x, what="QuantizedKVCache.update")
        if x.ndim != 4 or x.shape[0] != self.B or x.shape[1] != self.H or x.shape[3] != self.D:
            raise RuntimeError(
                f"Sizes of tensors must match except in dimension 2: cache "
                f"[{self.B}, {self.H}, *, {self.D}] vs new {list(x.shape)}")
        if x.dtype != self.dtype:
            raise TypeError(f"QuantizedKVCache: new chunk dtype {x.dtype} != cached {self.dtype}")
        xc = x.detach().contiguous()
        tn = xc.shape[2]
        if tn == 0:  # nothing to store; raises where the reference's quantizer would
            self.qz._check_reduce(xc, self.gran)
            return
        gn = self._groups_for(tn)
        self._grow(self.T + tn, self.ng + gn)
        gcode = _GRAN_CODE[self.gran]
        sz_pitch = {"per_token": self.cap, "per_channel": 1, "per_group": self.gcap}[self.gran]
        sz_off = {"per_token": self.T, "per_channel": 0, "per_group": self.ng}[self.gran]
        merge = int(self.gran == "per_channel" and self.T > 0)
        _C.call("lq_kv_append", xc.data_ptr(), _C.dt(xc), self.B * self.H, tn, self.D, gcode,
                self.qz.group_size, self.qz.n_bits, int(self.qz.symmetric), self.codes.data_ptr(),
                _C.dt(self.code_dtype), self.cap, self.T, self.scale.data_ptr(),
                self.zp.data_ptr(), sz_pitch, sz_off, merge, _C.stream_ptr(xc))
        self.T += tn
        self.ng += gn

    def views(self):
        """(codes, scale, zero_point) shaped like the reference's cache entries."""
        q = self.codes[:, :, :self.T]
        if self.gran == "per_token":
            return q, self.scale[:, :, :self.T], self.zp[:, :, :self.T]
        if self.gran == "per_group":
            return q, self.scale[:, :, :self.ng], self.zp[:, :, :self.ng]
        return q, self.scale, self.zp

    def dequantize(self) -> torch.Tensor:
        out = torch.empty(self.B, self.H, self.T, self.D, dtype=torch.float32, device=self.device)
        gcode = _GRAN_CODE[self.gran]
        sz_pitch = {"per_token": self.cap, "per_channel": 1, "per_group": self.gcap}[self.gran]
        _C.call("lq_kv_dequant", self.codes.data_ptr(), _C.dt(self.code_dtype), self.B * self.H,
                self.T, self.D, self.cap, gcode, self.qz.group_size, self.scale.data_ptr(),
                self.zp.data_ptr(), _C.dt(self.dtype), sz_pitch, out.data_ptr(),
                _C.stream_ptr(self.codes))
        return out


class QuantizedKVCache(nn.Module):
    """KV cache that quantizes on write and dequantizes on read
    (kv_cache_quant.py:312-426).

    Extensions (backwards compatible): ``value_quantizer`` gives V its own
    quantizer (default: the same one as K, as in the reference), and
    ``max_seq_len`` preallocates token capacity."""

    def __init__(
        self,
        num_layers: int,
        quantizer: Optional[KVCacheQuantizer] = None,
        value_quantizer: Optional[KVCacheQuantizer] = None,
        max_seq_len: int = 0,
    ):
        super().__init__()
        self.num_layers = num_layers
        self.quantizer = quantizer or PerTokenKVCacheQuantizer(n_bits=8)
        self.value_quantizer = value_quantizer
        self.max_seq_len = max_seq_len
        # per layer: (key_q, key_scale, key_zp, val_q, val_scale, val_zp) views or None
        self._cache: list[Optional[tuple]] = [None] * num_layers
        self._sides: list[Optional[tuple]] = [None] * num_layers

    def update(
        self,
        layer_idx: int,
        key: torch.Tensor,
        value: torch.Tensor,
    ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append new K, V [B, H, S_new, D] and return the full dequantized fp32
        K, V [B, H, S_total, D] (kv_cache_quant.py:336-382)."""
        self.append(layer_idx, key, value)
        ks, vs = self._sides[layer_idx]
        return ks.dequantize(), vs.dequantize()

    def _side_pair(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor):
        sides = self._sides[layer_idx]
        if sides is None:
            vq = self.value_quantizer or self.quantizer
            sides = (_CacheSide(self.quantizer, key, self.max_seq_len),
                     _CacheSide(vq, value, self.max_seq_len))
            self._sides[layer_idx] = sides
        return sides

    def append(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """The storing half of ``update``: quantize and append new K, V
        [B, H, S_new, D] without building the dequantized cache (for callers
        that attend with ``attend``)."""
        ks, vs = self._side_pair(layer_idx, key, value)
        ks.append(key)
        vs.append(value)
        self._cache[layer_idx] = ks.views() + vs.views()

    def attend(self, layer_idx: int, query: torch.Tensor, scale: Optional[float] = None,
               causal: bool = False) -> torch.Tensor:
        """softmax(query K^T * scale) V over a layer's cached tokens, where K
        and V are exactly the fp32 tensors ``update`` / ``get`` return
        (kv_cache_quant.py:221-267), computed from the codes in place.

        query [B, Hq, Sq, D] with Hq a multiple of the cached heads H (query
        head h reads kv head h // (Hq // H)); ``scale`` defaults to D ** -0.5;
        ``causal`` aligns the Sq queries to the end of the cache (query i sees
        tokens t <= T - Sq + i).  Returns [B, Hq, Sq, D] in query's dtype.
        Supported: head dim 64 or 128, the same code dtype for K and V, codes
        of at most 10 bits, per-group sizes that are multiples of 16."""
        sides = self._sides[layer_idx]
        if sides is None:
            raise RuntimeError(f"QuantizedKVCache.attend: layer {layer_idx} is empty")
        ks, vs = sides
        _C.require_cuda(query, what="QuantizedKVCache.attend")
        _C.require_float(query, "QuantizedKVCache.attend")
        if query.ndim != 4 or query.shape[0] != ks.B or query.shape[3] != ks.D or \
                query.shape[1] % ks.H:
            raise RuntimeError(
                f"QuantizedKVCache.attend: query {list(query.shape)} does not match the cache "
                f"[{ks.B}, {ks.H}*G, *, {ks.D}]")
        if ks.code_dtype != vs.code_dtype or ks.dtype != vs.dtype:
            raise NotImplementedError(
                "QuantizedKVCache.attend: K and V must share code and scale dtypes")
        for side in (ks, vs):
            if side.code_dtype == torch.int16 and side.qz.n_bits > 10:
                raise NotImplementedError(
                    "QuantizedKVCache.attend: asymmetric codes of more than 10 bits")
            if side.gran == "per_group" and side.qz.group_size % 16:
                raise NotImplementedError(
                    "QuantizedKVCache.attend: per-group sizes must be multiples of 16")
        q = query.contiguous()
        B, Hq, Sq, D = q.shape
        sm = float(D ** -0.5 if scale is None else scale)
        out = torch.empty_like(q)
        if B * Hq * Sq == 0:
            return out
        nbytes = _C.lib().lq_kv_attention_workspace_bytes(B, Hq, ks.H, Sq, D, ks.T)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device) if nbytes else None

        def side_args(sd):
            pitch = {"per_token": sd.cap, "per_channel": 1, "per_group": sd.gcap}[sd.gran]
            return (sd.codes.data_ptr(), _GRAN_CODE[sd.gran], sd.qz.group_size,
                    sd.scale.data_ptr(), sd.zp.data_ptr(), pitch)

        _C.call("lq_kv_attention", q.data_ptr(), _C.dt(q), B, Hq, ks.H, Sq, D, ks.T, ks.cap,
                _C.dt(ks.code_dtype), *side_args(ks), *side_args(vs), _C.dt(ks.dtype), sm,
                int(bool(causal)), out.data_ptr(), _C.ptr(ws), nbytes, _C.stream_ptr(q))
        return out

    def _cat_scales(self, old_scale: torch.Tensor, new_scale: torch.Tensor, seq_dim: int) -> torch.Tensor:
        """The reference's scale merge rule (kv_cache_quant.py:384-406), as a
        standalone helper: cat for per-token / per-group, torch.maximum for
        per-channel.  ``update`` applies the same rule inside its kernels."""
        gran = _gran(self.quantizer.granularity)
        if gran == "per_channel":
            return torch.maximum(old_scale, new_scale)
        return torch.cat([old_scale, new_scale], dim=2)

    def get(self, layer_idx: int) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        """Dequantized K, V of a layer, or None if empty (kv_cache_quant.py:408-415)."""
        sides = self._sides[layer_idx]
        if sides is None:
            return None
        return sides[0].dequantize(), sides[1].dequantize()

    def reset(self) -> None:
        """Clear all cached states (kv_cache_quant.py:417-419)."""
        self._cache = [None] * self.num_layers
        self._sides = [None] * self.num_layers

    @property
    def seq_len(self) -> int:
        """Tokens cached in layer 0 (kv_cache_quant.py:421-426)."""
        if self._cache[0] is None:
            return 0
        return self._cache[0][0].shape[2]


def kv_cache_memory_ratio(
    n_bits: int,
    orig_bits: int = 16,
    granularity: KVQuantGranularity = KVQuantGranularity.PER_TOKEN,
    head_dim: int = 128,
    seq_len: int = 2048,
) -> float:
    """Quantized / original KV-cache size estimate (kv_cache_quant.py:433-458):
    n_bits / orig_bits plus one 32-bit scale per head_dim values (per-token),
    per seq_len values (per-channel) or per 32 values (per-group)."""
    base = n_bits / orig_bits
    g = _gran(granularity)
    if g == "per_token":
        overhead = 32 / (head_dim * n_bits)
    elif g == "per_channel":
        overhead = 32 / (seq_len * n_bits)
    else:
        overhead = 32 / (32 * n_bits)
    return base + overhead
