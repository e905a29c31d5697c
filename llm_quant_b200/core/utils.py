"""llm_quant_b200.core.utils -- the calibration and metric helpers of
llm_quant.core.utils, for code written against the reference.

These run once per calibration batch or per layer, off the data-parallel hot
path, so they are plain eager PyTorch on whatever device their inputs live
on (CPU included).  Names, signatures, defaults and results follow
core/utils.py of the reference:

* MinMaxObserver (core/utils.py:25-67): running min / max, per tensor or
  per channel;
* ActivationCollector (core/utils.py:74-113): forward hooks that keep each
  named layer's first input and its output on the host;
* quantization_mse / quantization_snr / kurtosis (core/utils.py:120-149);
* make_dummy_linear / make_calibration_data (core/utils.py:156-184): seeded
  test inputs, equal to the reference's for the same arguments.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn as nn

__all__ = [
    "MinMaxObserver", "ActivationCollector", "quantization_mse", "quantization_snr",
    "kurtosis", "make_dummy_linear", "make_calibration_data",
]


class MinMaxObserver:
    """Running minimum and maximum over calibration batches.

    ``per_channel=False`` keeps two scalars; ``per_channel=True`` keeps one
    value per index of ``channel_dim`` (every other dim is reduced).
    ``get_range()`` raises ``AssertionError`` before the first ``update``."""

    def __init__(self, per_channel: bool = False, channel_dim: int = -1):
        self.per_channel = per_channel
        self.channel_dim = channel_dim
        self.min_val: Optional[torch.Tensor] = None
        self.max_val: Optional[torch.Tensor] = None

    def _batch_range(self, x: torch.Tensor):
        if not self.per_channel:
            return x.min(), x.max()
        keep = self.channel_dim % x.ndim
        dims = [d for d in range(x.ndim) if d != keep]
        return x.amin(dim=dims), x.amax(dim=dims)

    def update(self, x: torch.Tensor) -> None:
        lo, hi = self._batch_range(x)
        if self.min_val is None:
            self.min_val, self.max_val = lo.clone(), hi.clone()
            return
        self.min_val = torch.minimum(self.min_val, lo)
        self.max_val = torch.maximum(self.max_val, hi)

    def get_range(self):
        """(min_val, max_val) seen so far."""
        assert self.min_val is not None, "No data observed yet"
        return self.min_val, self.max_val

    def reset(self) -> None:
        self.min_val = self.max_val = None


class ActivationCollector:
    """Forward hooks on the named submodules of ``model``.  Every forward
    appends the module's first positional input (and its output, when that
    is a tensor) to ``inputs[name]`` / ``outputs[name]``, detached and
    copied to host memory so calibration sets do not hold device memory."""

    def __init__(self, model: nn.Module, layer_names: List[str]):
        modules = dict(model.named_modules())
        self.inputs: Dict[str, List[torch.Tensor]] = {}
        self.outputs: Dict[str, List[torch.Tensor]] = {}
        self._hooks = []
        for name in layer_names:
            self.inputs[name], self.outputs[name] = [], []
            self._hooks.append(modules[name].register_forward_hook(self._recorder(name)))

    def _recorder(self, name: str):
        ins, outs = self.inputs[name], self.outputs[name]

        def record(_module, args, result):
            ins.append(args[0].detach().cpu())
            if isinstance(result, torch.Tensor):
                outs.append(result.detach().cpu())
        return record

    def get_inputs(self) -> Dict[str, List[torch.Tensor]]:
        return self.inputs

    def get_outputs(self) -> Dict[str, List[torch.Tensor]]:
        return self.outputs

    def remove_hooks(self) -> None:
        while self._hooks:
            self._hooks.pop().remove()


def quantization_mse(original: torch.Tensor, quantized: torch.Tensor) -> torch.Tensor:
    """Mean of the squared quantization error (a 0-dim tensor)."""
    return (original - quantized).pow(2).mean()


def quantization_snr(original: torch.Tensor, quantized: torch.Tensor) -> torch.Tensor:
    """Signal-to-quantization-noise ratio in dB: 10 log10(sum x^2 / sum e^2),
    the noise energy floored at 1e-12."""
    noise = (original - quantized).pow(2).sum().clamp(min=1e-12)
    return 10.0 * torch.log10(original.pow(2).sum() / noise)


def kurtosis(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Excess kurtosis along ``dim`` (fourth central moment over the squared
    variance, minus 3; the variance floored at 1e-12); ``dim`` is removed."""
    centred = x - x.mean(dim=dim, keepdim=True)
    var = centred.pow(2).mean(dim=dim, keepdim=True).clamp(min=1e-12)
    m4 = centred.pow(4).mean(dim=dim, keepdim=True)
    return (m4 / var.pow(2) - 3.0).squeeze(dim)


def make_dummy_linear(in_features: int = 768, out_features: int = 768,
                      bias: bool = True) -> nn.Linear:
    """An ``nn.Linear`` with reproducible N(0, 0.02) weights and a zero bias.

    Seeds the global generator with 42 and draws in the same order as the
    reference (the layer's default initialisation, then the normal draw), so
    the weights equal the reference's."""
    torch.manual_seed(42)
    linear = nn.Linear(in_features, out_features, bias=bias)
    with torch.no_grad():
        linear.weight.normal_(0.0, 0.02)
        if bias:
            linear.bias.zero_()
    return linear


def make_calibration_data(batch_size: int = 4, seq_len: int = 64, hidden: int = 768,
                          n_batches: int = 8, seed: int = 0) -> List[torch.Tensor]:
    """``n_batches`` N(0, 1) tensors of shape (batch_size, seq_len, hidden)
    from a CPU generator seeded with ``seed`` (the reference's values), placed
    on torch's default device."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.get_default_device()
    return [torch.randn(batch_size, seq_len, hidden, generator=g, device="cpu").to(dev)
            for _ in range(n_batches)]
