"""llm_quant_b200 -- B200 (sm_100a) implementation of llm_quant's quantization hot path.

Drop-in for the hot-path modules of MindIntels/llm_quant: the same names,
signatures and results (bit-exact on the same inputs), computed by
hand-written CUDA kernels in ``liblq_sm100.so`` on CUDA tensors:

* ``llm_quant_b200.core.quantizer``: QScheme, ste_round, compute_qparams,
  quantize_tensor, dequantize_tensor, fake_quantize, QuantizedLinear
  (W4A16 tensor-core forward);
* ``llm_quant_b200.core.rotation``: hadamard_matrix, fast_hadamard_transform
  (butterfly), hadamard_fake_quantize (fused QuaRot activation path), and the
  reference's rotation-construction helpers (random Hadamard / orthogonal,
  Cayley, weight rotation; eager PyTorch, off the hot path);
* ``llm_quant_b200.core.utils``: the reference's observers, metrics and
  calibration helpers (eager PyTorch, off the hot path);
* ``llm_quant_b200.qlora``: NF4 quantize / dequantize, double quantization,
  QLoRALinear (packed 4-bit storage), QLoRA;
* ``llm_quant_b200.kv_cache_quant``: KV-cache quantizers and QuantizedKVCache.

``install_as_llm_quant()`` registers these modules under the reference's
import names (``llm_quant``, ``llm_quant.core.quantizer``, ...) for code
written against the reference.
"""

from .core.quantizer import (
    QScheme,
    ste_round,
    compute_qparams,
    quantize_tensor,
    dequantize_tensor,
    fake_quantize,
    QuantizedLinear,
)
from .core.rotation import (
    hadamard_matrix,
    random_hadamard_matrix,
    random_orthogonal,
    cayley_transform,
    CayleyRotation,
    rotate_weight_right,
    rotate_weight_left,
    apply_rotation_to_linear,
    fast_hadamard_transform,
    hadamard_fake_quantize,
)
from .core.utils import (
    MinMaxObserver,
    ActivationCollector,
    quantization_mse,
    quantization_snr,
    kurtosis,
    make_dummy_linear,
    make_calibration_data,
)
from .qlora import (
    QLoRA, QLoRALinear, NF4_TABLE,
    nf4_quantize, nf4_dequantize,
    double_quantize, double_dequantize,
)
from .kv_cache_quant import (
    KVQuantGranularity, KVCacheQuantizer, QuantizedKVCache,
    PerTokenKVCacheQuantizer, PerChannelKVCacheQuantizer,
    PerGroupKVCacheQuantizer, kv_cache_memory_ratio,
)
from .gptq import GPTQLinear
from .spqr import SpQRLinear

__all__ = [
    "QScheme", "ste_round", "compute_qparams",
    "quantize_tensor", "dequantize_tensor", "fake_quantize",
    "QuantizedLinear",
    "hadamard_matrix", "random_hadamard_matrix", "random_orthogonal",
    "cayley_transform", "CayleyRotation",
    "rotate_weight_right", "rotate_weight_left",
    "apply_rotation_to_linear", "fast_hadamard_transform", "hadamard_fake_quantize",
    "MinMaxObserver", "ActivationCollector",
    "quantization_mse", "quantization_snr", "kurtosis",
    "make_dummy_linear", "make_calibration_data",
    "QLoRA", "QLoRALinear", "NF4_TABLE",
    "nf4_quantize", "nf4_dequantize",
    "double_quantize", "double_dequantize",
    "KVQuantGranularity", "KVCacheQuantizer", "QuantizedKVCache",
    "PerTokenKVCacheQuantizer", "PerChannelKVCacheQuantizer",
    "PerGroupKVCacheQuantizer", "kv_cache_memory_ratio",
    "GPTQLinear", "SpQRLinear",
    "install_as_llm_quant",
]


def install_as_llm_quant() -> None:
    """Make ``import llm_quant[.core[.quantizer|.rotation|.utils]|.qlora|
    .kv_cache_quant|.gptq|.spqr]`` resolve to this package (for code and tests written against the
    reference; of gptq / spqr only the layers are here)."""
    import sys
    from . import core, qlora, kv_cache_quant, gptq, spqr
    from .core import quantizer, rotation, utils
    mod = sys.modules[__name__]
    sys.modules["llm_quant"] = mod
    sys.modules["llm_quant.core"] = core
    sys.modules["llm_quant.core.quantizer"] = quantizer
    sys.modules["llm_quant.core.rotation"] = rotation
    sys.modules["llm_quant.core.utils"] = utils
    sys.modules["llm_quant.qlora"] = qlora
    sys.modules["llm_quant.kv_cache_quant"] = kv_cache_quant
    sys.modules["llm_quant.gptq"] = gptq
    sys.modules["llm_quant.spqr"] = spqr
