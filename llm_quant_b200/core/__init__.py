"""llm_quant_b200.core -- core quantization primitives (hot path on B200)."""

from .quantizer import (
    QScheme,
    ste_round,
    compute_qparams,
    quantize_tensor,
    dequantize_tensor,
    fake_quantize,
    QuantizedLinear,
)
from .rotation import (
    hadamard_matrix,
    fast_hadamard_transform,
    hadamard_fake_quantize,
)
