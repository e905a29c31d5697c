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
from .utils import (
    MinMaxObserver,
    ActivationCollector,
    quantization_mse,
    quantization_snr,
    kurtosis,
    make_dummy_linear,
    make_calibration_data,
)
