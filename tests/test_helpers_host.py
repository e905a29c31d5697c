"""CPU tests: the reference's rotation-construction helpers and core.utils
(off the hot path, eager torch) against fixtures written by running the
reference itself (tests/golden/helpers.npz), plus the import surface that
code written against the reference uses."""

import numpy as np
import pytest
import torch

from golden_io import load


@pytest.fixture(scope="module")
def G():
    return load("helpers.npz")


def T(case, field):
    arr, dt = case[field]
    t = torch.from_numpy(np.array(arr, copy=True))
    return t.to(torch.bfloat16) if dt == "bfloat16" else t


def test_reference_names_exported():
    """Every name of the reference's core facade and every hot-path name of
    its package facade (reference __init__.py:39-87, core/__init__.py:3-30)."""
    import llm_quant_b200 as L
    from llm_quant_b200 import core
    core_names = ["ste_round", "compute_qparams", "quantize_tensor", "dequantize_tensor",
                  "fake_quantize", "QuantizedLinear", "hadamard_matrix", "random_hadamard_matrix",
                  "random_orthogonal", "cayley_transform", "CayleyRotation",
                  "rotate_weight_right", "rotate_weight_left", "apply_rotation_to_linear",
                  "fast_hadamard_transform", "MinMaxObserver", "ActivationCollector",
                  "quantization_mse", "quantization_snr", "kurtosis", "make_dummy_linear",
                  "make_calibration_data"]
    for n in core_names:
        assert hasattr(core, n), n
        assert hasattr(L, n) and n in L.__all__, n
    for n in ["QScheme", "QLoRA", "QLoRALinear", "NF4_TABLE", "nf4_quantize", "nf4_dequantize",
              "double_quantize", "double_dequantize", "KVQuantGranularity", "KVCacheQuantizer",
              "QuantizedKVCache", "PerTokenKVCacheQuantizer", "PerChannelKVCacheQuantizer",
              "PerGroupKVCacheQuantizer", "kv_cache_memory_ratio", "GPTQLinear", "SpQRLinear"]:
        assert hasattr(L, n) and n in L.__all__, n


def test_install_as_llm_quant_module_paths():
    import importlib
    import sys
    import llm_quant_b200 as L
    saved = {k: v for k, v in sys.modules.items() if k == "llm_quant" or k.startswith("llm_quant.")}
    try:
        L.install_as_llm_quant()
        for path, name in [("llm_quant.core.utils", "MinMaxObserver"),
                           ("llm_quant.core.rotation", "random_hadamard_matrix"),
                           ("llm_quant.core.rotation", "CayleyRotation"),
                           ("llm_quant.core.quantizer", "QuantizedLinear"),
                           ("llm_quant.qlora", "QLoRALinear"),
                           ("llm_quant.kv_cache_quant", "QuantizedKVCache"),
                           ("llm_quant", "make_calibration_data")]:
            assert hasattr(importlib.import_module(path), name), (path, name)
    finally:
        for k in [k for k in sys.modules if k == "llm_quant" or k.startswith("llm_quant.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_random_hadamard_matrix(G):
    from llm_quant_b200.core.rotation import random_hadamard_matrix
    for name, c in G.items():
        if c["params"]["fn"] != "random_hadamard_matrix":
            continue
        p = c["params"]
        dt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[p["dtype"]]
        H = random_hadamard_matrix(p["n"], dt, generator=torch.Generator().manual_seed(p["seed"]))
        assert H.dtype == dt
        assert torch.equal(H, T(c, "H")), name


def test_random_orthogonal(G):
    from llm_quant_b200.core.rotation import random_orthogonal
    for name, c in G.items():
        if c["params"]["fn"] != "random_orthogonal":
            continue
        p = c["params"]
        Q = random_orthogonal(p["n"], generator=torch.Generator().manual_seed(p["seed"]))
        torch.testing.assert_close(Q, T(c, "Q"), atol=1e-6, rtol=1e-6)
        torch.testing.assert_close(Q @ Q.t(), torch.eye(p["n"]), atol=1e-5, rtol=1e-5)


def test_cayley(G):
    from llm_quant_b200.core.rotation import CayleyRotation, cayley_transform
    c = G["cayley"]
    torch.testing.assert_close(cayley_transform(T(c, "A")), T(c, "Q"), atol=1e-6, rtol=1e-6)
    c = G["cayley_rot"]
    cr = CayleyRotation(c["params"]["dim"])
    assert set(cr.state_dict()) == {"params"}
    with torch.no_grad():
        cr.params.copy_(T(c, "p"))
    torch.testing.assert_close(cr(), T(c, "Q"), atol=1e-6, rtol=1e-6)
    cr().sum().backward()
    assert cr.params.grad is not None and cr.params.grad.shape == cr.params.shape
    torch.testing.assert_close(CayleyRotation(5, init="hadamard")(), torch.eye(5))


def test_rotate_weight(G):
    from llm_quant_b200.core.rotation import (apply_rotation_to_linear, rotate_weight_left,
                                              rotate_weight_right)
    c = G["rotate"]
    w, r10, r6 = T(c, "W"), T(c, "R10"), T(c, "R6")
    # a BLAS product: its summation order may follow the thread count
    close = dict(atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(rotate_weight_right(w, r10), T(c, "right"), **close)
    torch.testing.assert_close(rotate_weight_left(w, r6), T(c, "left"), **close)
    lin = torch.nn.Linear(10, 6)
    with torch.no_grad():
        lin.weight.copy_(w)
    apply_rotation_to_linear(lin, r10)
    torch.testing.assert_close(lin.weight.data, T(c, "right"), **close)
    with torch.no_grad():
        lin.weight.copy_(w)
    apply_rotation_to_linear(lin, r6, side="left")
    torch.testing.assert_close(lin.weight.data, T(c, "left"), **close)
    with pytest.raises(ValueError, match="side must be 'right' or 'left', got 'up'"):
        apply_rotation_to_linear(lin, r6, side="up")


def test_min_max_observer(G):
    from llm_quant_b200.core.utils import MinMaxObserver
    c = G["observer"]
    batches = [T(c, f"b{i}") for i in range(3)]
    for key, kw in [("tensor", dict()), ("ch_last", dict(per_channel=True, channel_dim=-1)),
                    ("ch0", dict(per_channel=True, channel_dim=0)),
                    ("ch1", dict(per_channel=True, channel_dim=1))]:
        o = MinMaxObserver(**kw)
        with pytest.raises(AssertionError, match="No data observed yet"):
            o.get_range()
        for b in batches:
            o.update(b)
        lo, hi = o.get_range()
        assert torch.equal(lo, T(c, f"{key}_min")) and torch.equal(hi, T(c, f"{key}_max")), key
        o.reset()
        assert o.min_val is None and o.max_val is None


def test_metrics(G):
    from llm_quant_b200.core.utils import kurtosis, quantization_mse, quantization_snr
    c = G["metrics"]
    x, y = T(c, "x"), T(c, "y")
    assert torch.equal(quantization_mse(x, y), T(c, "mse"))
    assert torch.equal(quantization_snr(x, y), T(c, "snr"))
    assert torch.equal(kurtosis(x, dim=0), T(c, "kurt0"))
    assert torch.equal(kurtosis(x), T(c, "kurt1"))
    assert quantization_mse(x, x).item() == 0.0


def test_seeded_helpers(G):
    from llm_quant_b200.core.utils import make_calibration_data, make_dummy_linear
    c = G["dummy_linear"]
    lin = make_dummy_linear(64, 32)
    assert torch.equal(lin.weight.data, T(c, "w")) and torch.equal(lin.bias.data, T(c, "b"))
    nb = make_dummy_linear(16, 8, bias=False)
    assert nb.bias is None and torch.equal(nb.weight.data, T(c, "w_nb"))
    c = G["calib"]
    data = make_calibration_data(2, 4, 8, 3, seed=5)
    assert len(data) == 3
    for i, d in enumerate(data):
        assert torch.equal(d, T(c, f"d{i}"))


def test_activation_collector():
    from llm_quant_b200.core.utils import ActivationCollector
    model = torch.nn.Sequential(torch.nn.Linear(8, 8), torch.nn.ReLU(), torch.nn.Linear(8, 4))
    col = ActivationCollector(model, ["0", "2"])
    x = torch.randn(3, 8)
    with torch.no_grad():
        y = model(x)
        model(x)
    ins, outs = col.get_inputs(), col.get_outputs()
    assert len(ins["0"]) == 2 and torch.equal(ins["0"][0], x)
    assert torch.equal(outs["2"][0], y) and ins["2"][0].shape == (3, 8)
    col.remove_hooks()
    model(x)
    assert len(ins["0"]) == 2
