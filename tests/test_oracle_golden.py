"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

Every comparison is bitwise (sign of zero included, NaN positions compared),
except the Hadamard transform, whose reference is a dense matmul whose
rounding order cannot be restated exactly (tolerances as in the reference's
tests/test_rotation.py:100-106 for fp32; 1e-2 relative for half types).
"""

import numpy as np
import pytest

from golden_io import cases, same_bits
from oracle import lq_oracle as O


def _p(c, k):
    return c[k][0]


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "quantizer")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_quantizer_cases(name, c):
    p = c["params"]
    dt = p["dtype"]
    x = _p(c, "x")
    s, zp = O.compute_qparams(x, dt, p["n_bits"], p["symmetric"], p["scheme"], p["group_size"])
    assert same_bits(s, _p(c, "scale")), "scale"
    assert same_bits(zp, _p(c, "zp")), "zero_point"
    if p["scheme"] == "per_group":
        xin = O.pad_groups(x, p["group_size"])
    else:
        xin = x
    q, qdt = O.quantize_tensor(xin, dt, s, dt, zp, dt, p["n_bits"], p["symmetric"])
    assert qdt == c["q"][1]
    assert same_bits(q, _p(c, "q")), "quantize_tensor"
    dq, _ = O.dequantize_tensor(q, qdt, s, dt, zp, dt)
    assert same_bits(dq, _p(c, "dq")), "dequantize_tensor"
    fq = O.fake_quantize(x, dt, p["n_bits"], p["symmetric"], p["scheme"], p["group_size"])
    assert same_bits(fq, _p(c, "fq")), "fake_quantize"


def test_ste_round_known_answer():
    (_, c), = list(cases("quantizer.npz", "ste"))
    assert same_bits(O.ste_round(_p(c, "x")), _p(c, "y"))
    # the reference's own known answer (tests/test_quantizer.py:20-24)
    assert same_bits(O.ste_round(np.array([1.3, 2.7, -0.5, 0.0], np.float32)),
                     np.array([1.0, 3.0, 0.0, 0.0], np.float32))


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "mixed")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_mixed_dtype_promotion(name, c):
    x, xdt = c["x"]
    s, sdt = c["scale"]
    zp, zdt = c["zp"]
    q, qdt = O.quantize_tensor(x, xdt, s, sdt, zp, zdt, 4, False)
    assert qdt == c["q"][1]
    assert same_bits(q, _p(c, "q"))
    dq, ddt = O.dequantize_tensor(q, qdt, s, sdt, zp, zdt)
    assert ddt == c["dq"][1]
    assert same_bits(dq, _p(c, "dq"))


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "qlinear")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_quantized_linear_buffers(name, c):
    p = c["params"]
    wi, s, zp = O.quantized_linear_quantize_weights(_p(c, "w"), p["dtype"], p["n_bits"],
                                                   p["symmetric"], p["group_size"])
    assert np.array_equal(wi, _p(c, "weight_int"))
    assert same_bits(s, _p(c, "scale")) and same_bits(zp, _p(c, "zero_point"))
    w = O.quantized_linear_dequant_weight(wi, s, c["scale"][1], zp, c["zero_point"][1],
                                          p["group_size"], p["in_features"])
    y = _p(c, "x").astype(np.float64) @ w.astype(np.float64).T + _p(c, "bias").astype(np.float64)
    np.testing.assert_allclose(y, _p(c, "y"), rtol=1e-5, atol=1e-5)


def test_hadamard_entries_and_matrix():
    for _, c in cases("rotation.npz", "hadamard_entries"):
        dt = c["params"]["dtype"]
        ent = _p(c, "ent")
        for k in range(len(ent)):
            assert O.hadamard_entry(2 ** k, dt) == ent[k], (dt, k)
    for _, c in cases("rotation.npz", "hadamard"):
        assert same_bits(O.hadamard_matrix(8, c["params"]["dtype"]), _p(c, "H"))


@pytest.mark.parametrize("name,c", list(cases("rotation.npz", "fht")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_fht_oracle_vs_reference(name, c):
    dt = c["params"]["dtype"]
    y = O.fast_hadamard_transform(_p(c, "x"), dt)
    tol = 1e-5 if dt == "float32" else 1e-2
    np.testing.assert_allclose(y, _p(c, "y"), rtol=tol, atol=tol)


def test_nf4_table():
    (_, c), = list(cases("nf4.npz", "table"))
    assert same_bits(O.NF4_TABLE, _p(c, "table"))


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "nf4")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_nf4_cases(name, c):
    p = c["params"]
    codes, scales = O.nf4_quantize(_p(c, "x"), p["dtype"], p["group_size"])
    assert np.array_equal(codes, _p(c, "codes"))
    assert same_bits(scales, _p(c, "scales"))
    deq = O.nf4_dequantize(codes, scales, p["dtype"], p["group_size"])
    assert same_bits(deq, _p(c, "deq"))


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "nf4_grid")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_nf4_decision_grid(name, c):
    p = c["params"]
    codes, scales = O.nf4_quantize(_p(c, "x"), p["dtype"], p["group_size"])
    assert np.array_equal(codes.astype(np.uint8), _p(c, "codes"))
    assert same_bits(scales, _p(c, "scales"))


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "double_quant")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_double_quant(name, c):
    p = c["params"]
    q, dq = O.double_quantize(_p(c, "s"), p["dtype"], p["dq_group_size"])
    assert same_bits(q, _p(c, "q")) and same_bits(dq, _p(c, "dq"))
    rs = O.double_dequantize(q, dq, p["dtype"], p["dq_group_size"])
    assert same_bits(rs, _p(c, "restored"))


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "qlora")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_qlora_pack_base(name, c):
    p = c["params"]
    dt, gs = p["dtype"], p["group_size"]
    codes, scales = O.nf4_quantize(_p(c, "w"), dt, gs)
    assert np.array_equal(codes, _p(c, "nf4_codes")) and same_bits(scales, _p(c, "nf4_scales"))
    if p["double_quant"]:
        q, dq = O.double_quantize(scales, dt, 256)
        assert same_bits(q, _p(c, "dq_q_scales")) and same_bits(dq, _p(c, "dq_scales"))
        scales = O.double_dequantize(q, dq, dt, 256)
    wb = O.nf4_dequantize(codes, scales, dt, gs, orig_shape=(p["out_features"], p["in_features"]))
    assert same_bits(wb, _p(c, "w_base"))


@pytest.mark.parametrize("name,c", list(cases("kv.npz", "kv")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_kv_quantizer(name, c):
    p = c["params"]
    q, s, zp = O.kv_quantize(_p(c, "x"), p["dtype"], p["n_bits"], p["symmetric"],
                             p["granularity"], p["group_size"])
    assert q.dtype == _p(c, "q").dtype and np.array_equal(q, _p(c, "q"))
    assert same_bits(s, _p(c, "scale")) and same_bits(zp, _p(c, "zp"))
    deq = O.kv_dequantize(q, s, p["dtype"], zp, p["dtype"], p["granularity"], p["group_size"])
    assert same_bits(deq, _p(c, "deq"))


@pytest.mark.parametrize("name,c", list(cases("kv.npz", "kv_cache")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_kv_cache_sequence(name, c):
    p = c["params"]
    qz = dict(n_bits=p["n_bits"], symmetric=p["symmetric"], granularity=p["granularity"],
              group_size=p["group_size"])
    cache = O.QuantizedKVCacheOracle(2, p["dtype"], qz)
    for j in range(len(p["chunks"])):
        fk, fv = cache.update(1, _p(c, f"k{j}"), _p(c, f"v{j}"))
        assert same_bits(fk, _p(c, f"fk{j}")), j
        assert same_bits(fv, _p(c, f"fv{j}")), j


def test_kv_cache_mixed_granularity():
    (_, c), = list(cases("kv.npz", "kv_cache_mixed"))
    cache = O.QuantizedKVCacheOracle(
        1, "bfloat16", dict(n_bits=8, symmetric=True, granularity="per_channel"),
        dict(n_bits=4, symmetric=True, granularity="per_token"))
    for j in range(3):
        fk, fv = cache.update(0, _p(c, f"k{j}"), _p(c, f"v{j}"))
        assert same_bits(fk, _p(c, f"fk{j}")) and same_bits(fv, _p(c, f"fv{j}"))


@pytest.mark.parametrize("name,c", list(cases("layers.npz", "gptq")), ids=lambda v: v if isinstance(v, str) else "")
def test_oracle_gptq_linear(name, c):
    p = c["params"]
    wi, s, z = O.gptq_linear_pack(c["w_q"][0], c["W"][0], "float32", p["n_bits"], p["symmetric"],
                                  p["group_size"])
    assert np.array_equal(wi, c["weight_int"][0])
    assert same_bits(s, c["scale"][0]) and same_bits(z, c["zero_point"][0])
    w = O.quantized_linear_dequant_weight(wi, s, "float32", z, "float32", p["group_size"],
                                          p["in_features"])
    assert same_bits(w.T, c["wT"][0])


@pytest.mark.parametrize("name,c", list(cases("layers.npz", "spqr")), ids=lambda v: v if isinstance(v, str) else "")
def test_oracle_spqr_linear(name, c):
    p = c["params"]
    mask = c["mask"][0].astype(bool)
    wi, s, z, vals = O.spqr_linear_pack(c["W"][0], mask, "float32", p["n_bits"], p["group_size"])
    assert np.array_equal(wi, c["weight_int"][0])
    assert same_bits(s, c["scale"][0]) and same_bits(z, c["zero_point"][0])
    assert same_bits(vals, c["outlier_vals"][0])
    w = O.spqr_linear_dequant_weight(wi, s, "float32", z, "float32", p["group_size"],
                                     p["in_features"], mask, vals)
    assert same_bits(w.T, c["wT"][0])
