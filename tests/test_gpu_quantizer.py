"""GPU parity: core.quantizer against the reference's golden outputs and the oracle.

Bit-exact (sign of zero and NaN positions included) for scales, zero points,
codes and fake-quantized values; QuantizedLinear's fp32 forward within the
reference test's own float tolerance.
"""

import math

import numpy as np
import pytest
import torch

from golden_io import cases, same_bits
from gpu_util import to_dev, to_np, seeded
from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def _ids(v):
    return v if isinstance(v, str) else ""


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "quantizer")), ids=_ids)
def test_quantizer_golden(L, name, c):
    p = c["params"]
    dt = p["dtype"]
    x = to_dev(c["x"][0], dt)
    sch = L.QScheme(p["scheme"])
    s, zp = L.compute_qparams(x, p["n_bits"], p["symmetric"], sch, p["group_size"])
    assert s.dtype == x.dtype and tuple(s.shape) == c["scale"][0].shape
    assert same_bits(to_np(s), c["scale"][0]), "scale"
    assert same_bits(to_np(zp), c["zp"][0]), "zero_point"
    if p["scheme"] == "per_group":
        gs = p["group_size"]
        xp = torch.nn.functional.pad(x, (0, (-x.shape[1]) % gs)).reshape(x.shape[0], -1, gs)
    else:
        xp = x
    q = L.quantize_tensor(xp, s, zp, p["n_bits"], p["symmetric"])
    assert same_bits(to_np(q), c["q"][0]), "quantize_tensor"
    dq = L.dequantize_tensor(q, s, zp)
    assert same_bits(to_np(dq), c["dq"][0]), "dequantize_tensor"
    fq = L.fake_quantize(x, p["n_bits"], p["symmetric"], sch, p["group_size"])
    assert fq.dtype == x.dtype
    assert same_bits(to_np(fq), c["fq"][0]), "fake_quantize"


def test_ste_round_golden(L):
    (_, c), = list(cases("quantizer.npz", "ste"))
    y = L.ste_round(to_dev(c["x"][0], "float32"))
    assert same_bits(to_np(y), c["y"][0])
    x = torch.tensor([1.6, 2.3], device="cuda", requires_grad=True)
    L.ste_round(x).sum().backward()
    assert torch.equal(x.grad, torch.ones(2, device="cuda"))


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "mixed")), ids=_ids)
def test_mixed_dtype_golden(L, name, c):
    x = to_dev(*c["x"])
    s = to_dev(*c["scale"])
    zp = to_dev(*c["zp"])
    q = L.quantize_tensor(x, s, zp, 4, False)
    assert str(q.dtype).replace("torch.", "") == c["q"][1]
    assert same_bits(to_np(q), c["q"][0])
    dq = L.dequantize_tensor(q, s, zp)
    assert str(dq.dtype).replace("torch.", "") == c["dq"][1]
    assert same_bits(to_np(dq), c["dq"][0])


@pytest.mark.parametrize("name,c", list(cases("quantizer.npz", "qlinear")), ids=_ids)
def test_quantized_linear_golden(L, name, c):
    p = c["params"]
    lin = torch.nn.Linear(p["in_features"], p["out_features"]).to(to_dev(*c["w"]).dtype).cuda()
    with torch.no_grad():
        lin.weight.copy_(to_dev(*c["w"]))
        lin.bias.copy_(to_dev(*c["bias"]))
    ql = L.QuantizedLinear.from_linear(lin, p["n_bits"], p["symmetric"], p["group_size"])
    assert ql.weight_int.dtype == torch.int8
    assert np.array_equal(to_np(ql.weight_int), c["weight_int"][0])
    assert str(ql.scale.dtype).replace("torch.", "") == c["scale"][1]
    assert same_bits(to_np(ql.scale), c["scale"][0])
    assert same_bits(to_np(ql.zero_point), c["zero_point"][0])
    # fp32 forward as in the reference: bit-exact dequantized weight, fp32 GEMM
    w_ref = O.quantized_linear_dequant_weight(c["weight_int"][0], c["scale"][0], c["scale"][1],
                                              c["zero_point"][0], c["zero_point"][1],
                                              p["group_size"], p["in_features"])
    assert same_bits(to_np(ql.dequantized_weight()), w_ref)
    # the reference forward: F.linear(x fp32, w_float fp32, bias)
    y = torch.nn.functional.linear(to_dev(*c["x"]), ql.dequantized_weight(), ql.bias.float())
    np.testing.assert_allclose(to_np(y), c["y"][0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("shape,gs", [((512, 4096), 128), ((300, 1000), 128), ((64, 96), 32),
                                      ((17, 4096), 4096), ((9, 100), 8)])
@pytest.mark.parametrize("sym,bits", [(False, 4), (True, 4), (True, 8), (False, 8)])
def test_group_fake_quant_vs_oracle(L, dtype, shape, gs, sym, bits):
    x = seeded(shape, 7, 0.02, outliers=3).numpy()
    xo = O.rnd(x, dtype)
    xd = to_dev(xo, dtype)
    fq = L.fake_quantize(xd, bits, sym, L.QScheme.PER_GROUP, gs)
    assert same_bits(to_np(fq), O.fake_quantize(xo, dtype, bits, sym, "per_group", gs))


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("shape", [(64, 4096), (8, 5, 7), (3, 70000)])
@pytest.mark.parametrize("scheme", ["per_channel", "per_tensor"])
def test_channel_tensor_fake_quant_vs_oracle(L, dtype, shape, scheme):
    x = O.rnd(seeded(shape, 11, 1.0, outliers=2).numpy(), dtype)
    for sym, bits in ((True, 4), (False, 8)):
        fq = L.fake_quantize(to_dev(x, dtype), bits, sym, L.QScheme(scheme))
        assert same_bits(to_np(fq), O.fake_quantize(x, dtype, bits, sym, scheme))


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_per_channel_inner_axis_qparams(L, dtype):
    x = O.rnd(seeded((6, 10, 12), 3).numpy(), dtype)
    for cd in (1, 2):
        for sym in (True, False):
            s, z = L.compute_qparams(to_dev(x, dtype), 8, sym, L.QScheme.PER_CHANNEL, channel_dim=cd)
            so, zo = O.compute_qparams(x, dtype, 8, sym, "per_channel", channel_dim=cd)
            assert tuple(s.shape) == so.shape
            assert same_bits(to_np(s), so) and same_bits(to_np(z), zo)


def test_config1_full_size(L):
    """fake_quantize INT4 asym g128 on fp32 [4096, 4096] ~ N(0, 0.02), seed 0: bit-exact."""
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(4096, 4096, generator=g) * 0.02)
    fq = L.fake_quantize(w.cuda(), 4, False, L.QScheme.PER_GROUP, 128)
    ref = O.fake_quantize(w.numpy(), "float32", 4, False, "per_group", 128)
    assert same_bits(to_np(fq), ref)
    s, z = L.compute_qparams(w.cuda(), 4, False, L.QScheme.PER_GROUP, 128)
    assert tuple(s.shape) == (4096, 32, 1)
    zz = to_np(z)
    assert zz.min() >= 0 and zz.max() <= 15


def test_quantized_linear_state_dict_roundtrip(L):
    lin = torch.nn.Linear(256, 64).cuda()
    ql = L.QuantizedLinear.from_linear(lin, 4, False, 128)
    sd = ql.state_dict()
    assert set(sd) == {"weight_int", "scale", "zero_point", "bias"}
    ql2 = L.QuantizedLinear(256, 64, 4, False, 128).cuda()
    ql2.scale = torch.empty_like(ql.scale)
    ql2.zero_point = torch.empty_like(ql.zero_point)
    ql2.load_state_dict(sd)
    x = torch.randn(3, 256, device="cuda")
    assert torch.equal(ql(x), ql2(x))


@pytest.mark.parametrize("name,c", list(cases("grad.npz", "grad")), ids=_ids)
def test_fake_quantize_gradient_golden(L, name, c):
    """Forward bit-exact; gradient vs the reference's autograd within float
    tolerance (1e-5 relative for fp32, 1e-2 for half types: sums of the scale
    gradient are accumulated in a different order)."""
    p = c["params"]
    dt = p["dtype"]
    x = to_dev(c["x"][0], dt).requires_grad_(True)
    y = L.fake_quantize(x, p["n_bits"], p["symmetric"], L.QScheme(p["scheme"]), p["group_size"])
    assert same_bits(to_np(y), c["y"][0])
    y.backward(to_dev(c["go"][0], dt))
    gx, ref = to_np(x.grad), c["gx"][0]
    tol = 1e-5 if dt == "float32" else 1e-2
    np.testing.assert_allclose(gx, ref, rtol=tol, atol=tol * max(1.0, np.abs(ref).max()))


def test_fake_quantize_gradient_flows(L):
    """The reference's own check (tests/test_quantizer.py:96-101)."""
    x = torch.randn(8, 32, device="cuda", requires_grad=True)
    y = L.fake_quantize(x, n_bits=8)
    y.sum().backward()
    assert x.grad is not None and x.grad.shape == x.shape


def _tie_groups(sym, shift, seed):
    """16 rows x 4 groups of 128 fp32 values whose quotient x / scale lands on
    half-integers (ties), one ulp either side of them, and on integers: each
    group spans exactly 15 (asymmetric 4-bit: scale 1, zero point -min) or has
    max |x| = 7 (symmetric: scale 1).  Row 3 holds a NaN, row 5 an inf."""
    rng = np.random.default_rng(seed)
    x = np.empty((16, 512), np.float32)
    for r in range(16):
        for g in range(4):
            if sym:
                v = rng.integers(-12, 13, 128) / 2.0
                v[0] = 7.0 if g % 2 == 0 else -7.0
            else:
                v = rng.integers(2, 29, 128) / 2.0 + shift
                v[0], v[1] = shift, 15.0 + shift
            v = v.astype(np.float32)
            k = rng.choice(np.arange(2, 128), 24, replace=False)
            v[k[:12]] = np.nextafter(v[k[:12]], np.float32(np.inf))
            v[k[12:]] = np.nextafter(v[k[12:]], np.float32(-np.inf))
            x[r, 128 * g:128 * (g + 1)] = v
    x[3, 77] = np.nan
    x[5, 300] = np.inf
    return x


@pytest.mark.parametrize("sym,shift", [(False, 0.0), (False, -3.0), (False, -6.5), (True, 0.0)])
def test_fp32_group_ties(L, sym, shift):
    """fp32 per-group fake quantization and int8 codes where the quotient
    sits on, or one ulp beside, a rounding tie: the kernel's product-quotient
    path must hand these elements to the exact division (half to even, as the
    reference's torch.round)."""
    x = _tie_groups(sym, shift, seed=int(10 * shift) + 5 * sym + 100)
    scale, _ = O.compute_qparams(x, "float32", 4, sym, "per_group", 128)
    finite = np.isfinite(scale.reshape(16, 4))
    assert finite[[0, 1, 2, 4, 6]].all() and np.all(scale.reshape(16, 4)[finite] == 1.0)
    fq = L.fake_quantize(to_dev(x, "float32"), 4, sym, L.QScheme.PER_GROUP, 128)
    assert same_bits(to_np(fq), O.fake_quantize(x, "float32", 4, sym, "per_group", 128))
    xs = np.nan_to_num(x, nan=0.0, posinf=15.0)  # codes: finite weights
    lin = torch.nn.Linear(512, 16, bias=False).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(xs))
    ql = L.QuantizedLinear.from_linear(lin, 4, sym, 128)
    wi, _, _ = O.quantized_linear_quantize_weights(xs, "float32", 4, sym, 128)
    assert np.array_equal(to_np(ql.weight_int), wi)
