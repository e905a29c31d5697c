"""GPU parity of the int-weight layers GPTQ and SpQR produce: GPTQLinear
(gptq.py:257-325) and SpQRLinear (spqr.py:102-208).

Against the reference's own layers (tests/golden/layers.npz): the buffers
after ``pack`` bit for bit, the dequantized weight the forward builds bit for
bit (read out of the reference as layer(I) = W^T), the fp32 forward within
fp32 GEMM rounding.  The fused fp16 / bf16 forward (W4A16 kernel, plus the
sparse outlier kernel for SpQR), which the reference does not have, against
the fp32 product of the same dequantized weight: max |y - y_ref| <= 1e-2 *
max |y_ref|.
"""

import numpy as np
import pytest
import torch

from golden_io import cases, same_bits
from gpu_util import to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.asarray(a)).to(dtype).cuda()


def _ids(v):
    return v if isinstance(v, str) else ""


@pytest.mark.parametrize("name,c", list(cases("layers.npz", "gptq")), ids=_ids)
def test_gptq_linear_golden(L, name, c):
    p = c["params"]
    ql = L.GPTQLinear(p["in_features"], p["out_features"], n_bits=p["n_bits"],
                      symmetric=p["symmetric"], group_size=p["group_size"]).cuda()
    ql.pack(_t(c["w_q"][0], torch.int64), _t(c["W"][0]))
    with torch.no_grad():
        ql.bias.copy_(_t(c["bias"][0]))
    assert np.array_equal(to_np(ql.weight_int), c["weight_int"][0])
    assert same_bits(to_np(ql.scale), c["scale"][0]) and same_bits(to_np(ql.zero_point), c["zero_point"][0])
    assert same_bits(to_np(ql.dequantized_weight()).T, c["wT"][0])
    y = ql(_t(c["x"][0]))
    np.testing.assert_allclose(to_np(y), c["y"][0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name,c", list(cases("layers.npz", "spqr")), ids=_ids)
def test_spqr_linear_golden(L, name, c):
    p = c["params"]
    layer = L.SpQRLinear(p["in_features"], p["out_features"], n_bits=p["n_bits"],
                         group_size=p["group_size"]).cuda()
    layer.pack(_t(c["W"][0]), _t(c["mask"][0], torch.bool))
    with torch.no_grad():
        layer.bias.copy_(_t(c["bias"][0]))
    assert np.array_equal(to_np(layer.weight_int), c["weight_int"][0])
    assert same_bits(to_np(layer.scale), c["scale"][0])
    assert same_bits(to_np(layer.zero_point), c["zero_point"][0])
    assert same_bits(to_np(layer.outlier_vals), c["outlier_vals"][0])
    assert abs(layer.sparsity - p["sparsity"]) < 1e-12
    assert same_bits(to_np(layer.dequantized_weight()).T, c["wT"][0])
    y = layer(_t(c["x"][0]))
    np.testing.assert_allclose(to_np(y), c["y"][0], rtol=1e-5, atol=1e-5)


def _check(y, ref):
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, (err, ref.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 7, 16, 130])
def test_gptq_fused_half_forward(L, dtype, M):
    g = torch.Generator().manual_seed(M)
    W = torch.randn(256, 512, generator=g).cuda()
    w_q = torch.randint(-8, 8, (256, 512), generator=g).cuda()
    ql = L.GPTQLinear(512, 256, n_bits=4, symmetric=True, group_size=128).cuda()
    ql.pack(w_q, W)
    from llm_quant_b200.core import w4a16
    x = torch.randn(M, 512, generator=g).cuda().to(dtype)
    assert w4a16.eligible(ql, x)
    y = ql(x)
    assert y.dtype == dtype
    _check(y, x.float() @ ql.dequantized_weight().T + ql.bias.float())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 9, 64, 300])
def test_spqr_fused_half_forward_with_outliers(L, dtype, M):
    g = torch.Generator().manual_seed(100 + M)
    W = torch.randn(384, 256, generator=g).cuda()
    mask = (torch.rand(384, 256, generator=g) < 0.01).cuda()
    W[mask] *= 20  # outliers far outside the int range
    layer = L.SpQRLinear(256, 384, n_bits=4, group_size=64).cuda()
    layer.pack(W, mask)
    with torch.no_grad():
        layer.bias.copy_(torch.randn(384, generator=g).cuda() * 0.1)
    x = torch.randn(M, 256, generator=g).cuda().to(dtype)
    y = layer(x)
    assert y.dtype == dtype and y.shape == (M, 384)
    _check(y, x.float() @ layer.dequantized_weight().T + layer.bias.float())
    # the outlier correction is applied (the int part alone is far off)
    layer2 = L.SpQRLinear(256, 384, n_bits=4, group_size=64).cuda()
    layer2.pack(W, torch.zeros_like(mask))
    assert (layer2(x).float() - y.float()).abs().max() > 0.1


def test_layer_state_dicts_round_trip(L):
    g = torch.Generator().manual_seed(5)
    W = torch.randn(128, 128, generator=g).cuda()
    mask = (torch.rand(128, 128, generator=g) < 0.02).cuda()
    a = L.SpQRLinear(128, 128, n_bits=4, group_size=64).cuda()
    a.pack(W, mask)
    b = L.SpQRLinear(128, 128, n_bits=4, group_size=64).cuda()
    b.load_state_dict(a.state_dict())
    x = torch.randn(3, 128, generator=g).cuda().half()
    assert torch.equal(a(x), b(x))
    q = L.GPTQLinear(128, 128, group_size=64).cuda()
    q.pack(torch.randint(-8, 8, (128, 128), generator=g).cuda(), W)
    r = L.GPTQLinear(128, 128, group_size=64).cuda()
    r.load_state_dict(q.state_dict())
    assert torch.equal(q(x), r(x))
