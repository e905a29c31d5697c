"""GPU parity: QuantizedLinear W4A16 forward (tensor cores) against the
reference's dequantize-then-matmul (core/quantizer.py:262-280).

The reference builds the fp32 weight (q - zero) * scale and multiplies in
fp32.  The kernel rounds each dequantized weight to the activation dtype
(fp16: 2^-11, bf16: 2^-8 relative) and accumulates in fp32, so outputs are
compared with a tolerance relative to the output scale: max |y - y_ref| <=
1e-2 * max |y_ref| (and elementwise within 1e-2 of that scale).
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def _ref(ql, x):
    """fp64 product with the reference's exact fp32 dequantized weight."""
    w = ql.dequantized_weight().double()
    y = x.double() @ w.T
    if ql.bias is not None:
        y = y + ql.bias.double()
    return y


def _check(y, ref, tol=1e-2):
    scale = ref.abs().max().item()
    err = (y.double() - ref).abs().max().item()
    assert err <= tol * max(scale, 1e-6), f"max err {err:.3e} vs scale {scale:.3e}"


def _make(L, N, K, group, sym, wdtype, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        if bias:
            lin.bias.copy_(torch.randn(N, generator=g) * 0.1)
    lin = lin.to(wdtype).cuda()
    return L.QuantizedLinear.from_linear(lin, 4, sym, group)


@pytest.mark.parametrize("act", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 5, 16, 17, 32, 64, 100, 128, 200, 256, 300])
def test_w4a16_small_shapes(L, act, M):
    ql = _make(L, 256, 512, 128, False, torch.float16, 1)
    from llm_quant_b200.core import w4a16
    x = torch.randn(M, 512, generator=torch.Generator().manual_seed(M)).to(act).cuda()
    assert w4a16.eligible(ql, x)
    y = ql(x)
    assert y.dtype == act and y.shape == (M, 256)
    _check(y, _ref(ql, x))
    assert w4a16.check_error_flag(x.device) == 0


def test_w4a16_single_k_step_structured(L):
    """K = 64 (one pipeline stage): exposes operand-layout mistakes directly."""
    ql = _make(L, 128, 64, 64, False, torch.float16, 2, bias=False)
    x = torch.zeros(16, 64, dtype=torch.float16, device="cuda")
    for m in range(16):
        x[m, (m * 5) % 64] = 1.0  # y[m, n] picks one weight column
    _check(ql(x), _ref(ql, x), tol=2e-3)


@pytest.mark.parametrize("sym", [False, True])
@pytest.mark.parametrize("wdtype", [torch.float16, torch.bfloat16, torch.float32])
def test_w4a16_sym_and_scale_dtypes(L, sym, wdtype):
    ql = _make(L, 384, 1024, 128, sym, wdtype, 3)
    for act in (torch.float16, torch.bfloat16):
        x = torch.randn(48, 1024, generator=torch.Generator().manual_seed(4)).to(act).cuda()
        _check(ql(x), _ref(ql, x))


def test_w4a16_3d_input_and_no_bias(L):
    ql = _make(L, 128, 256, 64, False, torch.float16, 5, bias=False)
    x = torch.randn(2, 7, 256, device="cuda", dtype=torch.float16)
    y = ql(x)
    assert y.shape == (2, 7, 128)
    _check(y.reshape(14, 128), _ref(ql, x.reshape(14, 256)))


def test_w4a16_packed_cache_invalidated(L):
    ql = _make(L, 128, 256, 128, False, torch.float16, 6)
    x = torch.randn(8, 256, device="cuda", dtype=torch.float16)
    y0 = ql(x)
    w = torch.randn(128, 256, device="cuda", dtype=torch.float16) * 0.05
    ql.quantize_weights(w)
    y1 = ql(x)
    assert not torch.equal(y0, y1)
    _check(y1, _ref(ql, x))


@pytest.mark.parametrize("K,group", [(1024, 128), (960, 64), (1536, 192)])
@pytest.mark.parametrize("M", [300, 777, 1500])
def test_w4a16_many_tiles_per_sm(L, K, group, M):
    """N = 8192 (64 weight-row tiles) and M > 128: more tiles than SMs (the
    grid runs in several waves), the last token tile partial; K = 960 takes
    the 64-wide stages, group 192 the non-power-of-two group index; a single
    64-wide stage (K = 960 has 15) leaves one dequant group a stage fewer."""
    ql = _make(L, 8192, K, group, False, torch.float16, M + K)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().cuda()
    y = ql(x)
    _check(y, _ref(ql, x))
    y2 = ql(x)  # a second launch reuses the pipeline barriers from scratch
    assert torch.equal(y, y2)
    from llm_quant_b200.core import w4a16
    assert w4a16.check_error_flag(x.device) == 0


@pytest.mark.parametrize("M", [1, 16, 128, 1024, 4096])
def test_config5_full_size(L, M):
    """Linear(4096, 14336) int4 g128 asym with fp16 scales/zeros, fp16 x."""
    g = torch.Generator().manual_seed(0)
    lin = torch.nn.Linear(4096, 14336)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(14336, 4096, generator=g) * 0.02)
    lin = lin.half().cuda()
    ql = L.QuantizedLinear.from_linear(lin, 4, False, 128)
    assert ql.scale.dtype == torch.float16 and ql.scale.shape == (14336, 32)
    x = torch.randn(M, 4096, generator=g).half().cuda()
    y = ql(x)
    w = ql.dequantized_weight()  # exact reference fp32 weight
    ref = torch.nn.functional.linear(x.float(), w, ql.bias.float()).double()
    _check(y, ref)
    from llm_quant_b200.core import w4a16
    assert w4a16.check_error_flag(x.device) == 0
