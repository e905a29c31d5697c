"""Empty inputs through the drop-in surface on the GPU.

The reference's behaviour on zero-size tensors (recorded by running it on the
CPU) is part of the interface: where it returns an empty result, the same
shape and dtype come back here; where torch raises inside it (a reduction or a
reshape of zero elements), the same exception type is raised here.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def M():
    from llm_quant_b200 import kv_cache_quant, qlora
    from llm_quant_b200.core import quantizer, rotation
    return quantizer, rotation, qlora, kv_cache_quant


def test_qparams_and_fake_quant_empty_rows(M):
    Q = M[0]
    x = torch.randn(0, 256, device=DEV)
    with pytest.raises(RuntimeError):  # torch min() over zero elements (quantizer.py per-tensor)
        Q.compute_qparams(x, 4, False, Q.QScheme.PER_TENSOR)
    s, z = Q.compute_qparams(x, 4, False, Q.QScheme.PER_CHANNEL)
    assert s.shape == (0, 1) and z.shape == (0, 1) and s.dtype == x.dtype
    s, z = Q.compute_qparams(x, 4, False, Q.QScheme.PER_GROUP, 128)
    assert s.shape == (0, 2, 1) and z.shape == (0, 2, 1)
    with pytest.raises(RuntimeError):  # reshape of 0 elements into [0, -1]
        Q.fake_quantize(x, 4, False, Q.QScheme.PER_GROUP, 128)
    with pytest.raises(RuntimeError):
        Q.fake_quantize(x, 4, False, Q.QScheme.PER_TENSOR)
    y = Q.fake_quantize(x, 4, False, Q.QScheme.PER_CHANNEL)
    assert y.shape == (0, 256) and y.dtype == x.dtype
    y = Q.fake_quantize(torch.randn(4, 0, device=DEV), 4, False, Q.QScheme.PER_GROUP, 128)
    assert y.shape == (4, 0)
    s, z = Q.compute_qparams(torch.randn(4, 0, device=DEV), 8, False, Q.QScheme.PER_GROUP, 128)
    assert s.shape == (4, 0, 1) and z.shape == (4, 0, 1)
    # per-channel: a zero-size reduced dim raises (torch.amax / amin)
    for shape, kw in (((0, 0), {}), ((4, 0), {}), ((2, 0, 5), {}), ((0, 3, 5), {"channel_dim": 1})):
        with pytest.raises(IndexError):
            Q.compute_qparams(torch.randn(*shape, device=DEV), 8, False, Q.QScheme.PER_CHANNEL, **kw)
    with pytest.raises(IndexError):
        Q.fake_quantize(torch.randn(4, 0, device=DEV), 8, False, Q.QScheme.PER_CHANNEL)
    s, z = Q.compute_qparams(torch.randn(0, 3, 5, device=DEV), 8, True, Q.QScheme.PER_CHANNEL)
    assert s.shape == (0, 1, 1) and z.shape == (0, 1, 1)
    s, z = Q.compute_qparams(torch.randn(2, 0, 5, device=DEV), 8, False, Q.QScheme.PER_CHANNEL, channel_dim=1)
    assert s.shape == (1, 0, 1) and z.shape == (1, 0, 1)


def test_elementwise_empty(M):
    Q = M[0]
    q = Q.quantize_tensor(torch.randn(0, 4, device=DEV), torch.ones(0, 1, device=DEV),
                          torch.zeros(0, 1, device=DEV), 4, False)
    assert q.shape == (0, 4)
    d = Q.dequantize_tensor(torch.zeros(0, 4, device=DEV), torch.ones(0, 1, device=DEV),
                            torch.zeros(0, 1, device=DEV))
    assert d.shape == (0, 4)
    assert Q.ste_round(torch.randn(0, device=DEV)).shape == (0,)


def test_hadamard_empty(M):
    R = M[1]
    y = R.fast_hadamard_transform(torch.randn(0, 256, device=DEV))
    assert y.shape == (0, 256)
    with pytest.raises(AssertionError):  # last dim must be a power of 2 (rotation.py)
        R.fast_hadamard_transform(torch.randn(3, 0, device=DEV))


def test_nf4_empty(M):
    Qq = M[2]
    codes, scales = Qq.nf4_quantize(torch.randn(0, device=DEV), 64)
    assert codes.shape == (0,) and scales.shape == (0,)
    assert Qq.nf4_dequantize(codes, scales, 64).shape == (0,)
    qs, ds = Qq.double_quantize(torch.randn(0, device=DEV))
    assert qs.shape == (0,) and ds.shape == (0,)
    ql = Qq.QLoRALinear(256, 64, rank=8).to(DEV)
    ql.pack_base((torch.randn(64, 256) * 0.02).to(DEV))
    assert ql(torch.randn(0, 256, device=DEV)).shape == (0, 64)


def test_kv_empty_tokens(M):
    KV = M[3]
    k = torch.randn(1, 2, 0, 64, device=DEV)
    q, s, z = KV.PerTokenKVCacheQuantizer(8).quantize(k)
    assert q.shape == (1, 2, 0, 64) and s.shape == (1, 2, 0, 1) and z.shape == (1, 2, 0, 1)
    with pytest.raises(IndexError):  # amax over a zero-size token dim (per-channel)
        KV.PerChannelKVCacheQuantizer(8).quantize(k)
    with pytest.raises(IndexError):  # amax over a zero-size head dim (per-token)
        KV.PerTokenKVCacheQuantizer(8).quantize(torch.randn(1, 2, 3, 0, device=DEV))
    cache = KV.QuantizedKVCache(1)
    kk, vv = cache.update(0, k, k)
    assert kk.shape == (1, 2, 0, 64) and vv.shape == (1, 2, 0, 64)
    # a later chunk with tokens lands after the empty one
    k2 = torch.randn(1, 2, 5, 64, device=DEV)
    kk, vv = cache.update(0, k2, k2)
    assert kk.shape == (1, 2, 5, 64)
    ref = KV.QuantizedKVCache(1)
    rk, _ = ref.update(0, k2, k2)
    assert torch.equal(kk, rk)
