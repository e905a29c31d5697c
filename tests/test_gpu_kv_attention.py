"""GPU numerics: decode attention straight from the quantized KV cache
(QuantizedKVCache.attend -> lq_kv_attention).

The oracle is the reference's own dequantized cache (kv_cache_quant.py:221-267,
what update() returns; QuantizedKVCacheOracle restates it and the KV golden
tests pin it bit for bit) followed by float64 softmax attention
(oracle.kv_attention, itself checked against torch's SDPA on CPU).

Tolerance: the kernel takes the codes into the tensor cores as exact f16
integers (code - zero), the query as f16 hi + lo halves wherever a scale
is folded into it, the probabilities as f16 hi + lo halves, and accumulates
in fp32, so an fp32 result agrees to ~1e-6 relative; the bound below is
max|out - ref| <= 2e-5 * max|ref| for fp32 queries, and one rounding of the
output dtype (2^-8 for bf16, 2^-11 for fp16, relative to max|ref|) more for
half-precision queries.
"""

import numpy as np
import pytest
import torch

from gpu_util import to_np
from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def _tol(dtype):
    return {torch.float32: 2e-5, torch.float16: 2e-5 + 2.0 ** -11, torch.bfloat16: 2e-5 + 2.0 ** -8}[dtype]


def _check(out, q, cache, layer, scale=None, causal=False):
    fk, fv = cache.get(layer)
    ref = O.kv_attention(to_np(q.float()), to_np(fk), to_np(fv), scale, causal)
    got = to_np(out.float()).astype(np.float64)
    assert out.dtype == q.dtype and out.shape == q.shape
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    bound = _tol(q.dtype) * np.abs(ref).max()
    assert err <= bound, (err, bound)
    return err


def _fill(L, cache, B, H, D, chunks, dtype, seed, layer=0):
    g = torch.Generator().manual_seed(seed)
    for n in chunks:
        k = (torch.randn(B, H, n, D, generator=g) * 2).to(dtype).cuda()
        v = torch.randn(B, H, n, D, generator=g).to(dtype).cuda()
        cache.append(layer, k, v)


def _gran(L, name):
    return L.KVQuantGranularity(name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T", [1, 5, 16, 200, 1000, 4099])
def test_per_token_int8_default(L, dtype, T):
    cache = L.QuantizedKVCache(1)  # PerTokenKVCacheQuantizer(8), symmetric int8
    _fill(L, cache, 2, 2, 128, [T], dtype, T)
    q = torch.randn(2, 8, 1, 128, generator=torch.Generator().manual_seed(7)).to(dtype).cuda()
    _check(cache.attend(0, q), q, cache, 0)


@pytest.mark.parametrize("gran", ["per_token", "per_channel", "per_group"])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("D", [64, 128])
def test_granularities_codes_dims(L, gran, sym, bits, D):
    qz = L.KVCacheQuantizer(bits, sym, _gran(L, gran), 32)
    cache = L.QuantizedKVCache(1, qz)
    _fill(L, cache, 2, 3, D, [70, 1, 300], torch.float16, bits * 10 + D)
    q = torch.randn(2, 6, 1, D, generator=torch.Generator().manual_seed(3)).half().cuda()
    _check(cache.attend(0, q), q, cache, 0)
    qf = q.float()
    _check(cache.attend(0, qf), qf, cache, 0)


@pytest.mark.parametrize("kgran,vgran", [("per_token", "per_channel"), ("per_channel", "per_group"),
                                         ("per_group", "per_token")])
def test_separate_value_quantizer(L, kgran, vgran):
    cache = L.QuantizedKVCache(1, L.KVCacheQuantizer(8, True, _gran(L, kgran), 16),
                               value_quantizer=L.KVCacheQuantizer(6, True, _gran(L, vgran), 48))
    _fill(L, cache, 1, 2, 128, [100, 157], torch.bfloat16, 11)
    q = torch.randn(1, 8, 1, 128, generator=torch.Generator().manual_seed(4)).bfloat16().cuda()
    _check(cache.attend(0, q), q, cache, 0)


@pytest.mark.parametrize("G,Sq", [(1, 1), (4, 1), (8, 1), (4, 3), (16, 1), (5, 5), (32, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_query_rows_and_causal(L, G, Sq, causal):
    cache = L.QuantizedKVCache(1)
    _fill(L, cache, 2, 2, 128, [333], torch.float16, G * 10 + Sq)
    q = torch.randn(2, 2 * G, Sq, 128, generator=torch.Generator().manual_seed(G)).half().cuda()
    _check(cache.attend(0, q, causal=causal), q, cache, 0, causal=causal)


def test_scale_argument_and_update_path(L):
    cache = L.QuantizedKVCache(2, max_seq_len=100)  # odd reserve -> rounded capacity
    g = torch.Generator().manual_seed(0)
    for n in (40, 1, 1, 30):
        k = torch.randn(1, 4, n, 64, generator=g).half().cuda()
        v = torch.randn(1, 4, n, 64, generator=g).half().cuda()
        fk, fv = cache.update(1, k, v)
    q = torch.randn(1, 4, 1, 64, generator=g).half().cuda()
    _check(cache.attend(1, q, scale=0.3), q, cache, 1, scale=0.3)
    # against torch's SDPA over the dequantized cache (the reference's caller path)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), fk, fv, scale=0.3)
    assert (cache.attend(1, q, scale=0.3).float() - ref).abs().max() <= 2.0 ** -10 * ref.abs().max()


def test_large_batch_splits(L):
    """Many heads and a long cache: token splits plus the combine kernel."""
    cache = L.QuantizedKVCache(1)
    _fill(L, cache, 4, 8, 128, [2048, 2048, 100], torch.float16, 5)
    q = torch.randn(4, 32, 1, 128, generator=torch.Generator().manual_seed(9)).half().cuda()
    _check(cache.attend(0, q), q, cache, 0)


def test_matches_oracle_cache_directly(L):
    """The dequantized cache used as the reference equals the oracle's own
    restatement of QuantizedKVCache bit for bit on the same chunks."""
    g = torch.Generator().manual_seed(21)
    p = dict(n_bits=8, symmetric=False, granularity="per_token", group_size=32)
    cache = L.QuantizedKVCache(1, L.KVCacheQuantizer(8, False, _gran(L, "per_token"), 32))
    oc = O.QuantizedKVCacheOracle(1, "float16", p)
    for n in (17, 50):
        k = torch.randn(1, 2, n, 128, generator=g).half()
        v = torch.randn(1, 2, n, 128, generator=g).half()
        cache.append(0, k.cuda(), v.cuda())
        fk, fv = oc.update(0, k.float().numpy(), v.float().numpy())
    gk, gv = cache.get(0)
    assert np.array_equal(to_np(gk).view(np.uint32), fk.astype(np.float32).view(np.uint32))
    assert np.array_equal(to_np(gv).view(np.uint32), fv.astype(np.float32).view(np.uint32))
    q = torch.randn(1, 4, 1, 128, generator=g).float()
    out = cache.attend(0, q.cuda())
    ref = O.kv_attention(q.numpy(), fk, fv)
    assert np.abs(to_np(out) - ref).max() <= 2e-5 * np.abs(ref).max()


def test_unsupported_configs_raise(L):
    cache = L.QuantizedKVCache(1, L.KVCacheQuantizer(12, False, _gran(L, "per_token"), 32))
    _fill(L, cache, 1, 1, 64, [10], torch.float32, 0)
    with pytest.raises(NotImplementedError):
        cache.attend(0, torch.randn(1, 1, 1, 64).cuda())
    cache = L.QuantizedKVCache(1, L.KVCacheQuantizer(8, True, _gran(L, "per_group"), 8))
    _fill(L, cache, 1, 1, 64, [10], torch.float32, 0)
    with pytest.raises(NotImplementedError):
        cache.attend(0, torch.randn(1, 1, 1, 64).cuda())
    cache = L.QuantizedKVCache(1)
    _fill(L, cache, 1, 2, 96, [10], torch.float16, 0)
    with pytest.raises(ValueError):
        cache.attend(0, torch.randn(1, 2, 1, 96).half().cuda())
    with pytest.raises(RuntimeError):
        cache.attend(0, torch.randn(1, 3, 1, 96).half().cuda())
