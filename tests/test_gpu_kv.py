"""GPU parity: KV-cache quantizers and QuantizedKVCache.update, bit-exact."""

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


def _qz(L, p):
    return L.KVCacheQuantizer(p["n_bits"], p["symmetric"], L.KVQuantGranularity(p["granularity"]),
                              p["group_size"])


@pytest.mark.parametrize("name,c", list(cases("kv.npz", "kv")), ids=_ids)
def test_kv_quantizer_golden(L, name, c):
    p = c["params"]
    qz = _qz(L, p)
    x = to_dev(c["x"][0], p["dtype"])
    q, s, z = qz.quantize(x)
    assert q.dtype == (torch.int8 if p["symmetric"] else torch.int16)
    assert np.array_equal(to_np(q), c["q"][0])
    assert tuple(s.shape) == c["scale"][0].shape
    assert same_bits(to_np(s), c["scale"][0]) and same_bits(to_np(z), c["zp"][0])
    deq = qz.dequantize(q, s, z)
    assert deq.dtype == torch.float32
    assert same_bits(to_np(deq), c["deq"][0])
    assert same_bits(to_np(qz.fake_quantize(x)), c["deq"][0])
    s2, z2 = qz._compute_qparams(x)
    so = c["scale"][0] if p["granularity"] != "per_group" else c["scale"][0][:, :, :, None, :]
    assert same_bits(to_np(s2), so)


@pytest.mark.parametrize("name,c", list(cases("kv.npz", "kv_cache")), ids=_ids)
def test_kv_cache_golden(L, name, c):
    p = c["params"]
    cache = L.QuantizedKVCache(2, _qz(L, p))
    total = 0
    for j, n in enumerate(p["chunks"]):
        fk, fv = cache.update(1, to_dev(*c[f"k{j}"]), to_dev(*c[f"v{j}"]))
        total += n
        assert fk.shape[2] == total
        assert same_bits(to_np(fk), c[f"fk{j}"][0]), j
        assert same_bits(to_np(fv), c[f"fv{j}"][0]), j
    assert cache.get(0) is None
    fk2, fv2 = cache.get(1)
    assert torch.equal(fk2, fk) and torch.equal(fv2, fv)
    assert cache._cache[1][0].shape[2] == total


def test_kv_cache_mixed_granularity_golden(L):
    (_, c), = list(cases("kv.npz", "kv_cache_mixed"))
    G = L.KVQuantGranularity
    cache = L.QuantizedKVCache(1, L.KVCacheQuantizer(8, True, G.PER_CHANNEL),
                               value_quantizer=L.KVCacheQuantizer(4, True, G.PER_TOKEN))
    for j in range(3):
        fk, fv = cache.update(0, to_dev(*c[f"k{j}"]), to_dev(*c[f"v{j}"]))
        assert same_bits(to_np(fk), c[f"fk{j}"][0]) and same_bits(to_np(fv), c[f"fv{j}"][0])


@pytest.mark.parametrize("gran", ["per_token", "per_channel", "per_group"])
@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_kv_cache_capacity_growth_vs_oracle(L, gran, dtype):
    """Many ragged chunks (forcing several capacity doublings) against the oracle cache."""
    qcfg = dict(n_bits=4 if gran == "per_token" else 8, symmetric=gran != "per_group",
                granularity=gran, group_size=4)
    qz = L.KVCacheQuantizer(qcfg["n_bits"], qcfg["symmetric"], L.KVQuantGranularity(gran), 4)
    cache = L.QuantizedKVCache(1, qz)
    ocache = O.QuantizedKVCacheOracle(1, dtype, qcfg)
    g = torch.Generator().manual_seed(4)
    for j, n in enumerate([3, 70, 1, 5, 130, 64]):
        k = O.rnd((torch.randn(2, 3, n, 48, generator=g) * (1 + j)).numpy(), dtype)
        v = O.rnd(torch.randn(2, 3, n, 48, generator=g).numpy(), dtype)
        fk, fv = cache.update(0, to_dev(k, dtype), to_dev(v, dtype))
        ok, ov = ocache.update(0, k, v)
        assert same_bits(to_np(fk), ok) and same_bits(to_np(fv), ov), j


@pytest.mark.parametrize("gran", ["per_token", "per_channel", "per_group"])
@pytest.mark.parametrize("n_bits,head_dim", [(12, 48), (8, 6), (4, 20), (12, 10)])
def test_kv_cache_code_widths_and_head_dims(L, gran, n_bits, head_dim):
    """16-bit codes (n_bits > 8), head dims that are not powers of two or not
    multiples of 4, ragged chunks: full-cache read-out bit-exact vs the oracle."""
    qcfg = dict(n_bits=n_bits, symmetric=gran != "per_channel", granularity=gran, group_size=2)
    qz = L.KVCacheQuantizer(n_bits, qcfg["symmetric"], L.KVQuantGranularity(gran), 2)
    cache = L.QuantizedKVCache(1, qz)
    ocache = O.QuantizedKVCacheOracle(1, "bfloat16", qcfg)
    g = torch.Generator().manual_seed(9)
    for j, n in enumerate([5, 33, 2, 67]):
        k = O.rnd((torch.randn(2, 2, n, head_dim, generator=g) * (1 + j)).numpy(), "bfloat16")
        v = O.rnd(torch.randn(2, 2, n, head_dim, generator=g).numpy(), "bfloat16")
        fk, fv = cache.update(0, to_dev(k, "bfloat16"), to_dev(v, "bfloat16"))
        ok, ov = ocache.update(0, k, v)
        assert same_bits(to_np(fk), ok) and same_bits(to_np(fv), ov), j


def test_config3_layer(L):
    """One layer of the KV workload: K per-channel INT8, V per-token INT4, bf16
    [16, 8, 8192, 128] in 16 updates of 512 tokens; final update vs oracle."""
    G = L.KVQuantGranularity
    cache = L.QuantizedKVCache(1, L.PerChannelKVCacheQuantizer(8),
                               value_quantizer=L.PerTokenKVCacheQuantizer(4), max_seq_len=8192)
    g = torch.Generator().manual_seed(0)
    B, H, D, C = 16, 8, 128, 512
    kch, vch = [], []
    for j in range(16):
        k = torch.randn(B, H, C, D, generator=g)
        k[:, :, :, :4] *= 20
        v = torch.randn(B, H, C, D, generator=g)
        kch.append(k.to(torch.bfloat16))
        vch.append(v.to(torch.bfloat16))
        fk, fv = cache.update(0, kch[-1].cuda(), vch[-1].cuda())
    assert fk.shape == (B, H, 8192, D) and fv.dtype == torch.float32
    # oracle on a slice of batch / heads (per-channel and per-token qparams are
    # independent across (b, h)), replaying all 16 updates
    oc = O.QuantizedKVCacheOracle(1, "bfloat16", dict(n_bits=8, symmetric=True, granularity="per_channel"),
                                  dict(n_bits=4, symmetric=True, granularity="per_token"))
    for j in range(16):
        ok, ov = oc.update(0, kch[j][:2, :2].float().numpy(), vch[j][:2, :2].float().numpy())
    assert same_bits(to_np(fk[:2, :2]), ok) and same_bits(to_np(fv[:2, :2]), ov)


def test_reference_cache_behaviours(L):
    """The reference tests' cache behaviours (tests/test_kv_cache_quant.py:157-228)."""
    B, H, D = 2, 4, 32
    cache = L.QuantizedKVCache(num_layers=2)
    assert cache.seq_len == 0
    for t in range(5):
        fk, fv = cache.update(0, torch.randn(B, H, 1, D, device="cuda"), torch.randn(B, H, 1, D, device="cuda"))
    assert fk.shape == (B, H, 5, D) and cache.seq_len == 5
    cache.reset()
    assert cache.seq_len == 0 and cache.get(0) is None
    k0 = torch.randn(B, H, 8, D, device="cuda")
    fk, _ = cache.update(0, k0, k0)
    assert ((k0 - fk) ** 2).mean() < 0.01
