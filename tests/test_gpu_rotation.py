"""GPU parity: Hadamard transform and the fused rotate + fake-quant path.

The reference transform is a dense matmul (core/rotation.py:146-147) whose
summation order cannot be reproduced by a butterfly, so the transform is
checked within tolerance -- 1e-5 absolute/relative for fp32 as in the
reference's own test (tests/test_rotation.py:100-106), 1e-2 relative for
bf16/fp16 -- against the reference outputs and against an exact float64
butterfly.  The fused quantization step is then checked BIT-EXACT against
the oracle's fake_quantize applied to this implementation's own transform.
"""

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


def _tol(dt):
    return 1e-5 if dt == "float32" else 1e-2


@pytest.mark.parametrize("name,c", list(cases("rotation.npz", "fht")),
                         ids=lambda v: v if isinstance(v, str) else "")
def test_fht_golden(L, name, c):
    dt = c["params"]["dtype"]
    y = L.fast_hadamard_transform(to_dev(c["x"][0], dt))
    t = _tol(dt)
    np.testing.assert_allclose(to_np(y), c["y"][0], rtol=t, atol=t)


@pytest.mark.parametrize("dt", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("d", [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192,
                               16384, 32768])
def test_fht_all_sizes_vs_exact(L, dt, d):
    rows = max(1, min(64, (1 << 20) // d))
    x = O.rnd(seeded((rows, d), d).numpy(), dt)
    y = to_np(L.fast_hadamard_transform(to_dev(x, dt)))
    ref = O.fast_hadamard_transform(x, dt)
    # the exact result rounded once; the fp32 butterfly may differ by a few ulps
    t = 2e-5 if dt == "float32" else 1e-2
    scale = np.abs(x).max() * np.sqrt(d) / np.sqrt(d)
    np.testing.assert_allclose(y, ref, rtol=t, atol=t * max(1.0, scale))


def test_fht_3d_and_orthogonal(L):
    x = torch.randn(2, 8, 32, device="cuda")
    y = L.fast_hadamard_transform(x)
    assert y.shape == (2, 8, 32)
    # H is orthogonal and symmetric: applying it twice gives x back
    np.testing.assert_allclose(to_np(L.fast_hadamard_transform(y)), to_np(x), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dt", ["bfloat16", "float32", "float16"])
@pytest.mark.parametrize("d", [64, 1024, 2048, 4096, 8192, 16384])
@pytest.mark.parametrize("sym,bits", [(True, 4), (False, 4), (True, 8)])
def test_fused_rotate_quant_bit_exact_on_own_transform(L, dt, d, sym, bits):
    x = O.rnd(seeded((96, d), 5, 1.0, outliers=max(1, d // 100), factor=50.0).numpy(), dt)
    xd = to_dev(x, dt)
    h = to_np(L.fast_hadamard_transform(xd))
    fq, s, z = L.hadamard_fake_quantize(xd, bits, sym, return_qparams=True)
    ref = O.fake_quantize(h, dt, bits, sym, "per_channel")
    so, zo = O.compute_qparams(h, dt, bits, sym, "per_channel")
    assert same_bits(to_np(s), so) and same_bits(to_np(z), zo)
    assert same_bits(to_np(fq), ref)


def _edge_rows(d, dt):
    """Rows whose transforms are ordinary, constant, a narrow all-positive
    range, zero, tiny (scale below 2^-126), NaN, +-inf, huge and with strong
    outliers: every branch of the fused kernels' quantization."""
    rng = np.random.default_rng(d)
    rows = [rng.standard_normal(d)]
    e = np.zeros(d)
    e[0] = 3.0
    rows.append(e.copy())
    e[5] = 0.01
    rows.append(e)
    rows.append(np.zeros(d))
    rows.append(rng.standard_normal(d) * 1e-38)
    r = rng.standard_normal(d)
    r[7] = np.nan
    rows.append(r)
    r = rng.standard_normal(d)
    r[9] = np.inf
    rows.append(r)
    r = rng.standard_normal(d)
    r[3] = -np.inf
    rows.append(r)
    rows.append(rng.standard_normal(d) * 1e30)
    r = rng.standard_normal(d)
    r[::17] *= 100
    rows.append(r)
    rows.append(np.abs(rng.standard_normal(d)) + 40.0)
    return O.rnd(np.stack(rows).astype(np.float32), dt)


@pytest.mark.parametrize("dt", ["bfloat16", "float32", "float16"])
@pytest.mark.parametrize("d", [2048, 4096, 8192])
@pytest.mark.parametrize("sym,bits", [(True, 4), (False, 4), (True, 8), (False, 8), (True, 2)])
def test_fused_rotate_quant_edge_rows(L, dt, d, sym, bits):
    x = _edge_rows(d, dt)
    xd = to_dev(x, dt)
    h = to_np(L.fast_hadamard_transform(xd))
    fq, s, z = L.hadamard_fake_quantize(xd, bits, sym, return_qparams=True)
    so, zo = O.compute_qparams(h, dt, bits, sym, "per_channel")
    assert same_bits(to_np(s), so) and same_bits(to_np(z), zo)
    assert same_bits(to_np(fq), O.fake_quantize(h, dt, bits, sym, "per_channel"))


def test_config2_full_size(L):
    """QuaRot activation path, bf16 [8192, 4096], 1% channels x50 (seed 0)."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(8192, 4096, generator=g)
    idx = torch.randperm(4096, generator=g)[:41]
    a[:, idx] *= 50
    a = a.to(torch.bfloat16).cuda()
    h = L.fast_hadamard_transform(a)
    # transform vs exact (sampled rows to keep the float64 oracle fast)
    rows = torch.arange(0, 8192, 61)
    hx = to_np(h[rows])
    ref = O.fast_hadamard_transform(to_np(a[rows]), "bfloat16")
    np.testing.assert_allclose(hx, ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())
    fq = L.hadamard_fake_quantize(a, 4, True)
    unfused = L.fake_quantize(h, 4, True, L.QScheme.PER_CHANNEL)
    assert torch.equal(fq.view(torch.int16), unfused.view(torch.int16))
    assert same_bits(to_np(fq[rows]), O.fake_quantize(hx, "bfloat16", 4, True, "per_channel"))
