"""GPU parity: NF4 quantization, double quantization and QLoRALinear storage.

NF4 codes bit-exact (including every bf16 / fp16 value in [-1, 1] and fp32
values within 96 ulps of each decision boundary), scales and dequantized
values bit-exact.
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


def _ids(v):
    return v if isinstance(v, str) else ""


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "nf4")), ids=_ids)
def test_nf4_golden(L, name, c):
    p = c["params"]
    x = to_dev(c["x"][0], p["dtype"])
    codes, scales = L.nf4_quantize(x, p["group_size"])
    assert codes.dtype == torch.int64 and codes.shape == x.shape
    assert np.array_equal(to_np(codes), c["codes"][0])
    assert same_bits(to_np(scales), c["scales"][0])
    deq = L.nf4_dequantize(codes, scales, p["group_size"])
    assert same_bits(to_np(deq), c["deq"][0])


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "nf4_grid")), ids=_ids)
def test_nf4_decision_grid(L, name, c):
    p = c["params"]
    codes, scales = L.nf4_quantize(to_dev(c["x"][0], p["dtype"]), p["group_size"])
    assert np.array_equal(to_np(codes).astype(np.uint8), c["codes"][0])


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "double_quant")), ids=_ids)
def test_double_quant_golden(L, name, c):
    p = c["params"]
    q, dq = L.double_quantize(to_dev(c["s"][0], p["dtype"]), p["dq_group_size"])
    assert same_bits(to_np(q), c["q"][0]) and same_bits(to_np(dq), c["dq"][0])
    rs = L.double_dequantize(q, dq, p["dq_group_size"])
    assert same_bits(to_np(rs), c["restored"][0])


@pytest.mark.parametrize("name,c", list(cases("nf4.npz", "qlora")), ids=_ids)
def test_qlora_pack_base_golden(L, name, c):
    p = c["params"]
    w = to_dev(c["w"][0], p["dtype"])
    ql = L.QLoRALinear(p["in_features"], p["out_features"], rank=4, group_size=p["group_size"],
                       double_quant=p["double_quant"]).cuda()
    ql.pack_base(w)
    assert np.array_equal(to_np(ql.nf4_codes), c["nf4_codes"][0])
    assert same_bits(to_np(ql.nf4_scales), c["nf4_scales"][0])
    if p["double_quant"]:
        assert same_bits(to_np(ql.dq_q_scales), c["dq_q_scales"][0])
        assert same_bits(to_np(ql.dq_scales), c["dq_scales"][0])
    assert same_bits(to_np(ql._dequantize_base()), c["w_base"][0])


@pytest.mark.parametrize("dtype", ["bfloat16", "float32", "float16"])
@pytest.mark.parametrize("shape,gs", [((1024, 4096), 64), ((333, 777), 64), ((64, 64), 32),
                                      ((100, 50), 16), ((7, 9), 5)])
def test_nf4_vs_oracle(L, dtype, shape, gs):
    x = O.rnd(seeded(shape, 1, 0.02, outliers=2).numpy(), dtype)
    codes, scales = L.nf4_quantize(to_dev(x, dtype), gs)
    oc, os_ = O.nf4_quantize(x, dtype, gs)
    assert np.array_equal(to_np(codes), oc) and same_bits(to_np(scales), os_)
    # fused QLoRALinear path (packed codes + double quant) on the same weight
    if len(shape) == 2:
        ql = L.QLoRALinear(shape[1], shape[0], rank=2, group_size=gs).cuda()
        ql.pack_base(to_dev(x, dtype))
        assert np.array_equal(to_np(ql.nf4_codes), oc)
        q, dq = O.double_quantize(os_, dtype, 256)
        assert same_bits(to_np(ql.dq_q_scales), q) and same_bits(to_np(ql.dq_scales), dq)
        wb = O.nf4_dequantize(oc, O.double_dequantize(q, dq, dtype, 256), dtype, gs)
        assert same_bits(to_np(ql._dequantize_base()), wb)


def _g64_edge_weight(rows, cols):
    """bf16 weight, group 64: groups holding every bf16 value in [-1, 1] next
    to a 1.0 (scale 1, so each quotient is the value itself), random groups,
    an all-zero group, a tiny-valued group, and groups with +inf, -inf, NaN."""
    n = rows * cols
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(n) * 0.02).astype(np.float32)
    grid = (np.arange(0, 0x10000, dtype=np.uint32) << 16).view(np.float32)
    with np.errstate(invalid="ignore"):
        grid = grid[np.abs(grid) <= 1]
    n_grid_groups = min((len(grid) + 62) // 63, n // 64 - 8)
    for i in range(n_grid_groups):
        part = grid[i * 63:(i + 1) * 63]
        x[i * 64] = 1.0
        x[i * 64 + 1:i * 64 + 1 + len(part)] = part
    g = n // 64
    x[(g - 1) * 64:(g - 1) * 64 + 64] = 0.0
    x[(g - 2) * 64:(g - 1) * 64] *= 1e-30
    x[(g - 3) * 64 + 5] = np.inf
    x[(g - 4) * 64 + 9] = -np.inf
    x[(g - 5) * 64 + 17] = np.nan
    return O.rnd(x.reshape(rows, cols), "bfloat16")


@pytest.mark.parametrize("double_quant", [True, False])
@pytest.mark.parametrize("shape", [(16, 4096), (3, 6400), (17, 192), (1, 64 * 9)])
def test_pack_base_bf16_g64_edges(L, shape, double_quant):
    """bf16 / group 64 / whole groups (the one-thread-per-group packing kernel):
    full and partial double-quantization super-groups, every bf16 quotient in
    [-1, 1], zero, tiny, infinite and NaN groups; codes, scales and the
    dequantized base bit-exact against the oracle."""
    x = _g64_edge_weight(*shape)
    ql = L.QLoRALinear(shape[1], shape[0], rank=2, group_size=64, double_quant=double_quant).cuda()
    ql.pack_base(to_dev(x, "bfloat16"))
    oc, os_ = O.nf4_quantize(x, "bfloat16", 64)
    assert np.array_equal(to_np(ql.nf4_codes), oc)
    if double_quant:
        q, dq = O.double_quantize(os_, "bfloat16", 256)
        assert same_bits(to_np(ql.dq_q_scales), q) and same_bits(to_np(ql.dq_scales), dq)
        s = O.double_dequantize(q, dq, "bfloat16", 256)
    else:
        assert same_bits(to_np(ql.nf4_scales), os_)
        s = os_
    assert same_bits(to_np(ql._dequantize_base()), O.nf4_dequantize(oc, s, "bfloat16", 64))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape,gs", [((40, 96), 8), ((33, 72), 24), ((9, 200), 40), ((31, 256), 128),
                                      ((5, 77), 8)])
def test_packed_unpack_group_sizes(L, dtype, shape, gs):
    """QLoRALinear._dequantize_base for groups that are multiples of 8 (the
    coalesced unpack kernel; power-of-two and other sizes) and a tail that is
    not a whole 8-element chunk, with and without double quantization."""
    x = O.rnd(seeded(shape, 3, 0.02, outliers=2).numpy(), dtype)
    oc, os_ = O.nf4_quantize(x, dtype, gs)
    for double_quant in (True, False):
        ql = L.QLoRALinear(shape[1], shape[0], rank=2, group_size=gs, double_quant=double_quant).cuda()
        ql.pack_base(to_dev(x, dtype))
        assert np.array_equal(to_np(ql.nf4_codes), oc)
        if double_quant:
            q, dq = O.double_quantize(os_, dtype, 256)
            s = O.double_dequantize(q, dq, dtype, 256)
        else:
            s = os_
        assert same_bits(to_np(ql._dequantize_base()), O.nf4_dequantize(oc, s, dtype, gs))


def test_qlora_state_dict_is_reference_format(L):
    lin = torch.nn.Linear(96, 40).cuda().to(torch.bfloat16)
    ql = L.QLoRA(rank=4, group_size=64).wrap_linear(lin)
    sd = ql.state_dict()
    assert sd["nf4_codes"].dtype == torch.int64 and sd["nf4_codes"].shape == (40, 96)
    for k in ("nf4_scales", "dq_q_scales", "dq_scales", "dq_group_size_val", "lora_A", "lora_B", "bias"):
        assert k in sd
    assert "nf4_codes_packed" not in sd
    ql2 = L.QLoRALinear(96, 40, rank=4, group_size=64).cuda()
    ql2.load_state_dict(sd)
    assert torch.equal(ql2.nf4_codes, ql.nf4_codes)
    assert torch.equal(ql2._dequantize_base(), ql._dequantize_base())


def test_config4_layer_shapes(L):
    """NF4 g64 + double quant over one Llama-3-8B layer's shapes (bf16): bit-exact."""
    g = torch.Generator().manual_seed(0)
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096),
              (14336, 4096), (4096, 14336)]
    for i, (o, k) in enumerate(shapes):
        w = (torch.randn(o, k, generator=g) * 0.02).to(torch.bfloat16)
        ql = L.QLoRALinear(k, o, rank=4, group_size=64).cuda()
        ql.pack_base(w.cuda())
        wb = ql._dequantize_base()
        if i in (1, 6):  # oracle check on two of the seven (time)
            wn = w.float().numpy()
            oc, os_ = O.nf4_quantize(wn, "bfloat16", 64)
            assert np.array_equal(to_np(ql.nf4_codes), oc)
            q, dq = O.double_quantize(os_, "bfloat16", 256)
            ref = O.nf4_dequantize(oc, O.double_dequantize(q, dq, "bfloat16", 256), "bfloat16", 64)
            assert same_bits(to_np(wb), ref)
        # round-trip quality (reference test_roundtrip bound, scaled to N(0, 0.02))
        err = ((wb.float() - w.cuda().float()) ** 2).mean().item()
        assert err < 0.05 * 0.02 ** 2 / 0.25
