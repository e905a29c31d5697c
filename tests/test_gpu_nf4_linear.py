"""GPU tests of the fused NF4 base product of QLoRALinear.forward
(qlora.py:306-312) for fp16 / bf16 activations.

The reference's forward computes F.linear(x, _dequantize_base(), bias) plus
the LoRA term; with a half-precision base that call raises (its bias and LoRA
factors are fp32), so the oracle here is the same sum computed in fp32 from
the module's own dequantized base weight (which the QLoRA tests pin bit for
bit against the reference).  Tolerance, as for QuantizedLinear's W4A16
forward: max |y - y_ref| <= 1e-2 * max |y_ref|.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def _module(L, N, K, dtype, gs, dq, seed, rank=8):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).to(dtype).cuda()
    ql = L.QLoRALinear(K, N, rank=rank, group_size=gs, double_quant=dq).cuda()
    with torch.no_grad():
        ql.lora_B.copy_(torch.randn(N, rank, generator=g) * 0.05)
        ql.bias.copy_(torch.randn(N, generator=g) * 0.1)
    ql.pack_base(w)
    return ql, g


def _reference(ql, x):
    w = ql._dequantize_base().float()
    xf = x.float()
    return (xf @ w.T + ql.bias.float()
            + (xf @ ql.lora_A.float().T) @ ql.lora_B.float().T * ql.scaling)


def _check(y, ref):
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, (err, ref.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,K,gs,dq", [(128, 64, 64, True), (256, 128, 64, False),
                                       (384, 4096, 64, True), (128, 512, 128, True)])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 64, 100, 300])
def test_fused_forward_matches_fp32_reference(L, dtype, N, K, gs, dq, M):
    ql, g = _module(L, N, K, dtype, gs, dq, seed=N + K + M)
    x = torch.randn(M, K, generator=g).to(dtype).cuda()
    from llm_quant_b200 import nf4_linear
    assert nf4_linear.eligible(ql, x)
    y = ql(x)
    assert y.dtype == dtype and y.shape == (M, N)
    _check(y, _reference(ql, x))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [300, 1000])
def test_fused_forward_many_tiles_per_sm(L, dtype, M):
    """N = 8192: more 128 x BT tiles than SMs (several waves), the last
    token tile partial."""
    ql, g = _module(L, 8192, 1024, dtype, 64, True, seed=M)
    x = torch.randn(M, 1024, generator=g).to(dtype).cuda()
    _check(ql(x), _reference(ql, x))


def test_fused_forward_3d_input_and_no_bias(L):
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(256, 256, generator=g) * 0.02).to(torch.bfloat16).cuda()
    ql = L.QLoRALinear(256, 256, rank=4, group_size=64, bias=False).cuda()
    ql.pack_base(w)
    x = torch.randn(2, 7, 256, generator=g).to(torch.bfloat16).cuda()
    y = ql(x)
    assert y.shape == (2, 7, 256)
    w_ = ql._dequantize_base().float()
    ref = x.float() @ w_.T  # lora_B is zero-initialised
    _check(y, ref)


def test_gradients_flow(L):
    ql, g = _module(L, 256, 512, torch.bfloat16, 64, True, seed=11)
    x = torch.randn(33, 512, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    y = ql(x)
    gy = torch.randn_like(y)
    y.backward(gy)
    assert x.grad is not None and ql.lora_A.grad is not None and ql.lora_B.grad is not None
    assert ql.bias.grad is not None
    np.testing.assert_allclose(ql.bias.grad.cpu().numpy(), gy.float().sum(0).cpu().numpy(),
                               rtol=1e-5, atol=1e-4)
    # x.grad against the fp32 chain rule of the same forward
    w = ql._dequantize_base().float()
    lora_w = (ql.lora_B.float() @ ql.lora_A.float()) * ql.scaling
    ref = gy.float() @ (w + lora_w)
    _check(x.grad, ref)


def test_operand_rebuilt_after_repack(L):
    ql, g = _module(L, 128, 256, torch.bfloat16, 64, True, seed=21)
    x = torch.randn(20, 256, generator=g).to(torch.bfloat16).cuda()
    y1 = ql(x)
    w2 = (torch.randn(128, 256, generator=g) * 0.05).to(torch.bfloat16).cuda()
    ql.pack_base(w2)
    y2 = ql(x)
    _check(y2, _reference(ql, x))
    assert not torch.equal(y1, y2)


def test_fp32_path_is_the_reference_computation(L):
    g = torch.Generator().manual_seed(3)
    w = torch.randn(128, 64, generator=g).cuda() * 0.02
    ql = L.QLoRALinear(64, 128, rank=4, group_size=64).cuda()
    ql.pack_base(w)
    x = torch.randn(5, 64, generator=g).cuda()
    from llm_quant_b200 import nf4_linear
    assert not nf4_linear.eligible(ql, x)
    wb = ql._dequantize_base()
    ref = torch.nn.functional.linear(x, wb, ql.bias) + torch.nn.functional.linear(
        torch.nn.functional.linear(x, ql.lora_A), ql.lora_B) * ql.scaling
    assert torch.equal(ql(x), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,rank", [(1, 16), (5, 64), (8, 48), (16, 32), (16, 16), (17, 16), (200, 2),
                                    (1024, 16), (300, 24), (64, 5)])
def test_lora_fused_and_fallback(L, dtype, M, rank):
    """The LoRA term inside the base kernel (even rank <= 16 above 8 tokens,
    <= 64 up to 8) and the unfused path for other ranks give the fp32
    reference within the same bound."""
    from llm_quant_b200 import nf4_linear
    ql, g = _module(L, 256, 1024, dtype, 64, True, seed=M * 7 + rank, rank=rank)
    with torch.no_grad():
        ql.lora_A.copy_(torch.randn(rank, 1024, generator=g) * 0.05)
    x = torch.randn(M, 1024, generator=g).to(dtype).cuda()
    fused = nf4_linear.lora_fusable(ql, x)
    assert fused == (rank % 2 == 0 and rank <= (64 if M <= 8 else 16))
    with torch.no_grad():
        y = ql(x)
    ref = _reference(ql, x)
    _check(y, ref)
    # the LoRA term is really in the output: without it the error is large
    base = x.float() @ ql._dequantize_base().float().T + ql.bias.float()
    assert (y.float() - base).abs().max().item() > 0.1 * (ref - base).abs().max().item()


def test_lora_fused_config_shape(L):
    """Linear(4096, 14336) NF4 base, rank 16, M = 1024 (the qlora_linear bench shape)."""
    ql, g = _module(L, 14336, 4096, torch.bfloat16, 64, True, seed=99, rank=16)
    with torch.no_grad():
        ql.lora_A.copy_(torch.randn(16, 4096, generator=g) * 0.02)
    x = torch.randn(1024, 4096, generator=g).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y = ql(x)
    _check(y, _reference(ql, x))


@pytest.mark.parametrize("sdtype,pdtype", [(torch.bfloat16, torch.float32), (torch.float16, torch.float16),
                                           (torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32)])
@pytest.mark.parametrize("dq", [True, False])
@pytest.mark.parametrize("rank", [1, 16, 64])
def test_merge_lora_one_pass(L, sdtype, pdtype, dq, rank):
    """merge_lora = _dequantize_base() + scaling * lora_B @ lora_A, in the
    promoted dtype: the base part bit-exact, the rank-r product to float
    rounding of its summation order."""
    g = torch.Generator().manual_seed(rank + int(dq))
    N, K = 384, 640
    w = (torch.randn(N, K, generator=g) * 0.02).to(sdtype).cuda()
    ql = L.QLoRALinear(K, N, rank=rank, group_size=64, double_quant=dq).cuda()
    ql.pack_base(w)
    with torch.no_grad():
        ql.lora_A.copy_(torch.randn(rank, K, generator=g) * 0.05)
        ql.lora_B.copy_(torch.randn(N, rank, generator=g) * 0.05)
    ql.lora_A.data = ql.lora_A.data.to(pdtype)
    ql.lora_B.data = ql.lora_B.data.to(pdtype)
    from llm_quant_b200 import nf4_linear
    assert nf4_linear.merge_fusable(ql)
    with torch.no_grad():
        m = ql.merge_lora()
        ref = ql._dequantize_base() + ql.scaling * (ql.lora_B @ ql.lora_A)
    assert m.dtype == ref.dtype == torch.promote_types(sdtype, pdtype)
    tol = 1e-5 if m.dtype == torch.float32 else 1e-2
    torch.testing.assert_close(m.float(), ref.float(), rtol=tol, atol=tol * ref.abs().max().item())
    with torch.no_grad():  # a zero LoRA update leaves exactly the dequantized base
        ql.lora_B.zero_()
        assert torch.equal(ql.merge_lora().to(ref.dtype), ql._dequantize_base().to(ref.dtype))


def test_merge_lora_gradients(L):
    g = torch.Generator().manual_seed(8)
    w = (torch.randn(128, 256, generator=g) * 0.02).to(torch.bfloat16).cuda()
    ql = L.QLoRALinear(256, 128, rank=8, group_size=64).cuda()
    ql.pack_base(w)
    with torch.no_grad():
        ql.lora_B.copy_(torch.randn(128, 8, generator=g) * 0.05)
    m = ql.merge_lora()
    gm = torch.randn(m.shape, generator=g).cuda()
    m.backward(gm)
    a, b = ql.lora_A.detach(), ql.lora_B.detach()
    torch.testing.assert_close(ql.lora_A.grad, ql.scaling * b.t() @ gm, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ql.lora_B.grad, ql.scaling * gm @ a.t(), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("a_dtype", ["f32", "act"])
@pytest.mark.parametrize("M,K,rank", [(1, 64, 1), (5, 256, 7), (16, 1024, 16), (17, 4096, 16),
                                      (100, 512, 32), (33, 640, 48), (1024, 4096, 64)])
def test_lora_u_kernel(L, dtype, a_dtype, M, K, rank):
    """lq_lora_u = scaling * x @ lora_A^T in columns < rank, zeros up to 64,
    rounded once to the activation dtype (fp32 accumulation)."""
    from llm_quant_b200 import _C
    g = torch.Generator().manual_seed(M * 131 + rank)
    x = torch.randn(M, K, generator=g).to(dtype).cuda()
    a = (torch.randn(rank, K, generator=g) * 0.05).cuda()
    if a_dtype == "act":
        a = a.to(dtype)
    u = torch.full((M, 64), float("nan"), dtype=dtype, device="cuda")
    _C.call("lq_lora_u", x.data_ptr(), _C.dt(x), M, K, a.data_ptr(), _C.dt(a), rank, 0.75,
            u.data_ptr(), _C.stream_ptr(x))
    ref = 0.75 * (x.float() @ a.to(dtype).float().T)
    torch.testing.assert_close(u[:, :rank].float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item() + 1e-3)
    assert torch.equal(u[:, rank:].float(), torch.zeros(M, 64 - rank, device="cuda"))


def test_lora_b_cast_follows_updates(L):
    """The cached activation-dtype copy of lora_B is rebuilt after an in-place
    update (optimizer step) and after the parameter is rebound."""
    ql, g = _module(L, 256, 512, torch.bfloat16, 64, True, seed=77, rank=8)
    with torch.no_grad():
        ql.lora_A.copy_(torch.randn(8, 512, generator=g) * 0.05)
    x = torch.randn(4, 512, generator=g).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y1 = ql(x)
        ql.lora_B.add_(0.5)
        y2 = ql(x)
        _check(y2, _reference(ql, x))
        assert not torch.equal(y1, y2)
        ql.lora_B.data = torch.randn(256, 8, generator=g).cuda() * 0.1
        _check(ql(x), _reference(ql, x))


@pytest.mark.parametrize("M,N", [(4, 256), (300, 256), (1000, 14336)])
def test_two_entry_points_agree(L, M, N):
    """lq_nf4_qlora_forward (u kernel + fused kernel started behind it) and
    lq_lora_u followed by lq_nf4_linear_lora give bit-identical outputs.  At
    M = 1000, N = 14336 the fused kernel's last wave leaves 32 SMs idle and the
    u kernel runs on 32 blocks of two 16-token tiles each."""
    from llm_quant_b200 import _C, nf4_linear
    ql, g = _module(L, N, 1024, torch.bfloat16, 64, True, seed=M + 3, rank=16)
    with torch.no_grad():
        ql.lora_A.copy_(torch.randn(16, 1024, generator=g) * 0.05)
    x = torch.randn(M, 1024, generator=g).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y1 = ql(x)
    packed = nf4_linear.packed_operand(ql, x.dtype)
    a = ql.lora_A.detach().to(x.dtype).contiguous()
    lb = ql.lora_B.detach().to(x.dtype).contiguous()
    u = torch.empty(M, 64, dtype=x.dtype, device="cuda")
    y2 = torch.empty(M, N, dtype=x.dtype, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _C.stream_ptr(x)
    _C.call("lq_lora_u", x.data_ptr(), _C.dt(x), M, 1024, a.data_ptr(), _C.dt(a), 16, float(ql.scaling),
            u.data_ptr(), st)
    _C.call("lq_nf4_linear_lora", x.data_ptr(), _C.dt(x), M, N, 1024, packed.data_ptr(),
            ql.bias.detach().float().contiguous().data_ptr(), u.data_ptr(), lb.data_ptr(), 16, y2.data_ptr(),
            err.data_ptr(), st)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.equal(y1, y2)
