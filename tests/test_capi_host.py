"""CPU-side checks of the C-ABI library and the host logic (no GPU needed).

* liblq_sm100.so builds for sm_100a and exports every function
  include/lq_sm100.h declares;
* the NF4 decision thresholds compiled into the kernel are exactly the
  smallest fp32 values at which the reference's argmin code changes
  (re-derived here from the oracle);
* the Python layer fails loudly on CPU tensors (no fallback) and raises the
  reference's exception types for bad arguments before touching a device.
"""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lq_sm100.h")
NF4_SRC = os.path.join(ROOT, "llm_quant_b200", "csrc", "lq_nf4.cu")


@pytest.fixture(scope="module")
def lib_path():
    from llm_quant_b200 import build
    return build.build()


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(lq_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("lq_group_quant", "lq_token_group_quant", "lq_kv_dequant", "lq_kv_append",
                 "lq_tensor_qparams", "lq_affine", "lq_nf4_quantize", "lq_nf4_pack",
                 "lq_nf4_unpack", "lq_hadamard", "lq_hadamard_fake_quant"):
        assert must in names, must


def test_library_exports_every_declared_symbol(lib_path):
    lib = ctypes.CDLL(lib_path)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_library_is_sm100a(lib_path):
    # cuobjdump is not used (no reading of compiled code); the build flags
    # are the evidence: every object is compiled with -gencode sm_100a.
    from llm_quant_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)


def test_status_strings(lib_path):
    lib = ctypes.CDLL(lib_path)
    lib.lq_status_string.restype = ctypes.c_char_p
    assert lib.lq_status_string(0) == b"ok"
    assert lib.lq_status_string(-1) == b"invalid argument"
    lib.lq_version.restype = ctypes.c_int
    assert lib.lq_version() >= 100


def test_argument_validation_without_gpu(lib_path):
    """Bad arguments are rejected on the host before any launch."""
    lib = ctypes.CDLL(lib_path)
    lib.lq_last_error.restype = ctypes.c_char_p
    V, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.lq_hadamard.argtypes = [V, I, L, L, V, V]
    assert lib.lq_hadamard(None, 2, 4, 12, None, None) == -1  # d not a power of two
    assert b"power of 2" in lib.lq_last_error()
    assert lib.lq_hadamard(None, 2, 4, 65536, None, None) == -6  # above maximum
    lib.lq_group_quant.argtypes = [V, I, L, L, L, I, I, I, V, I, V, V, V]
    assert lib.lq_group_quant(None, 0, 4, 8, 0, 4, 1, 1, None, 0, None, None, None) == -1
    assert lib.lq_group_quant(None, 0, 4, 8, 4, 99, 1, 1, None, 0, None, None, None) == -1
    # empty tensors are a no-op
    assert lib.lq_group_quant(None, 0, 0, 8, 4, 4, 1, 1, None, 0, None, None, None) == 0


def _attn(lib, **kw):
    """lq_kv_attention with valid defaults (B=1, Hq=4, H=2, Sq=1, D=128,
    T=20, cap=32, int8 per-token, fp16) overridden by kw; pointers fake."""
    V, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.lq_kv_attention.argtypes = [V, I, L, L, L, L, L, L, L, I, V, I, L, V, V, L, V, I, L, V, V, L,
                                    I, ctypes.c_float, I, V, V, ctypes.c_size_t, V]
    a = dict(q=None, q_dtype=1, B=1, Hq=4, H=2, Sq=1, D=128, T=20, cap=32, code_dtype=3,
             k_codes=None, k_gran=0, k_group=32, k_scale=None, k_zp=None, k_pitch=32,
             v_codes=None, v_gran=0, v_group=32, v_scale=None, v_zp=None, v_pitch=32,
             s_dtype=1, sm_scale=0.1, causal=0, out=None, ws=None, ws_bytes=0, stream=None)
    a.update(kw)
    return lib.lq_kv_attention(*a.values())


def test_kv_attention_validation_without_gpu(lib_path):
    """lq_kv_attention rejects unsupported shapes / layouts on the host."""
    lib = ctypes.CDLL(lib_path)
    lib.lq_last_error.restype = ctypes.c_char_p
    assert _attn(lib, D=96) == -1 and b"head dim" in lib.lq_last_error()
    assert _attn(lib, Hq=3) == -1
    assert _attn(lib, cap=40) == -1  # not whole 16-token tiles
    assert _attn(lib, cap=16) == -1  # below T
    assert _attn(lib, code_dtype=5) == -2
    assert _attn(lib, k_gran=2, k_group=24, k_pitch=2) == -1
    assert _attn(lib, v_gran=2, v_group=16, v_pitch=1) == -1  # 16 tokens of rows < T = 20
    assert _attn(lib, k_pitch=16) == -1
    assert _attn(lib) == -1 and b"NULL" in lib.lq_last_error()
    fake = 4096
    ptrs = dict(q=fake, k_codes=fake, v_codes=fake, k_scale=fake, k_zp=fake, v_scale=fake,
                v_zp=fake, out=fake)
    assert _attn(lib, **dict(ptrs, k_scale=fake + 8)) == -5  # 16-byte alignment
    assert _attn(lib, B=0, **ptrs) == 0  # empty batch: no work
    lib.lq_kv_attention_workspace_bytes.restype = ctypes.c_size_t
    lib.lq_kv_attention_workspace_bytes.argtypes = [ctypes.c_int64] * 6
    assert lib.lq_kv_attention_workspace_bytes(1, 4, 2, 1, 128, 20) == 0  # one split
    # 8 x 8 kv heads, 4 rows each, 8192 tokens: split along the tokens
    n = lib.lq_kv_attention_workspace_bytes(8, 32, 8, 1, 128, 8192)
    assert n > 0 and n % (8 * 8 * 4 * 130 * 4) == 0
    assert lib.lq_kv_attention_workspace_bytes(1, 3, 2, 1, 128, 20) == 0  # Hq % H: invalid


def test_oracle_attention_matches_torch_sdpa():
    """oracle.kv_attention (GQA head mapping, bottom-right causal mask) equals
    torch's scaled_dot_product_attention in float64 on CPU."""
    import torch
    from oracle.lq_oracle import kv_attention
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 6, 4, 32))
    k = rng.standard_normal((2, 3, 40, 32))
    v = rng.standard_normal((2, 3, 40, 32))
    kt = torch.from_numpy(k).repeat_interleave(2, 1)
    vt = torch.from_numpy(v).repeat_interleave(2, 1)
    for causal in (False, True):
        mask = torch.ones(4, 40, dtype=torch.bool).tril(40 - 4) if causal else None
        ref = torch.nn.functional.scaled_dot_product_attention(torch.from_numpy(q), kt, vt,
                                                               attn_mask=mask, scale=0.2)
        assert np.abs(kv_attention(q, k, v, 0.2, causal) - ref.numpy()).max() < 1e-12


def _oracle_thresholds(dtype="float32"):
    """Smallest fp32 quotient p at which the reference's code of round_dtype(p)
    reaches i, for i = 1..15 (bisection over fp32 bit patterns)."""
    from oracle.lq_oracle import nf4_encode, rnd

    def code(v):
        return int(nf4_encode(rnd(np.array([v], np.float32), dtype))[0])

    def key(f):
        u = int(np.array([f], np.float32).view(np.int32)[0])
        return u if u >= 0 else -(u & 0x7FFFFFFF)

    def unkey(k):
        u = k if k >= 0 else ((-k) | -(2 ** 31))
        return np.array([u], np.int32).view(np.float32)[0]

    out = []
    for i in range(1, 16):
        lo, hi = key(np.float32(-1.0)), key(np.float32(1.0))
        while hi - lo > 1:
            mid = (lo + hi) // 2
            if code(unkey(mid)) >= i:
                hi = mid
            else:
                lo = mid
        out.append(np.float32(unkey(hi)))
    return out


def _kernel_theta_rows():
    src = open(NF4_SRC).read()
    body = src[src.index("kTheta[3][15] = {"):]
    body = body[:body.index("}};") + 3]
    hexes = re.findall(r"(-?0x[0-9a-f.]+p-?\d+)f", body)
    assert len(hexes) == 45
    vals = [np.float32(float.fromhex(h)) for h in hexes]
    return {"float32": vals[0:15], "float16": vals[15:30], "bfloat16": vals[30:45]}


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_nf4_kernel_thresholds_match_reference_rule(dtype):
    assert _kernel_theta_rows()[dtype] == _oracle_thresholds(dtype)


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_nf4_bucket_table_encoder_equals_argmin(dtype):
    """The kernel's encoder -- bucket b = rint(32 p) + 32 of [-1, 1], code =
    (code at the bucket's left edge) + (p >= threshold inside the bucket) --
    equals the reference argmin of round_dtype(p), on dense samples, every
    bf16 / fp16 value in [-1, 1], the thresholds and their fp32 neighbours."""
    from oracle.lq_oracle import nf4_encode, rnd
    th = np.array(_kernel_theta_rows()[dtype], np.float32)
    left = ((2 * np.arange(65) - 65) / 64).astype(np.float32)
    right = ((2 * np.arange(65) - 63) / 64).astype(np.float32)
    code_lo = (th[None, :] <= left[:, None]).sum(1)
    inside = (th[None, :] > left[:, None]) & (th[None, :] <= right[:, None])
    assert inside.sum(1).max() <= 1
    theta = np.where(inside.any(1), (th[None, :] * inside).sum(1), np.inf).astype(np.float32)
    u = (np.arange(0, 0x10000, dtype=np.uint32) << 16).view(np.float32)
    v16 = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    rng = np.random.default_rng(1)
    p = np.concatenate([u, v16, rng.uniform(-1, 1, 500000).astype(np.float32), th,
                        np.nextafter(th, np.float32(-2)), np.nextafter(th, np.float32(2)),
                        left, right, np.array([-0.0, 0.0, np.nan], np.float32)])
    p = p[np.isnan(p) | (np.abs(p) <= 1)]
    with np.errstate(invalid="ignore"):
        b = (np.rint(p.astype(np.float64) * 32) + 32)
    b = np.where(np.isnan(b), 0, b).astype(np.int64)
    code = code_lo[b] + (p >= theta[b])
    code = np.where(np.isnan(p), 0, code)
    assert np.array_equal(code, nf4_encode(rnd(p, dtype)))


def test_nf4_g64_bucket_table_encoder_equals_argmin():
    """The one-thread-per-group bf16 packing kernel buckets a quotient p by
    k = (bits(fp32(4096 p + 1.5*2^23 + 4608)) & 0x3F80) >> 7, bucket k holding
    p in [(256k - 9217)/8192, (256k - 8961)/8192], and codes it as (code at
    the bucket's left edge) + (p >= threshold inside the bucket).  That equals
    the reference argmin of round_bf16(p) for every bf16 value in [-1, 1],
    dense samples, the thresholds and their fp32 neighbours."""
    from oracle.lq_oracle import nf4_encode, rnd
    th = np.array(_kernel_theta_rows()["bfloat16"], np.float32)
    k = np.arange(128)
    left = ((256 * k - 9217) / 8192).astype(np.float32)
    right = ((256 * k - 8961) / 8192).astype(np.float32)
    code_lo = (th[None, :] <= left[:, None]).sum(1)
    inside = (th[None, :] > left[:, None]) & (th[None, :] <= right[:, None])
    assert inside.sum(1).max() <= 1
    theta = np.where(inside.any(1), (th[None, :] * inside).sum(1), np.inf).astype(np.float32)
    u = (np.arange(0, 0x10000, dtype=np.uint32) << 16).view(np.float32)
    rng = np.random.default_rng(2)
    p = np.concatenate([u, rng.uniform(-1, 1, 500000).astype(np.float32), th,
                        np.nextafter(th, np.float32(-2)), np.nextafter(th, np.float32(2)),
                        left, right, np.nextafter(left, np.float32(2)),
                        np.array([-1.0, 1.0, -0.0, 0.0], np.float32)])
    with np.errstate(invalid="ignore"):
        p = p[np.abs(p) <= 1]
    # 4096 p is exact in fp32, so the float32 add is the kernel's single-rounding FFMA
    f = (p * np.float32(4096)).astype(np.float32) + np.float32(12582912 + 4608)
    b = (f.view(np.uint32) & 0x3F80) >> 7
    assert b.min() >= 4 and b.max() <= 68
    code = code_lo[b] + (p >= theta[b])
    assert np.array_equal(code, nf4_encode(rnd(p, "bfloat16")))


def test_host_rejects_cpu_tensors():
    import llm_quant_b200 as L
    x = torch.randn(4, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        L.fake_quantize(x, 4, False, L.QScheme.PER_GROUP, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        L.nf4_quantize(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        L.PerTokenKVCacheQuantizer(4).quantize(torch.randn(1, 2, 3, 8))


def test_reference_error_types():
    import llm_quant_b200 as L
    with pytest.raises(AssertionError):
        L.hadamard_matrix(3)
    with pytest.raises(AssertionError):
        L.fast_hadamard_transform(torch.randn(2, 12))
    with pytest.raises(ValueError):
        L.compute_qparams(torch.randn(2, 4), scheme="nope")
    with pytest.raises(ValueError):
        L.KVCacheQuantizer(granularity="bad")._compute_qparams(torch.randn(1, 1, 2, 4))


def test_hadamard_matrix_matches_oracle():
    import llm_quant_b200 as L
    from oracle import lq_oracle as O
    from golden_io import same_bits
    for dt, odt in ((torch.float32, "float32"), (torch.bfloat16, "bfloat16"), (torch.float16, "float16")):
        for n in (1, 2, 8, 64, 2048):
            H = L.hadamard_matrix(n, dt).float().numpy()
            assert same_bits(H, O.hadamard_matrix(n, odt)), (dt, n)


def test_kv_memory_ratio_matches_reference_values():
    import llm_quant_b200 as L
    G = L.KVQuantGranularity
    assert L.kv_cache_memory_ratio(4) == 4 / 16 + 32 / (128 * 4)
    assert 0.4 < L.kv_cache_memory_ratio(8, head_dim=128) < 0.6
    assert L.kv_cache_memory_ratio(4, granularity=G.PER_CHANNEL, seq_len=2048) < \
        L.kv_cache_memory_ratio(4, granularity=G.PER_TOKEN)


def test_install_as_llm_quant():
    import sys
    import llm_quant_b200 as L
    saved = {k: v for k, v in sys.modules.items() if k == "llm_quant" or k.startswith("llm_quant.")}
    try:
        L.install_as_llm_quant()
        from llm_quant.core.quantizer import fake_quantize  # noqa: F401
        from llm_quant.qlora import nf4_quantize  # noqa: F401
        import llm_quant
        assert llm_quant.QuantizedKVCache is L.QuantizedKVCache
    finally:
        for k in [k for k in sys.modules if k == "llm_quant" or k.startswith("llm_quant.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_fp16_code_range_overflow_raises_like_reference():
    """The reference's clamp converts qmax to the tensor dtype; for fp16 and
    asymmetric 16-bit codes (qmax = 65535) that conversion raises.  The golden
    fixture records the reference raising; this layer raises the same error
    before any device work."""
    import llm_quant_b200 as L
    from golden_io import cases
    (name, c), = list(cases("quantizer.npz", "wide_raises"))
    assert c["params"]["raised"] is True
    with pytest.raises(RuntimeError, match="c10::Half without overflow"):
        L._C.check_clamp_bounds(torch.float16, 16, False)
    L._C.check_clamp_bounds(torch.float16, 16, True)    # qmax 32767 fits
    L._C.check_clamp_bounds(torch.bfloat16, 16, False)  # 65535 -> 65536 fits in bf16


def test_host_pipeline_arguments_without_gpu():
    """streaming.HostPipeline imports without a GPU and rejects a pipeline with
    no device buffers before touching CUDA."""
    from llm_quant_b200.streaming import HostPipeline
    with pytest.raises(ValueError):
        HostPipeline(device="cuda:0", buffers=0)
