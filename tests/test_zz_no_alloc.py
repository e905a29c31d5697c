"""GPU test of lq_tensor_qparams_noalloc, the entry point for callers that
cannot allocate device memory (an FFI host handed tensor pointers by another
runtime with no device allocator of its own, or an application whose device
memory is all reserved by a framework allocator).

It is called through the C ABI twice in a row (different sizes, so stale
partials of the first call would show) and must give the same scale and
zero point, bit for bit, as lq_tensor_qparams with a caller-provided
workspace.  This file is collected last so that a failure here does not stop
the other tests when pytest runs with -x.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from llm_quant_b200 import _C
    L = _C.lib()
    V, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    L.lq_tensor_qparams_noalloc.argtypes = [V, I, LL, I, I, V, V, V]
    L.lq_tensor_qparams_noalloc.restype = ctypes.c_int
    return L


def _with_workspace(C, x, bits, sym):
    n = x.numel()
    ws_bytes = C.lib().lq_tensor_qparams_workspace_size(n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    s = torch.empty((), dtype=x.dtype, device=x.device)
    z = torch.empty((1,) if sym else (), dtype=x.dtype, device=x.device)
    C.call("lq_tensor_qparams", x.data_ptr(), C.dt(x), n, bits, int(sym), s.data_ptr(),
           z.data_ptr(), ws.data_ptr(), ws_bytes, C.stream_ptr(x))
    return s, z


def _no_alloc(C, lib, x, bits, sym):
    s = torch.empty((), dtype=x.dtype, device=x.device)
    z = torch.empty((1,) if sym else (), dtype=x.dtype, device=x.device)
    rc = lib.lq_tensor_qparams_noalloc(x.data_ptr(), C.dt(x), x.numel(), bits, int(sym),
                                       s.data_ptr(), z.data_ptr(), C.stream_ptr(x))
    assert rc == 0, lib.lq_last_error()
    return s, z


def _bits(t):
    return t.float().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sym,bits", [(True, 8), (False, 4)])
def test_no_alloc_matches_workspace_version_two_calls(lib, dtype, sym, bits):
    from llm_quant_b200 import _C as C
    g = torch.Generator().manual_seed(11)
    # first call: a large tensor (many partials); second: a small one with a
    # different range, so leftovers of the first call would change the result
    x1 = (torch.randn(3000, 4097, generator=g) * 3.0).to(dtype).cuda()
    x2 = (torch.rand(777, generator=g) + 0.25).to(dtype).cuda()
    for x in (x1, x2):
        s_ref, z_ref = _with_workspace(C, x, bits, sym)
        s, z = _no_alloc(C, lib, x, bits, sym)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(s), _bits(s_ref)), (s, s_ref)
        assert np.array_equal(_bits(z), _bits(z_ref)), (z, z_ref)


def test_no_alloc_rejects_sizes_above_its_maximum(lib):
    from llm_quant_b200 import _C as C
    x = torch.zeros(16, device="cuda")
    s = torch.empty((), device="cuda")
    z = torch.empty(1, device="cuda")
    too_many = 16384 * 4096 + 1
    rc = lib.lq_tensor_qparams_noalloc(x.data_ptr(), C.F32, too_many, 8, 1, s.data_ptr(),
                                       z.data_ptr(), C.stream_ptr(x))
    assert rc == C.ERANGE
    assert b"maximum" in lib.lq_last_error()
