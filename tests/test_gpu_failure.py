"""Failure detection on the GPU without a GPU fault: the bounded device-side
wait that every pipelined kernel (NF4 pack, W4A16, GEMV) uses on its
mbarriers gives up after its limit and reports LQ_ETIMEOUT, and the context
stays usable.  The wait that runs out is on an mbarrier that nothing
arrives on; no copy is in flight, nothing is trapped or faulted."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _probe(limit_ns, arrive):
    from llm_quant_b200 import _C
    out = torch.full((2,), 7, dtype=torch.int64, device="cuda")
    _C.call("lq_wait_probe", limit_ns, arrive, out.data_ptr(), _C.stream_ptr(out))
    torch.cuda.synchronize()
    return int(out[0].item()), int(out[1].item())


def test_wait_gives_up_after_its_limit():
    from llm_quant_b200 import _C
    status, ns = _probe(20_000_000, 0)  # 20 ms, nothing arrives
    assert status == _C.ETIMEOUT
    assert 20_000_000 <= ns < 2_000_000_000


def test_wait_returns_when_the_phase_completes():
    status, ns = _probe(1_000_000_000, 1)
    assert status == 0
    assert ns < 100_000_000


def test_context_usable_after_timeout():
    """A timed-out wait leaves the device working: a quantization kernel
    right after gives the same codes as before the timeout."""
    import llm_quant_b200 as L
    w = torch.randn(64, 256, device="cuda") * 0.02
    before = L.fake_quantize(w, 4, False, L.QScheme.PER_GROUP, 128)
    status, _ = _probe(5_000_000, 0)
    from llm_quant_b200 import _C
    assert status == _C.ETIMEOUT
    after = L.fake_quantize(w, 4, False, L.QScheme.PER_GROUP, 128)
    assert torch.equal(before, after)


def test_probe_rejects_limits_above_ten_seconds():
    from llm_quant_b200 import _C
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        _C.call("lq_wait_probe", 20_000_000_000, 0, out.data_ptr(), _C.stream_ptr(out))
