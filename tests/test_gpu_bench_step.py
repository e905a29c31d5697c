"""The benchmarked step itself, checked: bench.py's default workload (NF4
pack_base + _dequantize_base of Llama-3-8B-shaped weights, seeds 1000 +
layer) captured as the CUDA graph the bench times and replayed once; the
results of layer 0's q and k projections equal the oracle bit for bit."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


class _Ctx:
    def __init__(self):
        self.torch = torch
        self.world, self.rank, self.local = 1, 0, 0
        self.dev = torch.device("cuda", 0)

    def barrier(self):
        pass


def test_bench_default_step_matches_oracle(monkeypatch):
    import bench
    from oracle import lq_oracle as O
    monkeypatch.setattr(bench, "NUM_LAYERS", 1)
    W = bench.NF4Workload(_Ctx())
    assert len(W.weights) == 7
    graph = bench.capture(torch, W.step, 1)
    for m in W.mods:  # clear the eager call's results: the replay must write them
        m.nf4_codes_packed.zero_()
        m.nf4_scales.zero_()
    graph.replay()
    torch.cuda.synchronize()
    # q [4096, 4096] of layer 0 (its first 1024 rows: whole blocks and whole
    # double-quantization groups) and k [1024, 4096]
    for j, rows in ((0, 1024), (1, 1024)):
        w = W.weights[j][:rows].float().cpu().numpy()
        m = W.mods[j]
        n, ng = w.size, w.size // 64
        codes, scales = O.nf4_quantize(w, "bfloat16", 64)
        q, dq = O.double_quantize(scales, "bfloat16", 256)
        assert np.array_equal(m.nf4_codes[:rows].cpu().numpy(), codes)
        assert np.array_equal(m.dq_q_scales[:ng].float().cpu().numpy(), q)
        assert np.array_equal(m.dq_scales[:ng // 256].float().cpu().numpy(), dq)
        ref = O.nf4_dequantize(codes, O.double_dequantize(q, dq, "bfloat16", 256), "bfloat16", 64)
        got = m._dequantize_base()[:rows].float().cpu().numpy().reshape(ref.shape)
        assert np.array_equal(got, ref) and n == ref.size
    del graph
