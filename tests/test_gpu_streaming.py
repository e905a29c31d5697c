"""GPU tests of HostPipeline (llm_quant_b200/streaming.py): host-resident
inputs streamed through the library's ops on three CUDA streams give exactly
the results of the same calls made one after another on one stream."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import llm_quant_b200
    return llm_quant_b200


def test_fake_quantize_stream_matches_direct(L):
    from llm_quant_b200.streaming import HostPipeline
    g = torch.Generator().manual_seed(0)
    hosts = [(torch.randn(512, 1024, generator=g) * 0.02).pin_memory() for _ in range(7)]
    outs = [torch.empty(512, 1024).pin_memory() for _ in range(7)]
    devs = [torch.empty(512, 1024, device="cuda") for _ in range(2)]
    ys = [None, None]
    pipe = HostPipeline(buffers=2)

    def up(i, b):
        devs[b].copy_(hosts[i], non_blocking=True)

    def work(i, b):
        ys[b] = L.fake_quantize(devs[b], 4, False, L.QScheme.PER_GROUP, 128)

    def down(i, b):
        ys[b].record_stream(torch.cuda.current_stream())
        outs[i].copy_(ys[b], non_blocking=True)

    for _ in range(3):  # repeated runs reuse the buffers and the ordering state
        for o in outs:
            o.fill_(float("nan"))
        pipe.run(len(hosts), up, work, down)
        torch.cuda.current_stream().synchronize()
        for h, o in zip(hosts, outs):
            ref = L.fake_quantize(h.cuda(), 4, False, L.QScheme.PER_GROUP, 128).cpu()
            assert torch.equal(o, ref)


def test_nf4_pack_stream_matches_direct(L):
    """QLoRALinear.pack_base + _dequantize_base of host weights through the
    pipeline (the packing kernels are programmatic dependent launches that
    follow a cross-stream wait on the upload): codes, scales and the
    dequantized base equal a direct call on the same weights."""
    from llm_quant_b200.streaming import HostPipeline
    g = torch.Generator().manual_seed(2)
    shapes = [(256, 1024), (1024, 512), (128, 4096), (512, 2048), (256, 1024)]
    hosts = [(torch.randn(o, k, generator=g) * 0.02).to(torch.bfloat16).pin_memory() for o, k in shapes]
    mods = [L.QLoRALinear(k, o, rank=4, group_size=64).cuda() for o, k in shapes]
    devs = [torch.empty(o, k, dtype=torch.bfloat16, device="cuda") for o, k in shapes]

    def res(m):
        return (m.nf4_codes_packed, m.nf4_scales, m.dq_q_scales, m.dq_scales)

    outs = [None] * len(shapes)
    deq = [torch.empty(o, k, dtype=torch.bfloat16).pin_memory() for o, k in shapes]
    last = [None] * len(shapes)
    pipe = HostPipeline(buffers=len(shapes))

    def up(i, b):
        devs[i].copy_(hosts[i], non_blocking=True)

    def work(i, b):
        mods[i].pack_base(devs[i])
        last[i] = mods[i]._dequantize_base()

    def down(i, b):
        cur = torch.cuda.current_stream()
        if outs[i] is None:
            outs[i] = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in res(mods[i])]
        for o, t in zip(outs[i], res(mods[i])):
            t.record_stream(cur)
            o.copy_(t, non_blocking=True)
        last[i].record_stream(cur)
        deq[i].copy_(last[i], non_blocking=True)

    pipe.run(len(shapes), up, work, down)
    torch.cuda.current_stream().synchronize()
    for i, (o, k) in enumerate(shapes):
        ref = L.QLoRALinear(k, o, rank=4, group_size=64).cuda()
        ref.pack_base(hosts[i].cuda())
        for got, want in zip(outs[i], res(ref)):
            assert torch.equal(got, want.cpu())
        assert torch.equal(deq[i], ref._dequantize_base().cpu())


def test_graph_outputs_reused(L):
    """Work that replays a CUDA graph rewrites the same output buffer every
    run: outputs_reused orders it after the previous run's download."""
    from llm_quant_b200.streaming import HostPipeline
    g = torch.Generator().manual_seed(1)
    n = 4
    hosts = [[torch.randn(256, 2048, generator=g).to(torch.bfloat16).pin_memory() for _ in range(n)]
             for _ in range(2)]
    outs = [torch.empty(256, 2048, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    devs = [torch.empty(256, 2048, device="cuda", dtype=torch.bfloat16) for _ in range(n)]
    graphs, ys = [], []
    for d in devs:
        L.hadamard_fake_quantize(d, 4, True)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            ys.append(L.hadamard_fake_quantize(d, 4, True))
        graphs.append(gr)
    pipe = HostPipeline(buffers=n)
    for r in range(2):
        src = hosts[r]
        pipe.run(n, lambda i, b: devs[i].copy_(src[i], non_blocking=True),
                 lambda i, b: graphs[i].replay(),
                 lambda i, b: outs[i].copy_(ys[i], non_blocking=True), outputs_reused=True)
        torch.cuda.current_stream().synchronize()
        for h, o in zip(src, outs):
            assert torch.equal(o, L.hadamard_fake_quantize(h.cuda(), 4, True).cpu())


def test_events_on_calling_stream_bracket_the_run(L):
    """The calling stream waits for all three streams: an event recorded after
    run() completes only once every download has landed."""
    from llm_quant_b200.streaming import HostPipeline
    host = torch.randn(1 << 22).pin_memory()
    out = torch.empty(1 << 22).pin_memory()
    dev = [torch.empty(1 << 22, device="cuda") for _ in range(2)]
    pipe = HostPipeline()
    done = torch.cuda.Event()
    pipe.run(3, lambda i, b: dev[b].copy_(host, non_blocking=True),
             lambda i, b: dev[b].mul_(2.0),
             lambda i, b: out.copy_(dev[b], non_blocking=True))
    done.record()
    done.synchronize()
    assert torch.equal(out, host * 2.0)


def test_buffers_argument_checked():
    from llm_quant_b200.streaming import HostPipeline
    with pytest.raises(ValueError):
        HostPipeline(buffers=0)
