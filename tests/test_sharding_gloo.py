"""Multi-process (world_size 2, gloo on CPU) tests of the layer-sharded driver.

The quantization kernels need a GPU, so here each rank "quantizes" its layers
with the CPU oracle's NF4 restatement (test code only); what is under test
is the host logic: the layer partition, the flat-byte packing and the final
gather to rank 0, plus host-side failure handling (a rank that raises).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_quant_b200.sharded import (PackedLayer, flatten_bytes, gather_to_rank0, layer_block,
                                    quantize_layers, unflatten_bytes)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_layer_block_partition():
    for L in (1, 7, 32):
        for W in (1, 2, 3, 4, 8):
            blocks = [layer_block(L, r, W) for r in range(W)]
            flat = [i for b in blocks for i in b]
            assert flat == list(range(L))
            sizes = [len(b) for b in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        layer_block(4, 2, 2)


def test_flatten_roundtrip():
    ts = [torch.arange(10, dtype=torch.uint8), torch.randn(3, 4).to(torch.bfloat16),
          torch.randn(5)]
    buf = flatten_bytes(ts)
    back = unflatten_bytes(buf, ts)
    for a, b in zip(ts, back):
        assert torch.equal(a.view(torch.uint8) if a.dtype == torch.uint8 else a, b)


def _layer_weight(i):
    g = torch.Generator().manual_seed(100 + i)
    return (torch.randn(8 + i, 64, generator=g) * 0.02).to(torch.bfloat16)


def _oracle_pack(i):
    from oracle import lq_oracle as O
    w = _layer_weight(i).float().numpy()
    codes, scales = O.nf4_quantize(w, "bfloat16", 64)
    c = codes.reshape(-1).astype(np.uint8)
    if c.size % 2:
        c = np.concatenate([c, np.zeros(1, np.uint8)])
    packed = (c[0::2] | (c[1::2] << 4)).astype(np.uint8)
    return PackedLayer(i, {"codes": torch.from_numpy(packed),
                           "scales": torch.from_numpy(scales).to(torch.bfloat16)})


def _worker(rank, world, port, num_layers, fail_rank, q, chunk=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host")
        layers = quantize_layers(num_layers, rank, world, _oracle_pack)
        flat = flatten_bytes([t for pl in layers for t in pl.tensors.values()])
        got = gather_to_rank0(flat) if chunk is None else gather_to_rank0(flat, chunk_bytes=chunk)
        if rank == 0:
            # rebuild every layer from the gathered bytes and compare
            out = []
            for r in range(world):
                like = [t for i in layer_block(num_layers, r, world)
                        for t in _oracle_pack(i).tensors.values()]
                out.extend(unflatten_bytes(got[r], like))
            ref = [t for i in range(num_layers) for t in _oracle_pack(i).tensors.values()]
            ok = all(torch.equal(a, b) for a, b in zip(out, ref)) and len(out) == len(ref)
            q.put(("ok", ok))
    except Exception as e:  # report, then leave cleanly
        q.put(("error", rank, str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, num_layers, fail_rank=-1, chunk=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, num_layers, fail_rank, q, chunk))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not q.empty():
        msgs.append(q.get())
    return msgs, [p.exitcode for p in procs]


def test_gather_world2():
    msgs, codes = _run(2, 5)
    assert ("ok", True) in msgs, msgs
    assert codes == [0, 0]


def test_gather_in_pieces_world3():
    """Each rank's buffer goes in many small pieces (48 bytes), reassembled
    in order on rank 0."""
    msgs, codes = _run(3, 7, chunk=48)
    assert ("ok", True) in msgs, msgs
    assert codes == [0, 0, 0]


def test_rank_failure_is_reported_not_hung():
    msgs, codes = _run(2, 4, fail_rank=1)
    errs = [m for m in msgs if m[0] == "error"]
    assert any(m[1] == 1 and "injected" in m[2] for m in errs)
    # rank 0 leaves with an error from the collective (peer gone / timeout)
    assert all(c == 0 for c in codes)


def test_gather_world3_uneven_exact_sizes():
    """7 layers over 3 ranks (3, 2, 2 layers): every rank's bytes arrive at
    their own size, nothing padded to the largest rank."""
    msgs, codes = _run(3, 7)
    assert ("ok", True) in msgs, msgs
    assert codes == [0, 0, 0]


def _layer_gather_worker(rank, world, port, n_layers, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from llm_quant_b200.sharded import LayerGather, layer_packed_nbytes
        # every rank knows every layer's sizes (the model config)
        sizes = [[t.numel() * t.element_size() for t in _layer_tensors(i)] for i in range(n_layers)]
        lg = LayerGather(layer_packed_nbytes(sizes), rank, world, torch.device("cpu"))
        for i in layer_block(n_layers, rank, world):
            lg.send(i, _layer_tensors(i))
        got = lg.wait()
        if rank == 0:
            ok = sorted(got) == list(range(n_layers))
            for i in range(n_layers):
                back = unflatten_bytes(got[i], _layer_tensors(i))
                ok = ok and all(torch.equal(a.view(torch.uint8), b.view(torch.uint8))
                                for a, b in zip(_layer_tensors(i), back))
            q.put(ok)
    finally:
        dist.destroy_process_group()


def _layer_tensors(i):
    g = torch.Generator().manual_seed(7 + i)
    return [torch.randint(0, 256, (33 + 5 * i,), generator=g, dtype=torch.uint8),
            torch.randn(3 + i, generator=g).to(torch.bfloat16), torch.randn(2, generator=g)]


@pytest.mark.parametrize("world,n_layers", [(2, 5), (3, 7)])
def test_layer_gather_overlapped(world, n_layers):
    """LayerGather: each rank sends its layers as it finishes them, rank 0
    receives every layer at its exact size, matched in layer order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_layer_gather_worker, args=(r, world, port, n_layers, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    assert all(p.exitcode == 0 for p in ps)
    assert q.get(timeout=10) is True
