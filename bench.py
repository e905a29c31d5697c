#!/usr/bin/env python
"""Benchmark of the llm_quant quantization hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload nf4|group|rotquant|kv]

N > 1 is launched one process per GPU (torchrun, NCCL); rank 0 prints one
JSON line.  Default workload (``nf4``): whole-model NF4 (block 64, double
quantization over 256 scales) quantize + dequantize of a Llama-3-8B-shaped
weight set, 32 layers x {q, o 4096x4096; k, v 1024x4096; gate, up
14336x4096; down 4096x14336}, bf16 ~ N(0, 0.02), the layers split in
contiguous blocks across the ranks (strong scaling, no data-path
collective; the final NCCL gather of packed codes + scales to rank 0 is
timed separately).  One step = QLoRALinear.pack_base + _dequantize_base on
every weight of the rank's layers.

value     = algorithmic bytes of all ranks per step / max-over-ranks step time
            (CUDA events, inputs resident in HBM; 14 GB of weights > L2).
e2e       = the same bytes / time of the same public-API calls with the
            weights copied from pinned host memory and the packed codes +
            scales copied back, every step.
roofline  = the dominant kernel timed alone with CUDA events on its stream.
cpu_baseline / --impl reference = the CPU oracle's restatement of the
            reference algorithm on a bounded sample, on the host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "group-quant HBM GB/s (% of peak) at 1/2/4/8 GPU; W4A16 dequant-GEMM TFLOP/s"
LLAMA3_8B = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
             ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
NUM_LAYERS = 32

# dram__bytes_read.sum + dram__bytes_write.sum of each workload's dominant
# kernel from one ncu capture of its --profile case (summarised under
# profiles/), per unit the kernel processes (weight / element), so the bench
# scales it to its own launch; the W4A16 figure is per launch (same shape as
# the bench).  Writes still held in L2 when a launch ends are not counted,
# which is why some ratios sit below the algorithmic bytes.
NCU_TRAFFIC = {
    "nf4": 281.4e6 / (28672 * 4096),     # nf4_pack_g64_kernel, 2.40 B per weight
    "group": 215.8e6 / (8192 * 4096),    # group_warp_kernel, 6.43 B per element
    "rotquant": 222.0e6 / (16384 * 4096),  # fht3_kernel, 3.31 B per element
    "kv": 277.2e6 / (8 * 8 * 8192 * 128),  # kv_dequant_seg_kernel, 4.13 B per element
    "w4a16": 44.7e6,                     # w4a16_kernel at M = 1024, bytes per launch
    "qlora_linear": 48.19e6,             # w4a16_kernel<nf4> at M = 1024, bytes per launch
    "kv_attention": 70.5e6 / (8 * 8 * 4096),  # kv_attn_kernel, 269 B per cached token
}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ─────────────────────────────────────────────────────────────────────────────
# process group / timing helpers
# ─────────────────────────────────────────────────────────────────────────────

class Ctx:
    def __init__(self, gpus: int):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.dev = torch.device("cuda", self.local)
        torch.cuda.set_device(self.dev)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled: bool):
        self.proc = None
        self.path = None
        if not enabled:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self, gpus):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx = int(parts[0])
                except ValueError:
                    continue
                if idx not in gpus:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        util = [float(r[4]) if r[4].replace(".", "").isdigit() else 0.0 for r in rows]
        loaded = [r for r, u in zip(rows, util) if u >= 50] or rows
        sm = [float(r[1]) for r in loaded if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in loaded for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(loaded)}


def capture(torch, fn, iters: int = 1):
    """CUDA graph of `iters` back-to-back calls of fn (after one eager call).
    The library's kernels are enqueued on torch's current stream, which is the
    capture stream inside torch.cuda.graph, so they are recorded like any
    other kernel; replays skip all host-side work."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    torch.cuda.synchronize()
    return g


def cuda_time_ms(torch, fn, iters: int, stream=None) -> float:
    """Average device time of one fn() call: `iters` calls captured in a CUDA
    graph, replayed 3 times (after one warm replay), timed with CUDA events on
    the replay stream."""
    g = capture(torch, fn, iters)
    g.replay()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(3):
        g.replay()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (3 * iters)
    del g
    return ms


# ─────────────────────────────────────────────────────────────────────────────
# CPU oracle timing (bounded sample; the oracle is the checker and baseline)
# ─────────────────────────────────────────────────────────────────────────────

def _threads():
    return max(1, os.cpu_count() or 1)


def cpu_time(fn_chunk, chunks, reps=3):
    """Median wall time of running fn_chunk over chunks on all host threads."""
    n = _threads()
    ts = []
    with ThreadPoolExecutor(max_workers=n) as ex:
        list(ex.map(fn_chunk, chunks[:1]))  # warm-up
        for _ in range(reps):
            t0 = time.perf_counter()
            list(ex.map(fn_chunk, chunks))
            ts.append(time.perf_counter() - t0)
    return statistics.median(ts), n


REF_INSTALL = os.path.join(ROOT, "baseline", "_ref")


def reference_package():
    """The reference package itself (its torch CPU code), from the installed
    copy in baseline/_ref (written by oracle/install_ref.py; not part of the
    product), or None with the reason when it is absent."""
    if not os.path.exists(os.path.join(REF_INSTALL, "llm_quant", "qlora.py")):
        return None, "the reference is not installed (python oracle/install_ref.py)"
    if REF_INSTALL not in sys.path:
        sys.path.insert(0, REF_INSTALL)
    import importlib
    mod = importlib.import_module("llm_quant")
    if not os.path.abspath(mod.__file__).startswith(REF_INSTALL):
        return None, f"llm_quant resolves to {mod.__file__}, not the installed reference"
    return mod, None


def reference_torch_leg(fn, nbytes, sample, reps=3):
    """Median wall time of the reference's own torch CPU call fn() (after one
    warm-up) with torch's intra-op threads on every host core."""
    import torch
    threads = torch.get_num_threads()
    torch.set_num_threads(_threads())
    try:
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(threads)
    t = statistics.median(ts)
    return {"value": nbytes / t / 1e9, "unit": "GB/s", "cores": _threads(),
            "kind": "reference_torch", "sample": f"{sample}, median of {reps}"}


# ─────────────────────────────────────────────────────────────────────────────
# workloads
# ─────────────────────────────────────────────────────────────────────────────

class NF4Workload:
    name = "nf4"
    workload = "qlora_nf4_llama3_8b_32layers_bf16_block64_dq256"

    def __init__(self, ctx):
        self.ctx = ctx
        torch = ctx.torch
        import llm_quant_b200 as L
        from llm_quant_b200.sharded import layer_block
        self.L = L
        self.layers = list(layer_block(NUM_LAYERS, ctx.rank, ctx.world))
        self.weights, self.mods = [], []
        for li in self.layers:
            g = torch.Generator(device=ctx.dev).manual_seed(1000 + li)
            for _, o, k in LLAMA3_8B:
                w = (torch.randn(o, k, generator=g, device=ctx.dev) * 0.02).to(torch.bfloat16)
                self.weights.append(w)
                self.mods.append(L.QLoRALinear(k, o, rank=16, group_size=64).to(ctx.dev))
        self.n_local = sum(w.numel() for w in self.weights)
        self.n_total = NUM_LAYERS * sum(o * k for _, o, k in LLAMA3_8B)

    @staticmethod
    def bytes_for(n: int) -> float:
        """Algorithmic bytes of pack (read bf16, write packed codes, block
        scales, q_scales, dq_scales) + unpack (read codes, q_scales, dq_scales;
        write bf16) for n weights."""
        ng = n / 64
        nd = ng / 256
        pack = 2 * n + n / 2 + 2 * ng + 2 * ng + 2 * nd
        unpack = n / 2 + 2 * ng + 2 * nd + 2 * n
        return pack + unpack

    def step(self):
        for m, w in zip(self.mods, self.weights):
            m.pack_base(w)
            m._dequantize_base()

    def launches_per_step(self):
        return 2 * len(self.weights)

    def kernels(self):
        """Time pack and unpack alone on weights of the largest shape of the
        rank, cycling through up to 4 of them (470 MB of bf16, more than L2)."""
        torch = self.ctx.torch
        n = max(w.numel() for w in self.weights)
        idx = [j for j, w in enumerate(self.weights) if w.numel() == n][:4]
        ng, nd = n / 64, n / 64 / 256
        c = [0, 0]

        def pack():
            j = idx[c[0] % len(idx)]
            self.mods[j].pack_base(self.weights[j])
            c[0] += 1

        def unpack():
            self.mods[idx[c[1] % len(idx)]]._dequantize_base()
            c[1] += 1
        for j in idx:
            self.mods[j].pack_base(self.weights[j])
        t_pack = cuda_time_ms(torch, pack, 8 * len(idx))
        t_unpack = cuda_time_ms(torch, unpack, 8 * len(idx))
        b_pack = 2 * n + n / 2 + 4 * ng + 2 * nd
        b_unpack = n / 2 + 2 * ng + 2 * nd + 2 * n
        return {
            "nf4_pack_g64_kernel (pack_base)": (b_pack, t_pack, n, "weights"),
            "nf4_unpack_vec_kernel (_dequantize_base)": (b_unpack, t_unpack, n, "weights"),
        }

    def api_int64_kernels(self):
        """nf4_quantize + nf4_dequantize through the functional API with int64
        codes (qlora.py:66-157), on the largest weights of the rank (each
        117 MB of bf16 and 470 MB of codes, more than L2): 2 + 8 + 8 + 2 +
        2 x 2/64 = 20.06 algorithmic bytes per weight."""
        torch = self.ctx.torch
        n = max(w.numel() for w in self.weights)
        idx = [j for j, w in enumerate(self.weights) if w.numel() == n][:2]
        c = [0]

        def f():
            w = self.weights[idx[c[0] % len(idx)]]
            codes, s = self.L.nf4_quantize(w, 64)
            self.L.nf4_dequantize(codes, s, 64, tuple(w.shape))
            c[0] += 1
        t = cuda_time_ms(torch, f, 2 * len(idx))
        b = (2 + 8 + 8 + 2) * n + 2 * 2 * (n / 64)
        return {"nf4_quant_kernel + nf4_dequant (API int64 codes)": (b, t, n, "weights")}

    def e2e(self, steps, graph):
        """The step's public-API calls (pack_base / _dequantize_base) with every
        weight copied in from pinned host memory and the packed codes + scales
        copied back to pinned host memory, every step, through HostPipeline:
        the upload of weight i+1 and the download of weight i-1's results
        overlap weight i's kernels.  One layer's seven host weights are reused
        as the source of every layer."""
        torch = self.ctx.torch
        from llm_quant_b200.streaming import HostPipeline
        host_in = [torch.empty(w.shape, dtype=w.dtype).pin_memory() for w in self.weights[:7]]
        for h, w in zip(host_in, self.weights[:7]):
            h.copy_(w.cpu())

        def results(m):
            return (m.nf4_codes_packed, m.nf4_scales, m.dq_q_scales, m.dq_scales)
        outs = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in results(m)] for m in self.mods]
        h2d = sum(w.numel() * w.element_size() for w in self.weights)
        d2h = sum(o.numel() * o.element_size() for os_ in outs for o in os_)
        n = len(self.weights)
        pipe = HostPipeline(self.ctx.dev, buffers=n)  # every weight has its own device buffer

        def up(i, _):
            self.weights[i].copy_(host_in[i % 7], non_blocking=True)

        def work(i, _):
            self.mods[i].pack_base(self.weights[i])
            self.mods[i]._dequantize_base()

        def down(i, _):
            cur = torch.cuda.current_stream()
            for o, t in zip(outs[i], results(self.mods[i])):
                t.record_stream(cur)
                o.copy_(t, non_blocking=True)

        def one_step():
            pipe.run(n, up, work, down)

        one_step()
        torch.cuda.synchronize()
        self.ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one_step()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps, h2d, d2h

    def gather(self):
        """Final gather of every rank's packed codes + scales to rank 0."""
        torch = self.ctx.torch
        if self.ctx.world == 1:
            return 0.0, 0
        from llm_quant_b200.sharded import flatten_bytes, gather_to_rank0
        flat = flatten_bytes([t for m in self.mods for t in
                              (m.nf4_codes_packed, m.nf4_scales, m.dq_q_scales, m.dq_scales)])
        # NCCL sets up the gather's peer connections on first use: warm them up
        gather_to_rank0(torch.zeros(1 << 20, dtype=torch.uint8, device=flat.device))
        torch.cuda.synchronize()
        self.ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        got = gather_to_rank0(flat)
        e1.record()
        torch.cuda.synchronize()
        # bytes that crossed NVLink into rank 0 (its own buffer stays put)
        received = sum(b.numel() for b in got[1:]) if got is not None else 0
        return e0.elapsed_time(e1), received

    def job_overlapped(self):
        """The whole-model job with its gather overlapped: every rank packs
        its layers eagerly and sends each layer's results to rank 0 as soon
        as its kernels are enqueued (sharded.LayerGather), rank 0 having
        posted all receives up front; timed with CUDA events on each rank's
        stream from a barrier to the completion of every transfer."""
        torch = self.ctx.torch
        if self.ctx.world == 1:
            return None
        from llm_quant_b200.sharded import LayerGather, layer_packed_nbytes
        per_layer = len(LLAMA3_8B)

        def results(m):
            return (m.nf4_codes_packed, m.nf4_scales, m.dq_q_scales, m.dq_scales)
        one = [t.numel() * t.element_size() for m in self.mods[:per_layer] for t in results(m)]
        nbytes = layer_packed_nbytes([one] * NUM_LAYERS)

        def job():
            lg = LayerGather(nbytes, self.ctx.rank, self.ctx.world, self.ctx.dev)
            for j, li in enumerate(self.layers):
                mods = self.mods[j * per_layer:(j + 1) * per_layer]
                for m, w in zip(mods, self.weights[j * per_layer:(j + 1) * per_layer]):
                    m.pack_base(w)
                    m._dequantize_base()
                lg.send(li, [t for m in mods for t in results(m)])
            return lg.wait()
        job()  # connections and allocator warm
        torch.cuda.synchronize()
        self.ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        got = job()
        e1.record()
        torch.cuda.synchronize()
        if self.ctx.rank == 0:
            assert len(got) == NUM_LAYERS
        return e0.elapsed_time(e1)

    @staticmethod
    def cpu_baseline():
        """Oracle NF4 pack (quant + double quant) + dequant of 2 M weights
        (rows of the 4096-wide q projection of layer 0), on all host cores."""
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        w = O.rnd((rng.standard_normal((512, 4096)) * 0.02).astype(np.float32), "bfloat16")
        chunks = [w[i:i + 16] for i in range(0, 512, 16)]  # 64 Ki weights = 4 dq groups each

        def run(c):
            codes, s = O.nf4_quantize(c, "bfloat16", 64)
            q, dq = O.double_quantize(s, "bfloat16", 256)
            O.nf4_dequantize(codes, O.double_dequantize(q, dq, "bfloat16", 256), "bfloat16", 64)

        t, n = cpu_time(run, chunks)
        b = NF4Workload.bytes_for(w.size)
        out = {"value": b / t / 1e9, "unit": "GB/s", "cores": n, "kind": "port",
               "sample": f"oracle NF4 pack+dequant of {w.size} bf16 weights ({len(chunks)} chunks "
                         f"on {n} threads), median of 3"}
        out["reference_torch"] = NF4Workload.reference_torch(w)
        return out

    @staticmethod
    def reference_torch(w):
        """The reference's own torch CPU path on the same sample:
        nf4_quantize + double_quantize + double_dequantize + nf4_dequantize
        (qlora.py:66-223), the calls pack_base / _dequantize_base make."""
        ref, why = reference_package()
        if ref is None:
            return {"unavailable": why}
        import torch
        from llm_quant import qlora as RQ
        x = torch.from_numpy(np.array(w, np.float32)).to(torch.bfloat16)

        def run():
            codes, s = RQ.nf4_quantize(x, 64)
            q, dq = RQ.double_quantize(s, 256)
            RQ.nf4_dequantize(codes, RQ.double_dequantize(q, dq, 256), 64, tuple(x.shape))
        return reference_torch_leg(run, NF4Workload.bytes_for(x.numel()),
                                   f"reference torch NF4 pack+dequant of {x.numel()} bf16 weights "
                                   "(packed-path bytes)")


class GroupWorkload:
    """fake_quantize INT4 asym group 128 of fp32 [4096, 4096] weights (weak
    scaling: each rank quantizes its own batch of 8 matrices per step)."""
    name = "group"
    workload = "fake_quantize_int4_asym_g128_fp32_4096x4096_x8_per_gpu"

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        self.ctx, self.L = ctx, L
        g = torch.Generator(device=ctx.dev).manual_seed(ctx.rank)
        self.ws = [torch.randn(4096, 4096, generator=g, device=ctx.dev) * 0.02 for _ in range(8)]
        self.n_local = sum(w.numel() for w in self.ws)
        self.n_total = self.n_local * ctx.world

    @staticmethod
    def bytes_for(n):
        return 8.0 * n

    def step(self):
        for w in self.ws:
            self.L.fake_quantize(w, 4, False, self.L.QScheme.PER_GROUP, 128)

    def launches_per_step(self):
        return len(self.ws)

    def kernels(self):
        """fake_quantize timed alone, cycling through the 8 matrices (512 MB of
        input, more than L2)."""
        c = [0]

        def f():
            self.L.fake_quantize(self.ws[c[0] % len(self.ws)], 4, False, self.L.QScheme.PER_GROUP, 128)
            c[0] += 1
        t = cuda_time_ms(self.ctx.torch, f, 48)
        n = self.ws[0].numel()
        return {"group_warp_kernel (fake_quantize)": (8.0 * n, t, n, "elements")}

    def e2e(self, steps, graph):
        """fake_quantize through the public API on matrices copied in from
        pinned host memory, results copied back, every step (HostPipeline:
        uploads, kernels and downloads of consecutive matrices overlap)."""
        torch = self.ctx.torch
        from llm_quant_b200.streaming import HostPipeline
        host = torch.empty(4096, 4096).pin_memory()
        host.copy_(self.ws[0].cpu())
        out = torch.empty(4096, 4096).pin_memory()
        devs = [torch.empty_like(self.ws[0]) for _ in range(2)]
        ys = [None, None]
        pipe = HostPipeline(self.ctx.dev, buffers=2)

        def up(i, b):
            devs[b].copy_(host, non_blocking=True)

        def work(i, b):
            ys[b] = self.L.fake_quantize(devs[b], 4, False, self.L.QScheme.PER_GROUP, 128)

        def down(i, b):
            ys[b].record_stream(torch.cuda.current_stream())
            out.copy_(ys[b], non_blocking=True)

        def one():
            pipe.run(len(self.ws), up, work, down)

        one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one()
        e1.record()
        torch.cuda.synchronize()
        nb = host.numel() * 4 * len(self.ws)
        return e0.elapsed_time(e1) / steps, nb, nb

    def gather(self):
        return 0.0, 0

    @staticmethod
    def cpu_baseline():
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        w = (rng.standard_normal((1024, 4096)) * 0.02).astype(np.float32)
        chunks = [w[i:i + 32] for i in range(0, 1024, 32)]
        t, n = cpu_time(lambda c: O.fake_quantize(c, "float32", 4, False, "per_group", 128), chunks)
        out = {"value": 8.0 * w.size / t / 1e9, "unit": "GB/s", "cores": n, "kind": "port",
               "sample": f"oracle fake_quantize of fp32 [1024, 4096] ({len(chunks)} chunks on "
                         f"{n} threads), median of 3"}
        ref, why = reference_package()
        if ref is None:
            out["reference_torch"] = {"unavailable": why}
        else:
            import torch
            from llm_quant.core import quantizer as RQ
            x = torch.from_numpy(w)
            out["reference_torch"] = reference_torch_leg(
                lambda: RQ.fake_quantize(x, 4, False, RQ.QScheme.PER_GROUP, 128), 8.0 * w.size,
                "reference torch fake_quantize of fp32 [1024, 4096]")
        return out


class RotQuantWorkload:
    """QuaRot activation path: Hadamard (d = 4096) + per-token INT4 sym fake
    quant of bf16 [8192, 4096] activations with 1% outlier channels x50,
    fused in one kernel; a step processes 4 distinct batches (512 MB in and
    out, more than L2; weak scaling: each rank its own activations)."""
    name = "rotquant"
    workload = "quarot_fht4096_pertoken_int4_bf16_8192x4096_x4"

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        self.ctx, self.L = ctx, L
        g = torch.Generator(device=ctx.dev).manual_seed(ctx.rank)
        self.xs = []
        for _ in range(4):
            a = torch.randn(8192, 4096, generator=g, device=ctx.dev)
            idx = torch.randperm(4096, generator=g, device=ctx.dev)[:41]
            a[:, idx] *= 50
            self.xs.append(a.to(torch.bfloat16))
        self.n_local = sum(a.numel() for a in self.xs)
        self.n_total = self.n_local * ctx.world

    @staticmethod
    def bytes_for(n):
        return 4.0 * n

    def step(self):
        for a in self.xs:
            self.L.hadamard_fake_quantize(a, 4, True)

    def launches_per_step(self):
        return len(self.xs)

    def kernels(self):
        c = [0]

        def f():
            self.L.hadamard_fake_quantize(self.xs[c[0] % 4], 4, True)
            c[0] += 1
        t = cuda_time_ms(self.ctx.torch, f, 40)
        n = self.xs[0].numel()
        return {"fht3_kernel (hadamard_fake_quantize)": (4.0 * n, t, n, "elements")}

    def e2e(self, steps, graph):
        """hadamard_fake_quantize through the public API on batches copied in
        from pinned host memory, results copied back, every step
        (HostPipeline)."""
        torch = self.ctx.torch
        from llm_quant_b200.streaming import HostPipeline
        host = torch.empty(8192, 4096, dtype=torch.bfloat16).pin_memory()
        host.copy_(self.xs[0].cpu())
        out = torch.empty_like(host).pin_memory()
        devs = [torch.empty_like(self.xs[0]) for _ in range(2)]
        ys = [None, None]
        pipe = HostPipeline(self.ctx.dev, buffers=2)

        def up(i, b):
            devs[b].copy_(host, non_blocking=True)

        def work(i, b):
            ys[b] = self.L.hadamard_fake_quantize(devs[b], 4, True)

        def down(i, b):
            ys[b].record_stream(torch.cuda.current_stream())
            out.copy_(ys[b], non_blocking=True)

        def one():
            pipe.run(len(self.xs), up, work, down)

        one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one()
        e1.record()
        torch.cuda.synchronize()
        nb = host.numel() * 2 * len(self.xs)
        return e0.elapsed_time(e1) / steps, nb, nb

    def gather(self):
        return 0.0, 0

    @staticmethod
    def cpu_baseline():
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        a = O.rnd(rng.standard_normal((256, 4096)).astype(np.float32), "bfloat16")
        chunks = [a[i:i + 8] for i in range(0, 256, 8)]

        def run(c):
            h = O.fast_hadamard_transform(c, "bfloat16")
            O.fake_quantize(h, "bfloat16", 4, True, "per_channel")

        t, n = cpu_time(run, chunks)
        return {"value": 4.0 * a.size / t / 1e9, "unit": "GB/s", "cores": n, "kind": "port",
                "sample": f"oracle Hadamard + per-token INT4 of bf16 [256, 4096] ({n} threads), "
                          "median of 3"}


class KVWorkload:
    """KV-cache quantization: 32 layers x K, V bf16 [16, 8, 8192, 128], K
    per-channel INT8, V per-token INT4, 16 QuantizedKVCache.update calls of
    512 tokens per layer, each returning the full fp32 K and V (the
    reference's contract); layers split across ranks (strong scaling)."""
    name = "kv"
    workload = "kv_cache_32layers_bf16_16x8x8192x128_K_perchan_int8_V_pertoken_int4_16x512"
    B, H, D, C, U = 16, 8, 128, 512, 16

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        from llm_quant_b200.sharded import layer_block
        self.ctx, self.L = ctx, L
        self.layers = list(layer_block(NUM_LAYERS, ctx.rank, ctx.world))
        # inputs of one layer (16 chunks of K and V) are generated once and
        # reused by every layer of the rank: 2 x 256 MB
        g = torch.Generator(device=ctx.dev).manual_seed(ctx.rank)
        self.k = []
        self.v = []
        for _ in range(self.U):
            k = torch.randn(self.B, self.H, self.C, self.D, generator=g, device=ctx.dev)
            k[..., :4] *= 20
            self.k.append(k.to(torch.bfloat16))
            self.v.append(torch.randn(self.B, self.H, self.C, self.D, generator=g,
                                      device=ctx.dev).to(torch.bfloat16))
        E = self.B * self.H * self.C * self.D * self.U  # elements of one tensor of one layer
        self.E = E
        self.n_local = len(self.layers)
        self.n_total = NUM_LAYERS

    def bytes_per_layer(self):
        c = self.E // self.U
        # per tensor: 16 x (read 2c + write 1c codes) + sum_i (read i*c codes + write 4*i*c)
        return 2 * (self.U * 3 * c + sum(i * c + 4 * i * c for i in range(1, self.U + 1)))

    def bytes_for(self, n_layers):
        return self.bytes_per_layer() * n_layers

    def _layer(self):
        L = self.L
        cache = L.QuantizedKVCache(1, L.PerChannelKVCacheQuantizer(8),
                                   value_quantizer=L.PerTokenKVCacheQuantizer(4),
                                   max_seq_len=self.C * self.U)
        for j in range(self.U):
            cache.update(0, self.k[j], self.v[j])

    def step(self):
        for _ in self.layers:
            self._layer()

    def launches_per_step(self):
        return len(self.layers) * self.U * 4

    def kernels(self):
        torch = self.ctx.torch
        L = self.L
        cache = L.QuantizedKVCache(1, L.PerChannelKVCacheQuantizer(8),
                                   value_quantizer=L.PerTokenKVCacheQuantizer(4),
                                   max_seq_len=self.C * self.U)
        for j in range(self.U):
            cache.update(0, self.k[j], self.v[j])
        side = cache._sides[0][0]
        t = cuda_time_ms(torch, side.dequantize, 10)
        n = side.T * self.B * self.H * self.D
        return {"kv_dequant_seg_kernel (full-cache fp32 read-out)": (5.0 * n, t, n, "elements")}

    def e2e(self, steps, graph):
        """Every layer's 16 update() calls through the public API with the new
        K, V chunks copied in from pinned host memory and the layer's final
        fp32 K, V copied back, every step; HostPipeline overlaps the chunk
        uploads, the kernels and the layer downloads."""
        torch = self.ctx.torch
        from llm_quant_b200.streaming import HostPipeline
        L = self.L
        hk = [k.cpu().pin_memory() for k in self.k]
        hv = [v.cpu().pin_memory() for v in self.v]
        dks = [torch.empty_like(self.k[0]) for _ in range(2)]
        dvs = [torch.empty_like(self.v[0]) for _ in range(2)]
        outk = torch.empty(self.B, self.H, self.C * self.U, self.D).pin_memory()
        outv = torch.empty_like(outk).pin_memory()
        st = {}
        pipe = HostPipeline(self.ctx.dev, buffers=2)

        def up(i, b):
            j = i % self.U
            dks[b].copy_(hk[j], non_blocking=True)
            dvs[b].copy_(hv[j], non_blocking=True)

        def work(i, b):
            if i % self.U == 0:
                st["cache"] = L.QuantizedKVCache(1, L.PerChannelKVCacheQuantizer(8),
                                                 value_quantizer=L.PerTokenKVCacheQuantizer(4),
                                                 max_seq_len=self.C * self.U)
            st["out"] = st["cache"].update(0, dks[b], dvs[b])

        def down(i, b):
            if i % self.U == self.U - 1:  # the layer's full cache after its last update
                cur = torch.cuda.current_stream()
                for o, t in zip((outk, outv), st["out"]):
                    t.record_stream(cur)
                    o.copy_(t, non_blocking=True)

        def one():
            pipe.run(len(self.layers) * self.U, up, work, down)

        one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one()
        e1.record()
        torch.cuda.synchronize()
        h2d = len(self.layers) * 2 * self.E * 2
        d2h = len(self.layers) * 2 * self.E * 4
        return e0.elapsed_time(e1) / steps, h2d, d2h

    def gather(self):
        return 0.0, 0

    @staticmethod
    def cpu_baseline():
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        kq = dict(n_bits=8, symmetric=True, granularity="per_channel")
        vq = dict(n_bits=4, symmetric=True, granularity="per_token")
        chunks = []
        for b in range(8):  # 8 (batch*head) slices x 16 updates of 512 tokens
            ks = [O.rnd(rng.standard_normal((1, 1, 512, 128)).astype(np.float32), "bfloat16")
                  for _ in range(16)]
            vs = [O.rnd(rng.standard_normal((1, 1, 512, 128)).astype(np.float32), "bfloat16")
                  for _ in range(16)]
            chunks.append((ks, vs))

        def run(c):
            cache = O.QuantizedKVCacheOracle(1, "bfloat16", kq, vq)
            for k, v in zip(*c):
                cache.update(0, k, v)

        t, n = cpu_time(run, chunks)
        c = 512 * 128 * 8
        b = 2 * (16 * 3 * c + sum(i * c + 4 * i * c for i in range(1, 17)))
        return {"value": b / t / 1e9, "unit": "GB/s", "cores": n, "kind": "port",
                "sample": f"oracle QuantizedKVCache, 8 (batch, head) slices x 16 updates of 512 "
                          f"tokens, head_dim 128 ({n} threads), median of 3"}


class W4A16Workload:
    """QuantizedLinear W4A16 forward: Linear(4096, 14336), int4 asym group 128
    with fp16 scales / zeros, fp16 activations ~ N(0, 1).  Six such layers
    with distinct weights (6 x 29 MB packed, more than L2, like consecutive
    layers of a model); a step is the forward of all six at M = 1024 tokens
    (the headline point); every M in {1, 16, 128, 1024, 4096} is timed in
    `kernels`, cycling through the layers.  Weak scaling (replicas)."""
    name = "w4a16"
    workload = "quantized_linear_w4a16_K4096_N14336_g128_fp16_M1024_x6_layers"
    main_kernel = "w4a16_kernel"
    Ms = (1, 16, 128, 1024, 4096)
    K, N = 4096, 14336
    LAYERS = 6

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        self.ctx, self.L = ctx, L
        g = torch.Generator(device=ctx.dev).manual_seed(0)
        self.qls = []
        for _ in range(self.LAYERS):
            lin = torch.nn.Linear(self.K, self.N, device=ctx.dev)
            with torch.no_grad():
                lin.weight.copy_(torch.randn(self.N, self.K, generator=g, device=ctx.dev) * 0.02)
            self.qls.append(L.QuantizedLinear.from_linear(lin.half(), 4, False, 128))
            del lin
        self.ql = self.qls[0]
        self.x = {m: torch.randn(m, self.K, generator=g, device=ctx.dev).half() for m in self.Ms}
        for ql in self.qls:
            ql(self.x[1])  # builds the packed operand
        self.n_local = self.LAYERS
        self.n_total = self.LAYERS * ctx.world
        self.unit = "TFLOP/s"

    def flops(self, m):
        return 2.0 * m * self.K * self.N

    def bytes_for(self, n):  # FLOPs: this workload's metric is TFLOP/s
        return self.flops(1024) * n

    def step(self):
        for ql in self.qls:
            ql(self.x[1024])

    def launches_per_step(self):
        return self.LAYERS

    def kernels(self):
        out = {}
        for m in self.Ms:
            x = self.x[m]
            c = [0]

            def f():
                self.qls[c[0] % self.LAYERS](x)
                c[0] += 1
            t = cuda_time_ms(self.ctx.torch, f, 4 * self.LAYERS)
            wbytes = self.N * self.K / 2 + self.N * (self.K // 128) * 4
            kname = "w4a16_gemv_kernel" if m <= 8 else "w4a16_kernel"
            out[f"{kname} M={m}"] = (self.flops(m), t, m, wbytes + 2 * m * self.K + 2 * m * self.N)
        return out

    def e2e(self, steps, graph):
        """Forward through the public API (each layer captured in a CUDA
        graph) with x copied in from pinned host memory and y copied back,
        every step; HostPipeline overlaps layer l+1's upload and layer l-1's
        download with layer l's forward."""
        torch = self.ctx.torch
        from llm_quant_b200.streaming import HostPipeline
        host = self.x[1024].cpu().pin_memory()
        out = torch.empty(1024, self.N, dtype=self.x[1024].dtype).pin_memory()
        devs = [torch.empty_like(self.x[1024]) for _ in self.qls]
        torch.cuda.synchronize()
        graphs, ys = [], []
        for ql, dev in zip(self.qls, devs):
            dev.copy_(self.x[1024])
            ql(dev)
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2):
                ys.append(ql(dev))
            graphs.append(g2)
        pipe = HostPipeline(self.ctx.dev, buffers=len(self.qls))  # a graph's input is its own buffer

        def up(i, b):
            devs[i].copy_(host, non_blocking=True)

        def work(i, b):
            graphs[i].replay()

        def down(i, b):
            out.copy_(ys[i], non_blocking=True)

        def one():
            pipe.run(len(self.qls), up, work, down, outputs_reused=True)

        one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one()
        e1.record()
        torch.cuda.synchronize()
        return (e0.elapsed_time(e1) / steps, host.numel() * 2 * self.LAYERS,
                out.numel() * 2 * self.LAYERS)

    def gather(self):
        return 0.0, 0

    @staticmethod
    def cpu_baseline():
        """Oracle QuantizedLinear forward: exact fp32 dequantized weight (the
        reference's w_float) times x in fp32 (numpy BLAS), M = 64 tokens."""
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        K, N, M = 4096, 14336, 64
        w = O.rnd((rng.standard_normal((N, K)) * 0.02).astype(np.float32), "float16")
        wi, s, z = O.quantized_linear_quantize_weights(w, "float16", 4, False, 128)
        x = O.rnd(rng.standard_normal((M, K)).astype(np.float32), "float16")
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            wf = O.quantized_linear_dequant_weight(wi, s, "float16", z, "float16", 128, K)
            _ = x @ wf.T
            ts.append(time.perf_counter() - t0)
        t = statistics.median(ts)
        return {"value": 2.0 * M * K * N / t / 1e12, "unit": "TFLOP/s",
                "cores": _threads(), "kind": "port",
                "sample": f"oracle dequant + numpy fp32 matmul, M={M}, K={K}, N={N}, median of 3"}


class QLoRALinearWorkload(W4A16Workload):
    """QLoRALinear forward with a bf16 NF4 base (block 64, double quant) of
    Linear(4096, 14336) shape, rank-16 LoRA, bf16 activations: the fused NF4
    base product (lq_nf4_linear) plus the LoRA path.  Six layers with distinct
    weights; a step is the forward of all six at M = 1024 tokens, and FLOPs
    count the base product only (the rank-16 LoRA path adds 0.8 % more work
    inside the timed region).  `kernels` times the fused base product alone at
    every M.  Weak scaling (replicas)."""
    name = "qlora_linear"
    workload = "qlora_linear_nf4_bf16_K4096_N14336_block64_dq256_M1024_x6_layers"
    main_kernel = "w4a16_kernel<nf4>"

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        from llm_quant_b200 import nf4_linear
        self.ctx, self.L, self.nl = ctx, L, nf4_linear
        g = torch.Generator(device=ctx.dev).manual_seed(0)
        self.qls = []
        for _ in range(self.LAYERS):
            w = (torch.randn(self.N, self.K, generator=g, device=ctx.dev) * 0.02).to(torch.bfloat16)
            ql = L.QLoRALinear(self.K, self.N, rank=16, group_size=64).to(ctx.dev)
            with torch.no_grad():
                ql.lora_B.normal_(0, 0.02, generator=g)
            ql.pack_base(w)
            ql.requires_grad_(False)
            self.qls.append(ql)
        self.ql = self.qls[0]
        self.x = {m: torch.randn(m, self.K, generator=g, device=ctx.dev).to(torch.bfloat16)
                  for m in self.Ms}
        for ql in self.qls:
            ql(self.x[1])  # builds the kernel operand
        self.n_local = self.LAYERS
        self.n_total = self.LAYERS * ctx.world
        self.unit = "TFLOP/s"

    def kernels(self):
        out = {}
        for m in self.Ms:
            x = self.x[m]
            c = [0]

            def f():
                self.nl.base_linear(self.qls[c[0] % self.LAYERS], x)
                c[0] += 1
            t = cuda_time_ms(self.ctx.torch, f, 4 * self.LAYERS)
            wbytes = self.N * self.K / 2 + self.N * (self.K // 64) * 4
            kname = "w4a16_gemv_kernel<nf4>" if m <= 8 else "w4a16_kernel<nf4>"
            out[f"{kname} M={m}"] = (self.flops(m), t, m, wbytes + 2 * m * self.K + 2 * m * self.N)
        return out

    @staticmethod
    def cpu_baseline():
        """Oracle QLoRALinear base product: NF4 dequant (double quant) of the
        bf16 base, then x @ W^T in fp32 (numpy BLAS), M = 64 tokens."""
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        K, N, M = 4096, 14336, 64
        w = O.rnd((rng.standard_normal((N, K)) * 0.02).astype(np.float32), "bfloat16")
        codes, sc = O.nf4_quantize(w, "bfloat16", 64)
        q, dq = O.double_quantize(sc, "bfloat16", 256)
        x = O.rnd(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            wf = O.nf4_dequantize(codes, O.double_dequantize(q, dq, "bfloat16", 256), "bfloat16", 64)
            _ = x @ wf.reshape(N, K).T
            ts.append(time.perf_counter() - t0)
        t = statistics.median(ts)
        return {"value": 2.0 * M * K * N / t / 1e12, "unit": "TFLOP/s",
                "cores": _threads(), "kind": "port",
                "sample": f"oracle NF4 dequant + numpy fp32 matmul, M={M}, K={K}, N={N}, median of 3"}


class KVAttentionWorkload:
    """Decode attention over the quantized KV cache (QuantizedKVCache.attend):
    4 layers, each a cache of B=8 x 8 kv heads x 8192 tokens x head_dim 128
    quantized per token to symmetric INT8 (the cache's default quantizer) from
    fp16; 32 query heads (4 per kv head), one query token.  A step attends all
    4 layers (4 x 138 MB of codes and scales: more than L2, each layer read
    from HBM).  Independent replicas per GPU (weak scaling)."""
    name = "kv_attention"
    workload = "kv_decode_attention_int8_pertoken_B8_Hkv8_Hq32_T8192_D128_fp16_x4layers"
    main_kernel = "kv_attn_kernel"
    B, H, HQ, T, D, LAYERS = 8, 8, 32, 8192, 128, 4

    def __init__(self, ctx):
        torch = ctx.torch
        import llm_quant_b200 as L
        self.ctx, self.L = ctx, L
        g = torch.Generator(device=ctx.dev).manual_seed(ctx.rank)
        self.cache = L.QuantizedKVCache(self.LAYERS, max_seq_len=self.T)
        for layer in range(self.LAYERS):
            for _ in range(self.T // 2048):
                k = torch.randn(self.B, self.H, 2048, self.D, generator=g, device=ctx.dev).half()
                v = torch.randn(self.B, self.H, 2048, self.D, generator=g, device=ctx.dev).half()
                self.cache.append(layer, k, v)
                del k, v
        self.q = torch.randn(self.B, self.HQ, 1, self.D, generator=g, device=ctx.dev).half()
        self.n_local = self.LAYERS
        self.n_total = self.LAYERS * ctx.world

    def bytes_per_layer(self):
        bht = self.B * self.H * self.T
        # K + V int8 codes, fp16 scale + zero point per token for each, q in, out
        return 2 * bht * self.D + 2 * 2 * bht * 2 + 2 * self.B * self.HQ * self.D * 2

    def bytes_for(self, n_layers):
        return self.bytes_per_layer() * n_layers

    def step(self):
        for layer in range(self.LAYERS):
            self.cache.attend(layer, self.q)

    def kernels(self):
        torch = self.ctx.torch
        c = [0]

        def f():
            self.cache.attend(c[0] % self.LAYERS, self.q)
            c[0] += 1
        t = cuda_time_ms(torch, f, 4 * self.LAYERS)
        n = self.B * self.H * self.T
        return {"kv_attn_kernel + combine (one layer)": (float(self.bytes_per_layer()), t, n,
                                                         "cached tokens")}

    def e2e(self, steps, graph):
        """attend() through the public API for every layer, with the query
        copied in from pinned host memory and the output copied back.  One
        stream: with 256 KB of transfers per step, HostPipeline's per-item
        stream and event handling cost more host time than the overlap saves
        (measured 1326 against 1759 GB/s before the combine kernel became a
        programmatic dependent launch)."""
        torch = self.ctx.torch
        hq = self.q.cpu().pin_memory()
        dq = torch.empty_like(self.q)
        outs = [torch.empty(self.q.shape, dtype=self.q.dtype).pin_memory() for _ in range(self.LAYERS)]

        def one():
            for layer in range(self.LAYERS):
                dq.copy_(hq, non_blocking=True)
                outs[layer].copy_(self.cache.attend(layer, dq), non_blocking=True)

        one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            one()
        e1.record()
        torch.cuda.synchronize()
        nb = self.q.numel() * 2 * self.LAYERS
        return e0.elapsed_time(e1) / steps, nb, nb

    def gather(self):
        return 0.0, 0

    @staticmethod
    def cpu_baseline():
        """The reference's read path on the host: dequantize the cached codes
        to fp32 (oracle kv_dequantize) and attend (numpy), for 2 (batch, kv
        head) slices of the same cache shape."""
        from oracle import lq_oracle as O
        rng = np.random.default_rng(0)
        T, D, G, n = 8192, 128, 4, 2
        sl = []
        for _ in range(n):
            k = O.rnd(rng.standard_normal((1, 1, T, D)).astype(np.float32), "float16")
            v = O.rnd(rng.standard_normal((1, 1, T, D)).astype(np.float32), "float16")
            kq = O.kv_quantize(k, "float16", 8, True, O.PER_TOKEN)
            vq = O.kv_quantize(v, "float16", 8, True, O.PER_TOKEN)
            q = O.rnd(rng.standard_normal((1, G, 1, D)).astype(np.float32), "float16")
            sl.append((kq, vq, q))

        def run(x):
            (kc, ks, kz), (vc, vs, vz), q = x
            fk = O.kv_dequantize(kc, ks, "float16", kz, "float16")
            fv = O.kv_dequantize(vc, vs, "float16", vz, "float16")
            O.kv_attention(q, fk, fv)

        t, nt = cpu_time(run, sl)
        b = n * (2 * T * D + 2 * 2 * T * 2 + 2 * G * D * 2)
        return {"value": b / t / 1e9, "unit": "GB/s", "cores": min(nt, n), "kind": "port",
                "sample": f"oracle dequantize + float64 attention, {n} (batch, kv head) slices of "
                          f"{T} tokens x {D}, 4 query heads each ({nt} threads), median of 3"}


def profile_case(name, ctx):
    """A small case of each workload's dominant kernel for ncu captures:
    inputs larger than L2 (126 MB) but a few hundred MB at most, 3 launches."""
    torch = ctx.torch
    import llm_quant_b200 as L
    g = torch.Generator(device=ctx.dev).manual_seed(0)
    if name == "nf4":
        w = (torch.randn(28672, 4096, generator=g, device=ctx.dev) * 0.02).to(torch.bfloat16)
        m = L.QLoRALinear(4096, 28672, rank=16, group_size=64).to(ctx.dev)
        for _ in range(3):
            m.pack_base(w)
            m._dequantize_base()
    elif name == "group":
        w = torch.randn(8192, 4096, generator=g, device=ctx.dev) * 0.02
        for _ in range(3):
            L.fake_quantize(w, 4, False, L.QScheme.PER_GROUP, 128)
    elif name == "rotquant":
        a = torch.randn(16384, 4096, generator=g, device=ctx.dev).to(torch.bfloat16)
        for _ in range(3):
            L.hadamard_fake_quantize(a, 4, True)
    elif name == "kv":
        cache = L.QuantizedKVCache(1, L.PerChannelKVCacheQuantizer(8),
                                   value_quantizer=L.PerTokenKVCacheQuantizer(4), max_seq_len=8192)
        for _ in range(16):
            k = torch.randn(8, 8, 512, 128, generator=g, device=ctx.dev).to(torch.bfloat16)
            cache.update(0, k, k)
    elif name == "w4a16":
        lin = torch.nn.Linear(4096, 14336, device=ctx.dev).half()
        ql = L.QuantizedLinear.from_linear(lin, 4, False, 128)
        x = torch.randn(1024, 4096, generator=g, device=ctx.dev).half()
        for _ in range(3):
            ql(x)
        for _ in range(3):
            ql(x[:1])
    elif name == "kv_attention":
        cache = L.QuantizedKVCache(1, max_seq_len=4096)
        for _ in range(2):
            k = torch.randn(8, 8, 2048, 128, generator=g, device=ctx.dev).half()
            cache.append(0, k, k)
        q = torch.randn(8, 32, 1, 128, generator=g, device=ctx.dev).half()
        for _ in range(3):
            cache.attend(0, q)
    elif name == "qlora_linear":
        w = (torch.randn(14336, 4096, generator=g, device=ctx.dev) * 0.02).to(torch.bfloat16)
        ql = L.QLoRALinear(4096, 14336, rank=16, group_size=64).to(ctx.dev)
        ql.pack_base(w)
        ql.requires_grad_(False)
        x = torch.randn(1024, 4096, generator=g, device=ctx.dev).to(torch.bfloat16)
        from llm_quant_b200 import nf4_linear
        with torch.no_grad():
            for _ in range(3):  # the base product alone (the bench's timed kernel)
                nf4_linear.base_linear(ql, x)
            for _ in range(3):
                ql(x)
            for _ in range(3):
                ql(x[:1])
    torch.cuda.synchronize()
    print(f"profile case {name} done")


WORKLOADS = {"nf4": NF4Workload, "group": GroupWorkload, "rotquant": RotQuantWorkload,
             "kv": KVWorkload, "w4a16": W4A16Workload, "qlora_linear": QLoRALinearWorkload,
             "kv_attention": KVAttentionWorkload}


# ─────────────────────────────────────────────────────────────────────────────

def run_reference(args):
    """--impl reference: the CPU oracle (restatement of the reference's
    algorithm) on the host cores, bounded sample per step; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    W = WORKLOADS[args.workload]
    for _ in range(args.warmup):
        W.cpu_baseline()
    vals, ts = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cb = W.cpu_baseline()
        ts.append(time.perf_counter() - t0)
        vals.append(cb["value"])
    v = statistics.median(vals)
    cb["value"] = v
    unit = cb["unit"]
    line = {"metric": METRIC, "value": v, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.median(ts), "higher_is_better": True,
            "scaling": "strong" if args.workload in ("nf4", "kv") else "weak",
            "vs_baseline": None,
            "dtype": {"group": "f32", "w4a16": "f16", "kv_attention": "f16"}.get(args.workload, "bf16"),
            "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": W.workload, "sample": cb["sample"]},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def other_kernels(ctx, nf4, hbm, tflops):
    """The rest of the metric beside the NF4 line, each kernel timed alone
    with CUDA events on its stream over inputs larger than L2: the NF4
    functional API with int64 codes, group fake-quant (fp32 4096 x 4096,
    INT4 asym g128), Hadamard + per-token INT4 (bf16 8192 x 4096) and the
    QuantizedLinear W4A16 forward (K 4096, N 14336, g128) at every M."""
    torch = ctx.torch

    def hbm_entry(b, t):
        gbs = b / (t * 1e-3) / 1e9
        return {"ms": t, "GB/s": gbs, "frac_of_peak": gbs / hbm}

    out = {k: hbm_entry(b, t) for k, (b, t, _, _) in nf4.api_int64_kernels().items()}
    for cls in (GroupWorkload, RotQuantWorkload):
        w = cls(ctx)
        out.update({k: hbm_entry(b, t) for k, (b, t, _, _) in w.kernels().items()})
        del w
    w = W4A16Workload(ctx)
    for k, (fl, t, m, wb) in w.kernels().items():
        tf = fl / (t * 1e-3) / 1e12
        gbs = wb / (t * 1e-3) / 1e9
        out[k] = {"ms": t, "TFLOP/s": tf, "frac_of_tensor_peak": tf / tflops, "GB/s": gbs,
                  "frac_of_hbm_peak": gbs / hbm, "bound": "hbm" if m <= 16 else "tensor"}
    del w
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    ctx = Ctx(args.gpus)
    torch = ctx.torch
    from llm_quant_b200 import _C
    hbm, tflops, peak_kind = peaks()
    W = WORKLOADS[args.workload](ctx)
    torch.cuda.synchronize()
    # one step captured as a CUDA graph; warm-up and timed steps replay it
    l0 = _C.launch_count()
    graph = capture(torch, W.step, 1)  # one eager call + one captured call
    launches_per_step = (_C.launch_count() - l0) // 2
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = ClockSampler(ctx.local == 0)
    time.sleep(0.2 if ctx.local == 0 else 0.0)
    ctx.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ctx.barrier()
    ck = clocks.stop(set(range(ctx.world))) if ctx.local == 0 else None
    ms = ctx.max(e0.elapsed_time(e1) / args.steps)
    unit = getattr(W, "unit", "GB/s")
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    total_bytes = W.bytes_for(W.n_total)
    value = total_bytes / (ms * 1e-3) / scale
    launches = launches_per_step * args.steps
    launches_all = int(ctx.sum(float(launches)))

    # dominant kernel, timed alone
    kern = W.kernels()
    traffic = NCU_TRAFFIC.get(W.name)
    if unit == "TFLOP/s":
        name = f"{W.main_kernel} M=1024"
        fl, kms, m, wb = kern[name]
        achieved = fl / (kms * 1e-3) / 1e12
        roofline = {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": tflops,
                    "unit": "TFLOP/s", "frac": achieved / tflops, "peak_kind": peak_kind,
                    "traffic": traffic, "algorithmic_flops_per_launch": fl, "launch_ms": kms,
                    "units_per_launch": f"{m} tokens x 4096 x 14336"}
        kernels = {}
        for k, (fl, t, m, wb) in kern.items():
            tf = fl / (t * 1e-3) / 1e12
            gbs = wb / (t * 1e-3) / 1e9
            kernels[k] = {"ms": t, "TFLOP/s": tf, "frac_of_tensor_peak": tf / tflops,
                          "GB/s": gbs, "frac_of_hbm_peak": gbs / hbm,
                          "bound": "hbm" if m <= 16 else "tensor"}
    else:
        name, (kb, kms, units, unit_name) = max(kern.items(), key=lambda kv: kv[1][1])
        achieved = kb / (kms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm,
                    "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind,
                    "traffic": traffic if traffic is None else traffic * units,
                    "algorithmic_bytes_per_launch": kb, "launch_ms": kms,
                    "units_per_launch": f"{units} {unit_name}"}
        kernels = {k: {"ms": v[1], "GB/s": v[0] / (v[1] * 1e-3) / 1e9,
                       "frac_of_peak": v[0] / (v[1] * 1e-3) / 1e9 / hbm} for k, v in kern.items()}
    if W.name == "nf4" and ctx.world == 1 and not args.no_extra:
        kernels.update(other_kernels(ctx, W, hbm, tflops))

    e2e_ms, h2d, d2h = W.e2e(max(1, args.e2e_steps), graph)
    e2e_ms = ctx.max(e2e_ms)
    e2e = {"value": total_bytes / (e2e_ms * 1e-3) / scale, "unit": unit,
           "h2d_bytes_per_step": int(ctx.sum(h2d)), "d2h_bytes_per_step": int(ctx.sum(d2h)),
           "ms_per_step": e2e_ms}
    gather_ms, gather_bytes = W.gather()
    gather_ms = ctx.max(gather_ms)
    job_ms = W.job_overlapped() if hasattr(W, "job_overlapped") else None
    job_ms = ctx.max(job_ms) if job_ms is not None else None

    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        cpu = W.cpu_baseline()
    if ctx.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong" if W.name in ("nf4", "kv") else "weak",
            "vs_baseline": None,
            "dtype": {"group": "f32", "w4a16": "f16", "kv_attention": "f16"}.get(W.name, "bf16"),
            "data": "synthetic (seeded torch.randn on the device)",
            "config": {"workload": W.workload, "parallelism": f"layer-shard x{ctx.world}"
                       if W.name in ("nf4", "kv") else f"independent x{ctx.world}",
                       "l2": "inputs larger than L2 (no flush)",
                       "launch": "one CUDA graph per step",
                       "algorithmic_bytes_per_step": total_bytes,
                       **({"algorithmic_bytes_per_weight": {
                           "packed_path (value)": total_bytes / W.n_total,
                           "api_int64_codes": 20.0 + 4.0 / 64}} if W.name == "nf4" else {})},
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_all,
            "clocks": ck,
            # one whole-model job = one step + the gather of its packed
            # results to rank 0 (exact sizes, point to point): after the step
            # (value_with_gather) and overlapped with it, layer by layer
            # (job_overlapped_ms, eager launches, value_with_gather_overlapped)
            "gather": {"ms": gather_ms, "bytes_to_rank0": gather_bytes,
                       "value_with_gather": total_bytes / ((ms + gather_ms) * 1e-3) / scale,
                       **({"job_overlapped_ms": job_ms,
                           "value_with_gather_overlapped": total_bytes / (job_ms * 1e-3) / scale}
                          if job_ms else {})}
            if ctx.world > 1 and gather_bytes else None,
        }
        print(json.dumps(line))
    ctx.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="nf4")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-extra", action="store_true",
                    help="default line: skip the other workloads' kernel timings")
    ap.add_argument("--profile", action="store_true",
                    help="only run a small case of the workload's dominant kernel (for ncu)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 warm-up steps
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        profile_case(args.workload, Ctx(args.gpus))
        return 0
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
