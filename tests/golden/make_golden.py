"""Generate golden input/output vectors by running the reference llm_quant itself.

Run where the reference source tree (read-only) is available:

    python tests/golden/make_golden.py [--ref DIR] [quantizer rotation ...]

DIR defaults to $LQ_REFERENCE_SRC, else /root/reference.

The reference is pure PyTorch with relative imports; it is made importable as
``llm_quant`` through a symlink in a temporary directory (its files are never
copied).  Every case stores its seeded inputs and the reference outputs in
``tests/golden/*.npz``; ``bfloat16`` tensors are stored as their uint16 bit
patterns.  Case parameters live in the JSON string ``<case>/params``.

These fixtures pin the oracle (``oracle/lq_oracle.py``) and are the reference
side of the GPU parity tests; the tests read only the fixtures, never the reference.
"""

from __future__ import annotations

import json
import math
import os
import sys
import tempfile

import numpy as np
import torch

REF_SRC = os.environ.get("LQ_REFERENCE_SRC", "/root/reference")
HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference():
    tmp = tempfile.mkdtemp(prefix="lq_ref_")
    os.symlink(REF_SRC, os.path.join(tmp, "llm_quant"))
    sys.path.insert(0, tmp)
    import llm_quant  # noqa: F401  (the reference package)
    return llm_quant


DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def enc(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


class Store:
    def __init__(self):
        self.arrays = {}

    def add(self, case: str, params: dict, **tensors):
        assert f"{case}/params" not in self.arrays, case
        self.arrays[f"{case}/params"] = np.array(json.dumps(params))
        for k, v in tensors.items():
            if isinstance(v, torch.Tensor):
                self.arrays[f"{case}/{k}"] = enc(v)
                self.arrays[f"{case}/{k}.dtype"] = np.array(str(v.dtype).replace("torch.", ""))
            else:
                self.arrays[f"{case}/{k}"] = np.asarray(v)

    def save(self, name):
        path = os.path.join(HERE, name)
        np.savez_compressed(path, **self.arrays)
        print(f"wrote {path}: {len(self.arrays)} arrays, {os.path.getsize(path)} bytes")


def special_rows(x: torch.Tensor, kind: str) -> torch.Tensor:
    """Plant edge-case rows (first dim) into a 2-D+ float tensor."""
    x = x.clone()
    if kind == "zeros":
        x[0] = 0
    elif kind == "nan":
        x[1].view(-1)[3] = float("nan")
    elif kind == "inf":
        x[1].view(-1)[5] = float("inf")
    elif kind == "positive":
        x[0] = x[0].abs() + 0.5
    elif kind == "tiny":
        x[0] = x[0] * 1e-30 if x.dtype != torch.float16 else x[0] * 1e-6
    elif kind == "ties":
        # values on exact .5 code boundaries for sym 4-bit with amax 7
        x[0] = 0
        x[0].view(-1)[:8] = torch.tensor([7.0, -7.0, 0.5, 1.5, 2.5, -0.5, -2.5, 3.5])
    return x


# ─────────────────────────────────────────────────────────────────────────────

def gen_quantizer(ref):
    from llm_quant.core.quantizer import (compute_qparams, quantize_tensor, dequantize_tensor,
                                          fake_quantize, QScheme, QuantizedLinear, ste_round)
    st = Store()
    g = torch.Generator().manual_seed(1234)
    schemes = [
        ("per_group", (16, 256), 128),
        ("per_group", (3, 200), 128),
        ("per_group", (6, 70), 32),
        ("per_channel", (16, 64), 0),
        ("per_channel", (4, 6, 10), 0),
        ("per_tensor", (8, 64), 0),
    ]
    kinds = ["plain", "zeros", "nan", "inf", "positive", "tiny", "ties"]
    n = 0
    for dtn, dt in DT.items():
        for scheme, shape, gs in schemes:
            for kind in kinds:
                for sym in (True, False):
                    for bits in (4, 8):
                        if kind not in ("plain",) and bits == 8 and scheme != "per_group":
                            continue
                        x = torch.randn(shape, generator=g) * 0.7
                        if kind != "plain":
                            x = special_rows(x, kind)
                        x = x.to(dt)
                        sch = QScheme(scheme)
                        s, zp = compute_qparams(x, bits, sym, sch, gs if gs else 128)
                        if scheme == "per_group":
                            xg = x
                            pad = shape[1] % gs
                            if pad:
                                xg = torch.nn.functional.pad(x, (0, gs - pad))
                            xg = xg.reshape(shape[0], -1, gs)
                            q = quantize_tensor(xg, s, zp, bits, sym)
                        else:
                            q = quantize_tensor(x, s, zp, bits, sym)
                        dq = dequantize_tensor(q, s, zp)
                        fq = fake_quantize(x, bits, sym, sch, gs if gs else 128)
                        case = f"q{n:04d}"
                        n += 1
                        st.add(case, dict(fn="quantizer", dtype=dtn, scheme=scheme, shape=list(shape),
                                          group_size=gs if gs else 128, symmetric=sym, n_bits=bits,
                                          kind=kind),
                               x=x, scale=s, zp=zp, q=q, dq=dq, fq=fq)
    # ste_round known answer (tests/test_quantizer.py:20-24 of the reference)
    xs = torch.tensor([1.3, 2.7, -0.5, 0.0, -0.3, 2.5, float("inf")])
    st.add("ste", dict(fn="ste"), x=xs, y=ste_round(xs))
    # mixed-dtype quantize/dequantize (type promotion, 0-dim scalars)
    for i, (xd, sd, zd, zero_dim) in enumerate([
        ("bfloat16", "float32", "float32", True), ("bfloat16", "float32", "float32", False),
        ("float16", "bfloat16", "float16", False), ("float32", "bfloat16", "bfloat16", False),
        ("float16", "float32", "float16", True),
    ]):
        x = (torch.randn(5, 24, generator=g) * 3).to(DT[xd])
        if zero_dim:
            s = torch.tensor(0.0371, dtype=DT[sd])
            zp = torch.tensor(3.0, dtype=DT[zd])
        else:
            s = (torch.rand(5, 1, generator=g) * 0.1 + 0.01).to(DT[sd])
            zp = torch.round(torch.rand(5, 1, generator=g) * 8).to(DT[zd])
        q = quantize_tensor(x, s, zp, 4, False)
        dq = dequantize_tensor(q, s, zp)
        st.add(f"mixed{i}", dict(fn="mixed", zero_dim=zero_dim), x=x, scale=s, zp=zp, q=q, dq=dq)
    # QuantizedLinear: weight_int / scale / zero_point buffers and fp32 forward
    for i, (inf_, outf, bits, sym, gs, wdt) in enumerate([
        (256, 48, 4, False, 128, "float32"), (200, 16, 4, False, 128, "float16"),
        (64, 32, 8, True, 0, "float32"), (128, 64, 4, True, 32, "bfloat16"),
        (96, 24, 4, False, 32, "float16"), (64, 8, 8, False, 0, "float16"),
    ]):
        lin = torch.nn.Linear(inf_, outf)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(outf, inf_, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(outf, generator=g) * 0.1)
        lin = lin.to(DT[wdt])
        ql = QuantizedLinear.from_linear(lin, n_bits=bits, symmetric=sym, group_size=gs)
        x = torch.randn(5, inf_, generator=g)
        # forward needs fp32 x and fp32 bias: the module dequantizes to fp32
        ql_f = QuantizedLinear(inf_, outf, bits, sym, gs)
        ql_f.weight_int.copy_(ql.weight_int)
        ql_f.scale = ql.scale.clone()
        ql_f.zero_point = ql.zero_point.clone()
        with torch.no_grad():
            ql_f.bias.copy_(ql.bias.float())
        y = ql_f(x)
        st.add(f"qlin{i}", dict(fn="qlinear", in_features=inf_, out_features=outf, n_bits=bits,
                                symmetric=sym, group_size=gs, dtype=wdt),
               w=lin.weight.data, bias=lin.bias.data, weight_int=ql.weight_int, scale=ql.scale,
               zero_point=ql.zero_point, x=x, y=y)
    # wide codes (n_bits > 8): the reference's clamp converts qmax to the tensor
    # dtype (4095 acts as 4096 in bf16); fp16 with qmax = 65535 raises instead
    gw = torch.Generator().manual_seed(4242)
    w = 0
    for dtn, dt in DT.items():
        for bits in (10, 12, 16):
            for sym in (True, False):
                if dtn == "float16" and bits == 16 and not sym:
                    try:
                        fake_quantize(torch.randn(4, 64).half(), bits, sym, QScheme.PER_TENSOR)
                        raised = False
                    except RuntimeError:
                        raised = True
                    st.add("wide_fp16_raises", dict(fn="wide_raises", dtype=dtn, n_bits=bits,
                                                    symmetric=sym, raised=raised))
                    continue
                for scheme, shape, gs in (("per_group", (6, 192), 64), ("per_channel", (8, 48), 0),
                                          ("per_tensor", (4, 64), 0)):
                    x = (torch.randn(shape, generator=gw) * 2).to(dt)
                    sch = QScheme(scheme)
                    s, zp = compute_qparams(x, bits, sym, sch, gs if gs else 128)
                    if scheme == "per_group":
                        q = quantize_tensor(x.reshape(shape[0], -1, gs), s, zp, bits, sym)
                    else:
                        q = quantize_tensor(x, s, zp, bits, sym)
                    dq = dequantize_tensor(q, s, zp)
                    fq = fake_quantize(x, bits, sym, sch, gs if gs else 128)
                    st.add(f"w{w:04d}", dict(fn="quantizer", dtype=dtn, scheme=scheme, shape=list(shape),
                                             group_size=gs if gs else 128, symmetric=sym, n_bits=bits,
                                             kind="wide"),
                           x=x, scale=s, zp=zp, q=q, dq=dq, fq=fq)
                    w += 1
    st.save("quantizer.npz")


def gen_rotation(ref):
    from llm_quant.core.rotation import hadamard_matrix, fast_hadamard_transform
    st = Store()
    g = torch.Generator().manual_seed(99)
    for dtn, dt in DT.items():
        ent = []
        for k in range(0, 15):
            n = 2 ** k
            H = hadamard_matrix(n, dt) if n <= 1024 else None
            if H is not None:
                ent.append(H.abs().float().max().item())
                assert torch.all(H.abs() == H.abs().max())
            else:
                ent.append((torch.ones(1, dtype=dt) / math.sqrt(n)).float().item())
        st.add(f"hent_{dtn}", dict(fn="hadamard_entries", dtype=dtn), ent=np.array(ent, np.float32))
        st.add(f"h8_{dtn}", dict(fn="hadamard", n=8, dtype=dtn), H=hadamard_matrix(8, dt))
    for i, (shape, dtn) in enumerate([((4, 16), "float32"), ((3, 5, 64), "bfloat16"),
                                       ((2, 2048), "bfloat16"), ((3, 4096), "bfloat16"),
                                       ((2, 1024), "float16"), ((4, 256), "float32"),
                                       ((2, 2), "float32"), ((1, 8192), "bfloat16")]):
        x = torch.randn(shape, generator=g).to(DT[dtn])
        st.add(f"fht{i}", dict(fn="fht", dtype=dtn, shape=list(shape)), x=x,
               y=fast_hadamard_transform(x))
    st.save("rotation.npz")


def _bf16_grid_unit():
    """Every bfloat16 value in [-1, 1] (as float32)."""
    u = np.arange(0, 0x10000, dtype=np.uint32) << 16
    v = u.view(np.float32)
    v = v[np.isfinite(v) & (np.abs(v) <= 1.0)]
    return np.unique(v)


def _f16_grid_unit():
    v = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    v = v[np.isfinite(v) & (np.abs(v) <= 1.0)]
    return np.unique(v)


def _f32_midpoint_grid(table):
    """fp32 values within +-96 ulps of every NF4 level and every midpoint between levels."""
    t = table.numpy().astype(np.float32)
    pts = []
    for a, b in zip(t[:-1], t[1:]):
        for m in (np.float32((np.float64(a) + np.float64(b)) / 2), np.float32(a), np.float32(b)):
            up = dn = m
            pts.append(m)
            for _ in range(96):
                up = np.nextafter(up, np.float32(np.inf), dtype=np.float32)
                dn = np.nextafter(dn, np.float32(-np.inf), dtype=np.float32)
                pts += [up, dn]
    v = np.array(pts, np.float32)
    return np.unique(v[np.abs(v) <= 1.0])


def gen_nf4(ref):
    from llm_quant.qlora import (NF4_TABLE, nf4_quantize, nf4_dequantize, double_quantize,
                                 double_dequantize, QLoRALinear)
    st = Store()
    g = torch.Generator().manual_seed(7)
    st.add("table", dict(fn="table"), table=NF4_TABLE)
    for dtn, dt in DT.items():
        for i, (shape, gs, kind) in enumerate([((32, 64), 64, "plain"), ((7, 50), 64, "plain"),
                                               ((16, 128), 16, "plain"), ((8, 16), 16, "zeros"),
                                               ((4, 64), 64, "nan"), ((4, 64), 64, "inf"),
                                               ((3, 33), 32, "plain"), ((6, 64), 64, "tiny")]):
            x = torch.randn(shape, generator=g) * 0.5
            if kind != "plain":
                x = special_rows(x, kind) if kind != "zeros" else torch.zeros(shape)
            x = x.to(dt)
            codes, scales = nf4_quantize(x, gs)
            deq = nf4_dequantize(codes, scales, gs)
            st.add(f"nf4_{dtn}_{i}", dict(fn="nf4", dtype=dtn, shape=list(shape), group_size=gs,
                                          kind=kind),
                   x=x, codes=codes, scales=scales, deq=deq)
    # exhaustive decision-boundary grids: absmax is exactly 1 so x_norm == x
    grids = {"bfloat16": _bf16_grid_unit(), "float16": _f16_grid_unit(),
             "float32": _f32_midpoint_grid(NF4_TABLE)}
    for dtn, v in grids.items():
        gs = 64
        n = int(math.ceil(len(v) / (gs - 1)))
        xs = np.zeros((n, gs), np.float32)
        flat = np.concatenate([v, np.zeros(n * (gs - 1) - len(v), np.float32)])
        xs[:, :gs - 1] = flat.reshape(n, gs - 1)
        xs[:, gs - 1] = 1.0
        x = torch.from_numpy(xs).to(DT[dtn])
        codes, scales = nf4_quantize(x, gs)
        st.add(f"grid_{dtn}", dict(fn="nf4_grid", dtype=dtn, group_size=gs), x=x,
               codes=codes.to(torch.uint8), scales=scales)
    # double quantization
    for dtn, dt in DT.items():
        for i, (n, dgs) in enumerate([(256, 64), (1000, 256), (128, 32), (300, 256)]):
            s = (torch.rand(n, generator=g) * 0.1 + 0.01).to(dt)
            if i == 3:
                s[:256] = 0
            q, dq = double_quantize(s, dgs)
            rs = double_dequantize(q, dq, dgs)
            st.add(f"dq_{dtn}_{i}", dict(fn="double_quant", dtype=dtn, n=n, dq_group_size=dgs),
                   s=s, q=q, dq=dq, restored=rs)
    # QLoRALinear base packing and dequantized base weight
    for i, (inf_, outf, gs, dq, dtn) in enumerate([(64, 32, 64, True, "float32"),
                                                   (96, 40, 64, True, "bfloat16"),
                                                   (32, 16, 32, False, "bfloat16"),
                                                   (128, 24, 64, True, "float16")]):
        w = (torch.randn(outf, inf_, generator=g) * 0.02).to(DT[dtn])
        ql = QLoRALinear(inf_, outf, rank=4, group_size=gs, double_quant=dq)
        ql.pack_base(w)
        wb = ql._dequantize_base()
        extra = dict(dq_q_scales=ql.dq_q_scales, dq_scales=ql.dq_scales) if dq else {}
        st.add(f"qlora{i}", dict(fn="qlora", in_features=inf_, out_features=outf, group_size=gs,
                                 double_quant=dq, dtype=dtn),
               w=w, nf4_codes=ql.nf4_codes, nf4_scales=ql.nf4_scales, w_base=wb, **extra)
    st.save("nf4.npz")


def gen_kv(ref):
    from llm_quant.kv_cache_quant import (KVQuantGranularity as G, KVCacheQuantizer,
                                          QuantizedKVCache)
    st = Store()
    g = torch.Generator().manual_seed(2024)
    n = 0
    for dtn, dt in DT.items():
        for gran in ("per_token", "per_channel", "per_group"):
            for sym in (True, False):
                for bits in (4, 8):
                    for T, gs, kind in ((16, 8, "plain"), (13, 8, "plain"), (16, 4, "special")):
                        if gran != "per_group" and T == 13 and bits == 4:
                            continue
                        x = torch.randn(2, 4, T, 32, generator=g)
                        if kind == "special":
                            x[0, 0] = 0
                            x[0, 1, 2, 3] = float("nan")
                            x[1, 2, :, 5] *= 40
                            x[1, 3] = x[1, 3].abs() + 1
                        x = x.to(dt)
                        qz = KVCacheQuantizer(bits, sym, G(gran), gs)
                        q, s, zp = qz.quantize(x)
                        dqv = qz.dequantize(q, s, zp)
                        st.add(f"kv{n:04d}", dict(fn="kv", dtype=dtn, granularity=gran, symmetric=sym,
                                                  n_bits=bits, group_size=gs, kind=kind),
                               x=x, q=q, scale=s, zp=zp, deq=dqv)
                        n += 1
    # QuantizedKVCache update sequences
    seqs = [
        ("per_token", 8, True, 8, [3, 2, 1, 4], "bfloat16", None),
        ("per_channel", 8, True, 8, [4, 4, 4], "bfloat16", 10.0),
        ("per_channel", 4, False, 8, [2, 3], "float32", None),
        ("per_group", 4, True, 4, [4, 4, 4], "float16", None),
        ("per_group", 8, False, 4, [4, 6], "bfloat16", None),
        ("per_token", 4, False, 8, [5, 1, 1], "float32", None),
    ]
    for i, (gran, bits, sym, gs, chunks, dtn, boost) in enumerate(seqs):
        qz = KVCacheQuantizer(bits, sym, G(gran), gs)
        cache = QuantizedKVCache(2, qz)
        ks, vs, fks, fvs = [], [], [], []
        for j, c in enumerate(chunks):
            k = torch.randn(2, 3, c, 16, generator=g)
            v = torch.randn(2, 3, c, 16, generator=g)
            if boost is not None and j == 1:
                k = k * boost
            k, v = k.to(DT[dtn]), v.to(DT[dtn])
            fk, fv = cache.update(1, k, v)
            ks.append(k); vs.append(v); fks.append(fk); fvs.append(fv)
        tens = {}
        for j in range(len(chunks)):
            tens[f"k{j}"] = ks[j]; tens[f"v{j}"] = vs[j]
            tens[f"fk{j}"] = fks[j]; tens[f"fv{j}"] = fvs[j]
        st.add(f"cache{i}", dict(fn="kv_cache", granularity=gran, n_bits=bits, symmetric=sym,
                                 group_size=gs, chunks=chunks, dtype=dtn), **tens)
    # mixed granularity (K per-channel INT8 sym, V per-token INT4 sym) as two reference caches
    kc = QuantizedKVCache(1, KVCacheQuantizer(8, True, G.PER_CHANNEL))
    vc = QuantizedKVCache(1, KVCacheQuantizer(4, True, G.PER_TOKEN))
    tens = {}
    for j in range(3):
        k = torch.randn(2, 2, 8, 32, generator=g).to(torch.bfloat16)
        v = torch.randn(2, 2, 8, 32, generator=g).to(torch.bfloat16)
        fk, _ = kc.update(0, k, k)
        _, fv = vc.update(0, v, v)
        tens.update({f"k{j}": k, f"v{j}": v, f"fk{j}": fk, f"fv{j}": fv})
    st.add("cache_mixed", dict(fn="kv_cache_mixed", dtype="bfloat16", chunks=[8, 8, 8]), **tens)
    # wide codes (n_bits > 8; int16 codes when asymmetric, wrapped int8 when symmetric)
    gw = torch.Generator().manual_seed(4243)
    w = 0
    for dtn, dt in DT.items():
        for gran in ("per_token", "per_channel", "per_group"):
            for bits, sym in ((12, False), (16, True), (10, True)):
                x = (torch.randn(2, 3, 9, 24, generator=gw) * 2).to(dt)
                qz = KVCacheQuantizer(bits, sym, G(gran), 4)
                q, s, zp = qz.quantize(x)
                dqv = qz.dequantize(q, s, zp)
                st.add(f"kvw{w:04d}", dict(fn="kv", dtype=dtn, granularity=gran, symmetric=sym,
                                           n_bits=bits, group_size=4, kind="wide"),
                       x=x, q=q, scale=s, zp=zp, deq=dqv)
                w += 1
    st.save("kv.npz")


def gen_grad(ref):
    """fake_quantize gradients under the reference's autograd."""
    from llm_quant.core.quantizer import fake_quantize, QScheme
    st = Store()
    g = torch.Generator().manual_seed(77)
    n = 0
    for dtn in ("float32", "bfloat16", "float16"):
        for scheme, shape, gs in (("per_group", (12, 256), 128), ("per_group", (5, 70), 32),
                                  ("per_channel", (9, 48), 128), ("per_channel", (4, 3, 10), 128),
                                  ("per_tensor", (6, 40), 128)):
            for sym in (True, False):
                bits = 4
                x = torch.randn(shape, generator=g) * 0.5
                x.view(-1)[7] = x.view(-1)[3]  # a tie
                x = x.to(DT[dtn]).requires_grad_(True)
                go = torch.randn(shape, generator=g).to(DT[dtn])
                y = fake_quantize(x, bits, sym, QScheme(scheme), gs)
                y.backward(go)
                st.add(f"g{n:03d}", dict(fn="grad", dtype=dtn, scheme=scheme, shape=list(shape),
                                         group_size=gs, symmetric=sym, n_bits=bits),
                       x=x.detach(), go=go, y=y.detach(), gx=x.grad)
                n += 1
    st.save("grad.npz")


def gen_layers(ref):
    """GPTQLinear / SpQRLinear (gptq.py:257-325, spqr.py:102-208): buffers after
    pack, forward on seeded x, and the dequantized weight the forward builds,
    read out exactly as layer(I) = W^T (bias-free copies)."""
    from llm_quant.gptq import GPTQLinear
    from llm_quant.spqr import SpQRLinear
    st = Store()
    g = torch.Generator().manual_seed(777)
    for i, (inf_, outf, bits, sym, gs) in enumerate([(64, 16, 4, True, 32), (32, 16, 4, True, 0),
                                                     (200, 24, 4, False, 128), (128, 32, 3, True, 64),
                                                     (256, 128, 4, False, 64)]):
        W = torch.randn(outf, inf_, generator=g)
        lo, hi = (-(2 ** (bits - 1)), 2 ** (bits - 1) - 1) if sym else (0, 2 ** bits - 1)
        w_q = torch.randint(lo, hi + 1, (outf, inf_), generator=g)
        ql = GPTQLinear(inf_, outf, n_bits=bits, symmetric=sym, group_size=gs, bias=True)
        ql.pack(w_q, W)
        with torch.no_grad():
            ql.bias.copy_(torch.randn(outf, generator=g) * 0.1)
        x = torch.randn(5, inf_, generator=g)
        y = ql(x)
        nb = GPTQLinear(inf_, outf, n_bits=bits, symmetric=sym, group_size=gs, bias=False)
        nb.pack(w_q, W)
        wT = nb(torch.eye(inf_))
        st.add(f"gptq{i}", dict(fn="gptq", in_features=inf_, out_features=outf, n_bits=bits,
                                symmetric=sym, group_size=gs),
               W=W, w_q=w_q.to(torch.int8), weight_int=ql.weight_int, scale=ql.scale,
               zero_point=ql.zero_point, bias=ql.bias.data, x=x, y=y, wT=wT)
    for i, (inf_, outf, bits, gs, frac) in enumerate([(64, 32, 4, 32, 0.02), (32, 16, 8, 0, 0.05),
                                                      (200, 24, 4, 128, 0.01), (256, 128, 4, 64, 0.01)]):
        W = torch.randn(outf, inf_, generator=g)
        mask = torch.rand(outf, inf_, generator=g) < frac
        mask[0, 0] = True
        layer = SpQRLinear(inf_, outf, n_bits=bits, group_size=gs, bias=True)
        layer.pack(W, mask)
        with torch.no_grad():
            layer.bias.copy_(torch.randn(outf, generator=g) * 0.1)
        x = torch.randn(5, inf_, generator=g)
        y = layer(x)
        nb = SpQRLinear(inf_, outf, n_bits=bits, group_size=gs, bias=False)
        nb.pack(W, mask)
        wT = nb(torch.eye(inf_))
        st.add(f"spqr{i}", dict(fn="spqr", in_features=inf_, out_features=outf, n_bits=bits,
                                group_size=gs, sparsity=layer.sparsity),
               W=W, mask=mask.to(torch.uint8), weight_int=layer.weight_int, scale=layer.scale,
               zero_point=layer.zero_point, outlier_vals=layer.outlier_vals, bias=layer.bias.data,
               x=x, y=y, wT=wT)
    st.save("layers.npz")


def gen_helpers(ref):
    """The reference's rotation-construction helpers and core.utils (off the
    hot path; eager torch on the CPU in both packages)."""
    from llm_quant.core import rotation as R
    from llm_quant.core import utils as U
    st = Store()
    for n, dtn, seed in [(16, "float32", 123), (64, "float32", 7), (32, "bfloat16", 8)]:
        st.add(f"rhad_{n}_{dtn}", dict(fn="random_hadamard_matrix", n=n, dtype=dtn, seed=seed),
               H=R.random_hadamard_matrix(n, DT[dtn], generator=torch.Generator().manual_seed(seed)))
    for n, seed in [(8, 1), (32, 2)]:
        st.add(f"rorth_{n}", dict(fn="random_orthogonal", n=n, seed=seed),
               Q=R.random_orthogonal(n, generator=torch.Generator().manual_seed(seed)))
    g = torch.Generator().manual_seed(11)
    a = torch.randn(12, 12, generator=g)
    a = a - a.t()
    st.add("cayley", dict(fn="cayley_transform"), A=a, Q=R.cayley_transform(a))
    cr = R.CayleyRotation(6)
    with torch.no_grad():
        cr.params.copy_(torch.randn(cr.params.shape, generator=g) * 0.3)
    st.add("cayley_rot", dict(fn="CayleyRotation", dim=6), p=cr.params.data, Q=cr().detach())
    w = torch.randn(6, 10, generator=g)
    r10 = R.random_orthogonal(10, generator=torch.Generator().manual_seed(3))
    r6 = R.random_orthogonal(6, generator=torch.Generator().manual_seed(4))
    st.add("rotate", dict(fn="rotate_weight"), W=w, R10=r10, R6=r6,
           right=R.rotate_weight_right(w, r10), left=R.rotate_weight_left(w, r6))
    batches = [torch.randn(3, 5, 4, generator=g) * (i + 1) for i in range(3)]
    obs = {}
    for key, kw in [("tensor", dict()), ("ch_last", dict(per_channel=True, channel_dim=-1)),
                    ("ch0", dict(per_channel=True, channel_dim=0)),
                    ("ch1", dict(per_channel=True, channel_dim=1))]:
        o = U.MinMaxObserver(**kw)
        for b in batches:
            o.update(b)
        obs[f"{key}_min"], obs[f"{key}_max"] = o.get_range()
    st.add("observer", dict(fn="MinMaxObserver"), b0=batches[0], b1=batches[1], b2=batches[2], **obs)
    x = torch.randn(64, 8, generator=g)
    y = x + torch.randn(64, 8, generator=g) * 0.05
    st.add("metrics", dict(fn="metrics"), x=x, y=y, mse=U.quantization_mse(x, y),
           snr=U.quantization_snr(x, y), kurt0=U.kurtosis(x, dim=0), kurt1=U.kurtosis(x))
    lin = U.make_dummy_linear(64, 32)
    lin_nb = U.make_dummy_linear(16, 8, bias=False)
    st.add("dummy_linear", dict(fn="make_dummy_linear"), w=lin.weight.data, b=lin.bias.data,
           w_nb=lin_nb.weight.data)
    cal = U.make_calibration_data(2, 4, 8, 3, seed=5)
    st.add("calib", dict(fn="make_calibration_data"), d0=cal[0], d1=cal[1], d2=cal[2])
    st.save("helpers.npz")


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    args = sys.argv[1:]
    if "--ref" in args:
        i = args.index("--ref")
        REF_SRC = args[i + 1]
        del args[i:i + 2]
    ref = _import_reference()
    which = args or ["quantizer", "rotation", "nf4", "kv", "grad", "layers", "helpers"]
    for name in which:
        globals()[f"gen_{name}"](ref)
