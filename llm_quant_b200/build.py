"""Build liblq_sm100.so in-tree with nvcc for sm_100a (B200).

    python -m llm_quant_b200.build        # or: python llm_quant_b200/build.py

Each .cu under csrc/ is compiled to an object (in parallel, skipped when up
to date) and linked into llm_quant_b200/_lib/liblq_sm100.so.  The elementwise
quantization sources are compiled with --fmad=false on top of the explicit
__f*_rn intrinsics: the reference rounds after every torch op, so no two ops
may be contracted into one FMA.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
OBJDIR = os.path.join(HERE, "_lib", "obj")
LIB = os.path.join(LIBDIR, "liblq_sm100.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", INCLUDE,
          "--expt-relaxed-constexpr"]
# sources whose arithmetic must not be contracted (bit-exact parity)
EXACT = {"lq_group.cu", "lq_kv.cu", "lq_nf4.cu", "lq_hadamard.cu", "lq_affine.cu", "lq_api.cu"}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(OBJDIR, src.replace(".cu", ".o"))
    srcp = os.path.join(CSRC, src)
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(srcp), _headers_mtime()):
            return obj
    flags = list(COMMON)
    if src in EXACT:
        flags += ["--fmad=false"]
    cmd = [nvcc()] + ARCH + flags + ["-c", srcp, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
