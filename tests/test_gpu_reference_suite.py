"""The reference's own hot-path tests, unmodified, run against this package
on the GPU (the drop-in acceptance test).

Each test function of the reference's tests/test_quantizer.py,
test_rotation.py, test_utils.py, test_qlora.py and test_kv_cache_quant.py is
collected as one parametrised case here.  The case registers this package
under the reference's import names (``install_as_llm_quant``), makes CUDA
torch's default device (the reference's tests build their tensors without a
device, and this package has no CPU implementation of the hot path), imports
the reference's test module from its file and calls the test method.

The reference's test files are read from an installed copy of the reference
(``python oracle/install_ref.py`` writes it to baseline/_ref, which is
git-ignored and not part of the product) or from $LQ_REFERENCE_TESTS.
Where neither exists the suite is skipped with that reason.  Nothing is
copied from the reference into this repository.
"""

from __future__ import annotations

import ast
import importlib.util
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = ["test_quantizer.py", "test_rotation.py", "test_utils.py", "test_qlora.py",
         "test_kv_cache_quant.py"]


def _tests_dir():
    for d in (os.environ.get("LQ_REFERENCE_TESTS"),
              os.path.join(ROOT, "baseline", "_ref", "llm_quant", "tests")):
        if d and all(os.path.exists(os.path.join(d, f)) for f in FILES):
            return d
    return None


def _collect():
    """(file, class, method) of every ``class Test*`` / ``def test_*`` in the
    reference's files, read with ast (nothing is imported at collection)."""
    d = _tests_dir()
    if d is None:
        return []
    cases = []
    for f in FILES:
        with open(os.path.join(d, f)) as fh:
            tree = ast.parse(fh.read())
        for node in tree.body:
            if isinstance(node, ast.ClassDef) and node.name.startswith("Test"):
                for item in node.body:
                    if isinstance(item, ast.FunctionDef) and item.name.startswith("test_"):
                        cases.append((f, node.name, item.name))
    return cases


CASES = _collect()


@pytest.fixture(scope="module")
def reference_modules():
    """Import each reference test file once, with llm_quant -> this package."""
    import llm_quant_b200 as L
    saved = {k: v for k, v in sys.modules.items() if k == "llm_quant" or k.startswith("llm_quant.")}
    L.install_as_llm_quant()
    mods = {}
    d = _tests_dir()
    prev = torch.get_default_device()
    torch.set_default_device("cuda")
    try:
        for f in FILES:
            spec = importlib.util.spec_from_file_location(f"lq_reference_suite_{f[:-3]}",
                                                          os.path.join(d, f))
            m = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(m)
            mods[f] = m
    finally:
        torch.set_default_device(prev)
    yield mods
    for k in [k for k in sys.modules if k == "llm_quant" or k.startswith("llm_quant.")]:
        del sys.modules[k]
    sys.modules.update(saved)


@pytest.mark.skipif(not CASES, reason="the reference's test files are not installed "
                    "(python oracle/install_ref.py, or set LQ_REFERENCE_TESTS)")
@pytest.mark.parametrize("fname,cls,meth", CASES or [("-", "-", "-")],
                         ids=[f"{f[5:-3]}::{c}::{m}" for f, c, m in CASES] or ["unavailable"])
def test_reference_suite(reference_modules, fname, cls, meth):
    from llm_quant_b200 import _C
    obj = getattr(reference_modules[fname], cls)()
    prev = torch.get_default_device()
    before = _C.launch_count()
    torch.set_default_device("cuda")
    try:
        getattr(obj, meth)()
    finally:
        torch.set_default_device(prev)
    _LAUNCHES[fname] = _LAUNCHES.get(fname, 0) + _C.launch_count() - before


_LAUNCHES: dict = {}


@pytest.mark.skipif(not CASES, reason="the reference's test files are not installed")
def test_reference_suite_ran_on_the_kernels():
    """The hot-path suites above went through this package's CUDA kernels."""
    for f in ("test_quantizer.py", "test_rotation.py", "test_qlora.py", "test_kv_cache_quant.py"):
        assert _LAUNCHES.get(f, 0) > 0, f"{f}: no liblq_sm100 kernel launched"
