"""Install the reference package (MindIntels/llm_quant) into baseline/_ref.

    python oracle/install_ref.py [REFERENCE_SOURCE_DIR]

Test and measurement infrastructure only: the installed tree is what the
reference-suite GPU tests (tests/test_gpu_reference_suite.py) import the
reference's own test files from, and what bench.py's reference-torch CPU leg
times.  Nothing in the llm_quant_b200 package imports it.

The reference's source tree is itself the package (its __init__.py sits at
the root and imports ``.core``) and ships neither setup.py nor
pyproject.toml, so pip cannot install it in place.  The recipe copies it
under a temporary directory as ``llm_quant/``, writes a minimal
pyproject.toml beside it, and runs the one offline install allowed here:

    pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
                --target baseline/_ref <copy>

The source directory defaults to $LQ_REFERENCE_SRC, else /root/reference.
baseline/_ref is git-ignored (not product source) but travels to a GPU box
with the working tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TARGET = os.path.join(ROOT, "baseline", "_ref")

PYPROJECT = """\
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "llm_quant"
version = "0.0.0"

[tool.setuptools]
packages = ["llm_quant", "llm_quant.core", "llm_quant.tests"]
"""


def installed() -> bool:
    return os.path.exists(os.path.join(TARGET, "llm_quant", "qlora.py"))


def install(src: str | None = None, quiet: bool = True) -> str:
    src = src or os.environ.get("LQ_REFERENCE_SRC") or "/root/reference"
    if not os.path.exists(os.path.join(src, "__init__.py")):
        raise FileNotFoundError(f"no reference source tree at {src}")
    with tempfile.TemporaryDirectory() as tmp:
        pkg = os.path.join(tmp, "llm_quant")
        shutil.copytree(src, pkg, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        with open(os.path.join(tmp, "pyproject.toml"), "w") as f:
            f.write(PYPROJECT)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--find-links", "/opt/wheelhouse", "--no-deps", "--upgrade", "--target", TARGET, tmp]
        r = subprocess.run(cmd, capture_output=quiet, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference install failed:\n{r.stdout}\n{r.stderr}")
    return TARGET


if __name__ == "__main__":
    print(install(sys.argv[1] if len(sys.argv) > 1 else None, quiet=False))
