"""Install the reference package (Python, with its Triton kernels) into
``baseline/_ref/`` as a GPU comparator.

The reference checkout has no packaging metadata, so ``pip install`` cannot
take it as it is.  This recipe copies the checkout to a temporary directory
(the checkout itself is read-only), adds a minimal ``pyproject.toml`` that
names its ``aiwn`` package (packaging metadata only; no source of the
reference is changed), and runs the one offline install this build allows::

    python -m pip install --no-index --no-build-isolation --no-deps \
        --find-links /opt/wheelhouse --target baseline/_ref <copy>

    python baseline/install_ref.py --ref <reference checkout>   (or AIWN_REFERENCE=<...>)

``baseline/_ref/`` is git-ignored and travels with the working tree to the
GPU box, where ``bench.py`` imports ``aiwn.layers.indexed_linear`` from it
and times the reference's own ``_Fn`` (Triton forward, Triton dx and its
one-hot dtable) on the bench's device-resident inputs as
``reference_triton``.  Nothing under ``baseline/_ref/`` is imported by the
library, the tests' product path or ``smoke()``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "aiwn-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["aiwn*"]
"""


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=os.environ.get("AIWN_REFERENCE"), help="reference checkout (read only)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(os.path.join(args.ref, "aiwn")):
        print("no reference checkout given (--ref or AIWN_REFERENCE): reference package not installed")
        return 0
    os.makedirs(OUT, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "aiwn_reference")
        shutil.copytree(os.path.join(args.ref, "aiwn"), os.path.join(src, "aiwn"),
                        ignore=shutil.ignore_patterns("__pycache__", "build", "*.deb", "*.so", "*.o"))
        with open(os.path.join(src, "pyproject.toml"), "w") as f:
            f.write(PYPROJECT)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", OUT, "--upgrade", src]
        r = subprocess.run(cmd)
        if r.returncode != 0:
            print("pip install of the reference failed", file=sys.stderr)
            return r.returncode
    print("installed the reference package into", OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
