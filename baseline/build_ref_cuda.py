"""Build the reference's own CUDA extension for sm_100a, as a comparator.

The reference ships `aiwn/layers/indexed_linear_cuda.cu`, a PyTorch extension
(`forward(x, table, bias, bw)`, `backward(go, x, table, bw) -> [gx, gt]`).
This script compiles that file, unchanged and where it lies in the reference
checkout, with torch's extension builder (not the reference's setup script),
for sm_100a only, and leaves the module in ``baseline/_ref/`` (git-ignored;
it ships to the GPU box with the rest of the working tree).  Nothing of the
reference's source is copied.

    python baseline/build_ref_cuda.py --ref <reference checkout>   (or AIWN_REFERENCE=<...>)

`bench.py` times the module on the GPU as `reference_gpu` when it is present,
and `tests/test_reference_cuda_gpu.py` checks the library against it.
"""
from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "indexed_linear_cuda"
REL_SRC = os.path.join("aiwn", "layers", "indexed_linear_cuda.cu")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=os.environ.get("AIWN_REFERENCE"), help="reference checkout (read only)")
    args = ap.parse_args()
    if not args.ref:
        print("no reference checkout given (--ref or AIWN_REFERENCE): comparator not built")
        return 0
    src = os.path.join(args.ref, REL_SRC)
    if not os.path.exists(src):
        raise SystemExit(f"reference source not found: {src}")
    os.makedirs(OUT, exist_ok=True)
    # torch adds -gencode flags from this list; one architecture keeps the build short
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils.cpp_extension import load

    load(name=NAME, sources=[src], build_directory=OUT, extra_cuda_cflags=["-O3"], verbose=False)
    built = [f for f in os.listdir(OUT) if f.startswith(NAME) and f.endswith(".so")]
    print("built", [os.path.join(OUT, f) for f in built])
    return 0


if __name__ == "__main__":
    sys.exit(main())
