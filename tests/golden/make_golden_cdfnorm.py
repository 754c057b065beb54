"""Generate the IndexedLinearV2 golden fixtures (cdfnorm_*.npz) by running the
REFERENCE.

Run once, where a read-only checkout of the reference is available (it is
not present where the tests run), naming it with AIWN_REFERENCE::

    AIWN_REFERENCE=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_cdfnorm.py

Each case builds seeded CPU inputs and runs the reference's own modules on
CPU: ``aiwn.layers.indexed_linear_v2.GaussianCDFNorm`` (LayerNorm with
non-trivial gamma / beta, then the erf CDF) feeding
``aiwn.layers.indexed_linear.IndexedLinear`` (its ``_eager`` path on CPU
tensors) -- the chain of ``IndexedLinearV2.forward``
(aiwn/layers/indexed_linear_v2.py:80-88) -- and ``out.backward(go)``.  Stored:
inputs, xn (the prologue's output), out, and the gradients of x, gamma, beta,
table, bias and xn.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch



def _reference_dir() -> str:
    ref = os.environ.get("AIWN_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "aiwn")):
        raise SystemExit("set AIWN_REFERENCE to the reference checkout (the directory holding aiwn/)")
    return ref


HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    # name, N, IN, OUT, K, seed
    ("cdfnorm_20x20_k64", 512, 20, 20, 64, 41),
    ("cdfnorm_16x8_k128", 300, 16, 8, 128, 42),
]


def main():
    sys.path.insert(0, _reference_dir())
    from aiwn.layers.indexed_linear import IndexedLinear  # noqa: E402
    from aiwn.layers.indexed_linear_v2 import GaussianCDFNorm  # noqa: E402

    for name, N, IN, OUT, K, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(N, IN, generator=g) * 1.7 + 0.3
        gamma = 1.0 + 0.3 * torch.randn(IN, generator=g)
        beta = 0.2 * torch.randn(IN, generator=g)
        table = torch.randn(K, IN, OUT, generator=g) / IN ** 0.5
        bias = 0.1 * torch.randn(OUT, generator=g)
        go = torch.randn(N, OUT, generator=g)

        cdf = GaussianCDFNorm(IN)
        lin = IndexedLinear(IN, OUT, K)
        with torch.no_grad():
            cdf.ln.weight.copy_(gamma)
            cdf.ln.bias.copy_(beta)
            lin.table.copy_(table)
            lin.bias.copy_(bias)
        xr = x.clone().requires_grad_(True)
        xn = cdf(xr)
        xn.retain_grad()
        out = lin(xn)
        out.backward(go)
        f = lambda t: t.detach().contiguous().numpy().astype(np.float32, copy=True)  # noqa: E731
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            x=f(x), gamma=f(gamma), beta=f(beta), table=f(table), bias=f(bias), go=f(go),
            eps=np.float64(cdf.ln.eps), bw=np.float64(lin.bw), K=np.int64(K),
            xn=f(xn), out=f(out), gx=f(xr.grad), ggamma=f(cdf.ln.weight.grad), gbeta=f(cdf.ln.bias.grad),
            gt=f(lin.table.grad), gb=f(lin.bias.grad), gxn=f(xn.grad))
        print("wrote", name)


if __name__ == "__main__":
    main()
