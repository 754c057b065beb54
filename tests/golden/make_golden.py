"""Generate the golden fixtures in this directory by running the REFERENCE.

Run once, where a read-only checkout of the reference is available (it is
not present where the tests run), naming it with AIWN_REFERENCE::

    AIWN_REFERENCE=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py

For every case it builds seeded CPU inputs, calls the reference module's own
CPU path -- ``aiwn.layers.indexed_linear.IndexedLinear.forward`` on CPU
tensors, which dispatches to ``_eager`` (aiwn/layers/indexed_linear.py:184-190)
-- and then ``out.backward(go)``, i.e. PyTorch autograd's backward of that
path.  Inputs, outputs and gradients are written to ``<case>.npz``.

The bin indices and fractions are recomputed here with the same torch
expressions as aiwn/layers/indexed_linear.py:175-177 (they are internal to
``_eager``), and the ``bins_*`` cases hold large sweeps of x values for the
bit-exact bin tests.

bf16 arrays are stored as uint16 bit patterns.
"""
from __future__ import annotations

import hashlib
import math
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


def _ref_module():
    sys.path.insert(0, _reference_dir())
    from aiwn.layers.indexed_linear import IndexedLinear, indexed_dims  # noqa: E402
    return IndexedLinear, indexed_dims


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.detach().contiguous().numpy().astype(np.float32, copy=True)


def ref_bins(x: torch.Tensor, K: int, bw: float):
    """Same expressions as aiwn/layers/indexed_linear.py:175-177."""
    bk = ((x + 1) / bw).long().clamp(0, K - 1)
    hi = (bk + 1).clamp(max=K - 1)
    fr = ((x - (-1 + bk.float() * bw)) / bw).clamp(0, 1)
    return bk.to(torch.int32), hi.to(torch.int32), fr.float()


def seeded_table(K, IN, OUT, seed):
    """table ~ N(0, 1/IN) from a seeded CPU generator; tests regenerate it the
    same way (tests/golden_io.py) and check the stored sha256."""
    return torch.randn(K, IN, OUT, generator=torch.Generator().manual_seed(seed)) / math.sqrt(IN)


def run_case(name, IL, N, IN, OUT, K, x, seed_t, seed_b, seed_g, bias_scale=0.0):
    layer = IL(IN, OUT, K)
    table = seeded_table(K, IN, OUT, seed_t)
    with torch.no_grad():
        layer.table.copy_(table)
        gb_ = torch.Generator().manual_seed(seed_b)
        layer.bias.copy_(torch.randn(OUT, generator=gb_) * bias_scale)
    go = torch.randn(N, OUT, generator=torch.Generator().manual_seed(seed_g))
    xl = x.clone().requires_grad_(True)
    out = layer(xl)  # CPU tensors -> the reference's _eager path
    assert out.dtype == torch.float32
    out.backward(go)
    lo, hi, fr = ref_bins(x, K, layer.bw)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        K=np.int64(K), bw=np.float64(layer.bw), x_dtype=np.array("bf16" if x.dtype == torch.bfloat16 else "f32"),
        x=_bits(x), table_seed=np.int64(seed_t), table_shape=np.array([K, IN, OUT], np.int64),
        table_sha256=np.array(hashlib.sha256(_bits(table).tobytes()).hexdigest()), bias=_bits(layer.bias.detach()),
        go=_bits(go), out=_bits(out.detach()), gx=_bits(xl.grad), gt=_bits(layer.table.grad),
        gb=_bits(layer.bias.grad), lo=lo.numpy(), hi=hi.numpy(), fr=_bits(fr),
    )
    print(f"{name}: N={N} IN={IN} OUT={OUT} K={K} dtype={x.dtype}")


def edge_values(K: int, bw: float, n_rand: int, gen) -> torch.Tensor:
    """Bin edges -1 + k*bw (fp32, as the reference rounds them), their fp32
    neighbours, out-of-range values, and uniform values in [-1.25, 1.25]."""
    e = []
    for k in range(K + 1):
        c = torch.tensor(float(k), dtype=torch.float32) * bw + (-1)
        e += [c.item(), torch.nextafter(c, torch.tensor(2.0)).item(), torch.nextafter(c, torch.tensor(-2.0)).item()]
    e += [-1.0, 1.0, 0.0, -0.0, -1.5, 1.5, -3.0, 3.0, -1.0 - bw, 1.0 + bw, 1e-8, -1e-8]
    r = (torch.rand(n_rand, generator=gen) * 2.5 - 1.25).tolist()
    return torch.tensor(e + r, dtype=torch.float32)


def main():
    IL, indexed_dims = _ref_module()
    torch.manual_seed(0)

    # C1 shape (d=256, K=16 -> in=out=indexed_dims(256, 1024, 16)[0] = 64), fewer tokens
    d_idx = indexed_dims(256, 1024, 16)[0]
    assert d_idx == 64
    x = torch.rand(96, 64, generator=torch.Generator().manual_seed(0)) * 2 - 1
    run_case("c1_small", IL, 96, 64, 64, 16, x, 1, 3, 2)

    # C2 shape (d=256, K=128 -> in=out=20), bf16 x = tanh(N(0,1))
    assert indexed_dims(256, 1024, 128)[0] == 20
    x = torch.tanh(torch.randn(256, 20, generator=torch.Generator().manual_seed(10))).to(torch.bfloat16)
    run_case("c2_small_bf16", IL, 256, 20, 20, 128, x, 11, 13, 12, bias_scale=0.1)

    # C3 shape (d=512, K=512 -> in=out=20), fp32 x ~ U(-1,1)
    assert indexed_dims(512, 2048, 512)[0] == 20
    x = torch.rand(96, 20, generator=torch.Generator().manual_seed(20)) * 2 - 1
    run_case("c3_small", IL, 96, 20, 20, 512, x, 21, 23, 22, bias_scale=0.1)

    # the reference benchmark shape IndexedLinear(d_idx, 4*d_idx, K) = (20, 80), smaller K
    x = torch.rand(64, 20, generator=torch.Generator().manual_seed(30)) * 2 - 1
    run_case("refshape_20x80_k32", IL, 64, 20, 80, 32, x, 31, 33, 32, bias_scale=0.1)

    # C4 scaled down (K=64, x = clamp(N(0, 0.5), -1, 1))
    x = (torch.randn(64, 32, generator=torch.Generator().manual_seed(40)) * 0.5).clamp(-1, 1)
    run_case("c4_small", IL, 64, 32, 24, 64, x, 41, 43, 42, bias_scale=0.1)

    # C5 projection shapes (d_idx=16, ff_idx=8, K=128)
    x = torch.rand(64, 16, generator=torch.Generator().manual_seed(50)) * 2 - 1
    run_case("c5_up_16x8", IL, 64, 16, 8, 128, x, 51, 53, 52, bias_scale=0.1)

    # edge cases: K=2, tiny dims
    x = torch.rand(33, 1, generator=torch.Generator().manual_seed(60)) * 3 - 1.5
    run_case("k2_in1_out1", IL, 33, 1, 1, 2, x, 61, 63, 62, bias_scale=1.0)

    # non-power-of-two K, values on/near every bin edge and outside [-1, 1]
    for K, OUT in ((3, 3), (7, 5), (100, 12)):
        gen = torch.Generator().manual_seed(70 + K)
        v = edge_values(K, 2.0 / K, 64, gen)
        IN = 4
        n = (v.numel() + IN - 1) // IN
        v = torch.cat([v, torch.zeros(n * IN - v.numel())])
        x = v[torch.randperm(v.numel(), generator=gen)].reshape(n, IN)
        run_case(f"edges_k{K}_f32", IL, n, IN, OUT, K, x, 80 + K, 81 + K, 82 + K, bias_scale=0.5)
        xb = x.to(torch.bfloat16)
        run_case(f"edges_k{K}_bf16", IL, n, IN, OUT, K, xb, 90 + K, 91 + K, 92 + K, bias_scale=0.5)

    # bit-exact bin sweeps (no gradients): dense values around the edges for several K
    for K in (3, 7, 16, 100, 128, 512):
        bw = 2.0 / K
        gen = torch.Generator().manual_seed(100 + K)
        edges = torch.arange(K + 1, dtype=torch.float32) * bw + (-1)
        offs = torch.tensor([-3e-7, -1.2e-7, -6e-8, 0.0, 6e-8, 1.2e-7, 3e-7], dtype=torch.float32)
        near = (edges[:, None] + offs[None, :]).reshape(-1)
        uni = torch.rand(4096, generator=gen) * 2.2 - 1.1
        special = torch.tensor([float("inf"), float("-inf"), float("nan"), 1e30, -1e30, 3e19, -3e19, 1e19])
        xf = torch.cat([near, uni, special]).reshape(1, -1)
        lo, hi, fr = ref_bins(xf, K, bw)
        xb = torch.cat([near, uni]).to(torch.bfloat16).reshape(1, -1)
        lob, hib, frb = ref_bins(xb, K, bw)
        np.savez_compressed(os.path.join(HERE, f"bins_k{K}.npz"), K=np.int64(K), bw=np.float64(bw),
                            x_f32=_bits(xf), lo_f32=lo.numpy(), fr_f32=_bits(fr),
                            x_bf16=_bits(xb), lo_bf16=lob.numpy(), fr_bf16=_bits(frb))
        print(f"bins_k{K}: {xf.numel()} f32 + {xb.numel()} bf16 values")


if __name__ == "__main__":
    main()
