"""Loading of the golden fixtures written by tests/golden/make_golden.py."""
from __future__ import annotations

import glob
import hashlib
import math
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def seeded_table(K: int, IN: int, OUT: int, seed: int) -> np.ndarray:
    """table ~ N(0, 1/IN) from a seeded CPU torch generator (same recipe as
    make_golden.py)."""
    t = torch.randn(K, IN, OUT, generator=torch.Generator().manual_seed(seed)) / math.sqrt(IN)
    return t.numpy().astype(np.float32)


def case_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if not os.path.basename(p).startswith(("bins_", "cdfnorm_", "gpt_")))


def bins_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "bins_*.npz")))


def load_case(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["K"] = int(d["K"])
    d["bw"] = float(d["bw"])
    d["x_dtype"] = str(d["x_dtype"])
    if "table_seed" in d:
        K, IN, OUT = (int(v) for v in d["table_shape"])
        t = seeded_table(K, IN, OUT, int(d["table_seed"]))
        h = hashlib.sha256(t.tobytes()).hexdigest()
        assert h == str(d["table_sha256"]), f"{name}: regenerated table does not match the fixture hash"
        d["table"] = t
    return d


def load_bins(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["K"] = int(d["K"])
    d["bw"] = float(d["bw"])
    return d


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def as_f32(a: np.ndarray) -> np.ndarray:
    return bf16_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


def normwise_close(got, ref, rtol: float, what: str = ""):
    """|got - ref| <= rtol * (|ref| + max|ref|) elementwise.

    The reference sums (over in_d, out_d or tokens) in fp32 in its own
    order; single elements near zero after cancellation carry absolute, not
    relative, rounding error, so the tolerance is taken relative to the
    element plus the tensor's largest magnitude."""
    got = as_f32(np.asarray(got))
    ref = as_f32(np.asarray(ref))
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    fin = np.isfinite(ref)
    assert np.array_equal(fin, np.isfinite(got)), f"{what}: non-finite pattern differs"
    if not fin.any():
        return 0.0
    g, r = got[fin].astype(np.float64), ref[fin].astype(np.float64)
    scale = np.abs(r).max()
    err = np.abs(g - r)
    bound = rtol * (np.abs(r) + scale) + 1e-30
    worst = float((err / bound).max())
    assert worst <= 1.0, f"{what}: max err {err.max():.3e} exceeds rtol {rtol} (ratio {worst:.2f}, scale {scale:.3e})"
    return float(err.max() / max(scale, 1e-30))


def same_bits(a, b) -> bool:
    """Bitwise equality of fp32 arrays, with every NaN equal to every NaN
    (the CPU propagates the input NaN's payload, the GPU returns the canonical
    NaN; both are NaN in the reference's sense)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))
