"""The CPU oracle against the golden vectors produced by the reference.

Bins are bit-exact; forward within 1e-5 and fp32 gradients within 1e-4
(normwise), bf16 gradients within 2e-2.
"""
import numpy as np
import pytest

from golden_io import bins_names, case_names, load_bins, load_case, normwise_close, same_bits
from oracle import oracle

FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4
BF16_RTOL = 2e-2


@pytest.mark.parametrize("name", bins_names())
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_oracle_bins_bit_exact(name, dt):
    d = load_bins(name)
    x = d[f"x_{dt}"]
    lo, _, fr = oracle.bins(x, d["K"], d["bw"], x_dtype=dt)
    assert np.array_equal(lo, d[f"lo_{dt}"])
    assert same_bits(fr, d[f"fr_{dt}"])


@pytest.mark.parametrize("name", case_names())
def test_oracle_case(name):
    d = load_case(name)
    dt, K, bw = d["x_dtype"], d["K"], d["bw"]
    lo, hi, fr = oracle.bins(d["x"], K, bw, x_dtype=dt)
    assert np.array_equal(lo, d["lo"]) and np.array_equal(hi, d["hi"])
    assert same_bits(fr, d["fr"])
    out = oracle.forward(d["x"], d["table"], d["bias"], bw, x_dtype=dt)
    normwise_close(out, d["out"], FWD_RTOL, "out")
    gx, gt, gb = oracle.backward(d["go"], d["x"], d["table"], bw, x_dtype=dt)
    normwise_close(gx, d["gx"], BF16_RTOL if dt == "bf16" else GRAD_RTOL, "gx")
    normwise_close(gt, d["gt"], GRAD_RTOL, "gt")
    normwise_close(gb, d["gb"], GRAD_RTOL, "gb")


def test_oracle_threads_deterministic():
    d = load_case("c3_small")
    a = oracle.forward(d["x"], d["table"], d["bias"], d["bw"], nthreads=1)
    b = oracle.forward(d["x"], d["table"], d["bias"], d["bw"], nthreads=4)
    assert np.array_equal(a, b)
    g1 = oracle.backward(d["go"], d["x"], d["table"], d["bw"], nthreads=1)
    g4 = oracle.backward(d["go"], d["x"], d["table"], d["bw"], nthreads=4)
    for u, v in zip(g1, g4):
        assert np.array_equal(u, v)


# ---- IndexedLinearV2: the GaussianCDFNorm prologue ---------------------------

CDF_CASES = ["cdfnorm_20x20_k64", "cdfnorm_16x8_k128"]
XN_ATOL = 1e-6  # LayerNorm moments and erf round differently from ATen's (measured max 2.4e-7)


def load_cdf(name):
    import os
    return dict(np.load(os.path.join(os.path.dirname(__file__), "golden", f"{name}.npz")))


@pytest.mark.parametrize("name", CDF_CASES)
def test_oracle_cdfnorm_chain(name):
    """Prologue, IndexedLinear on xn and the prologue's backward, each against
    the reference's own values (tests/golden/make_golden_cdfnorm.py)."""
    d = load_cdf(name)
    eps, bw = float(d["eps"]), float(d["bw"])
    xn, _, _ = oracle.cdf_forward(d["x"], d["gamma"], d["beta"], eps)
    assert np.abs(xn - d["xn"]).max() <= XN_ATOL
    normwise_close(oracle.forward(d["xn"], d["table"], d["bias"], bw), d["out"], FWD_RTOL, "out")
    gxn, gt, gb = oracle.backward(d["go"], d["xn"], d["table"], bw)
    normwise_close(gxn, d["gxn"], GRAD_RTOL, "gxn")
    normwise_close(gt, d["gt"], GRAD_RTOL, "gt")
    normwise_close(gb, d["gb"], GRAD_RTOL, "gb")
    dx, dg, db = oracle.cdf_backward(d["gxn"], d["x"], d["gamma"], d["beta"], eps)
    normwise_close(dx, d["gx"], GRAD_RTOL, "dx")
    normwise_close(dg, d["ggamma"], GRAD_RTOL, "dgamma")
    normwise_close(db, d["gbeta"], GRAD_RTOL, "dbeta")
