"""IndexedLinearV2 (GaussianCDFNorm prologue + IndexedLinear) on the GPU
against the oracle and the reference's golden vectors.

The prologue's xn matches the reference within XN_ATOL (erf and the
LayerNorm moments round differently).  Because the input gradient jumps at
bin boundaries, the IndexedLinear part and the prologue's backward are each
checked against the oracle run on this library's own xn and gxn (same bins);
the whole chain is then checked against the golden values.
"""
import os

import numpy as np
import pytest
import torch

from golden_io import normwise_close
from oracle import oracle

import aiwn_b200
from aiwn_b200 import IndexedLinearV2, _lib

pytestmark = pytest.mark.gpu

DEV = "cuda"
XN_ATOL = 1e-6
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4
CDF_CASES = ["cdfnorm_20x20_k64", "cdfnorm_16x8_k128"]


def _load(name):
    return dict(np.load(os.path.join(os.path.dirname(__file__), "golden", f"{name}.npz")))


def _random_case(N, IN, OUT, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, IN, generator=g) * 1.5 - 0.2
    gamma = 1.0 + 0.3 * torch.randn(IN, generator=g)
    beta = 0.2 * torch.randn(IN, generator=g)
    table = torch.randn(K, IN, OUT, generator=g) / IN ** 0.5
    bias = 0.1 * torch.randn(OUT, generator=g)
    go = torch.randn(N, OUT, generator=g)
    return dict(x=x.numpy(), gamma=gamma.numpy(), beta=beta.numpy(), table=table.numpy(), bias=bias.numpy(),
                go=go.numpy(), eps=1e-5, bw=2.0 / K, K=K)


def _run_kernels(d):
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for k, v in d.items() if isinstance(v, np.ndarray)}
    N, IN = t["x"].shape
    OUT = t["table"].shape[2]
    xn = torch.empty_like(t["x"])
    mean = torch.empty(N, device=DEV)
    rstd = torch.empty(N, device=DEV)
    out = torch.empty(N, OUT, device=DEV)
    _lib.cdf_forward(t["x"], t["gamma"], t["beta"], float(d["eps"]), t["table"], t["bias"], xn, mean, rstd, out,
                     float(d["bw"]))
    gxn = torch.empty_like(xn)
    gt = torch.empty_like(t["table"])
    gb = torch.empty(OUT, device=DEV)
    _lib.backward(t["go"], xn, t["table"], gxn, gt, gb, float(d["bw"]))
    dx = torch.empty_like(t["x"])
    dg = torch.empty_like(t["gamma"])
    db = torch.empty_like(t["beta"])
    _lib.cdf_backward(gxn, t["x"], t["gamma"], t["beta"], mean, rstd, dx, dg, db)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in dict(xn=xn, mean=mean, rstd=rstd, out=out, gxn=gxn, gt=gt, gb=gb,
                                                   dx=dx, dg=dg, db=db).items()}


def _check_against_oracle(d, r):
    eps, bw = float(d["eps"]), float(d["bw"])
    xn, mean, rstd = oracle.cdf_forward(d["x"], d["gamma"], d["beta"], eps)
    assert np.abs(r["xn"] - xn).max() <= XN_ATOL
    normwise_close(r["mean"], mean, 1e-6, "mean")
    normwise_close(r["rstd"], rstd, 1e-6, "rstd")
    # the IndexedLinear part on this library's xn: identical bins
    normwise_close(r["out"], oracle.forward(r["xn"], d["table"], d["bias"], bw), FWD_RTOL, "out")
    gxn, gt, gb = oracle.backward(d["go"], r["xn"], d["table"], bw)
    normwise_close(r["gxn"], gxn, GRAD_RTOL, "gxn")
    normwise_close(r["gt"], gt, GRAD_RTOL, "gt")
    normwise_close(r["gb"], gb, GRAD_RTOL, "gb")
    # the prologue's backward on this library's gxn
    dx, dg, db = oracle.cdf_backward(r["gxn"], d["x"], d["gamma"], d["beta"], eps)
    normwise_close(r["dx"], dx, GRAD_RTOL, "dx")
    normwise_close(r["dg"], dg, GRAD_RTOL, "dgamma")
    normwise_close(r["db"], db, GRAD_RTOL, "dbeta")


@pytest.mark.parametrize("path", ["auto", "cluster"])
@pytest.mark.parametrize("name", CDF_CASES)
def test_cdf_kernels_vs_golden_and_oracle(name, path, monkeypatch):
    """auto: the prologue fused into the token forward; cluster: the
    standalone prologue pass followed by the cluster forward on xn."""
    monkeypatch.setenv("AIWN_IL_FORWARD", path)
    d = _load(name)
    r = _run_kernels(d)
    _check_against_oracle(d, r)
    assert np.abs(r["xn"] - d["xn"]).max() <= XN_ATOL
    normwise_close(r["out"], d["out"], FWD_RTOL, "out vs reference")
    normwise_close(r["gt"], d["gt"], GRAD_RTOL, "gt vs reference")
    normwise_close(r["dx"], d["gx"], GRAD_RTOL, "dx vs reference")
    normwise_close(r["dg"], d["ggamma"], GRAD_RTOL, "dgamma vs reference")
    normwise_close(r["db"], d["gbeta"], GRAD_RTOL, "dbeta vs reference")


@pytest.mark.parametrize("shape", [(4096, 20, 20, 512), (2000, 40, 12, 64), (777, 7, 36, 16)],
                         ids=["c3_shape", "in40_unfused", "in7_out36"])
def test_cdf_kernels_vs_oracle_random(shape):
    """C3's shape (fused), in_d > 32 (standalone prologue) and an odd width."""
    N, IN, OUT, K = shape
    d = _random_case(N, IN, OUT, K, seed=N + IN)
    _check_against_oracle(d, _run_kernels(d))


def test_indexed_linear_v2_module_matches_kernels():
    """The module (autograd path, leading dims flattened) gives the kernels'
    values and fills every parameter's gradient."""
    d = _load("cdfnorm_20x20_k64")
    N, IN = d["x"].shape
    OUT = d["table"].shape[2]
    m = IndexedLinearV2(IN, OUT, int(d["K"])).to(DEV)
    with torch.no_grad():
        m.cdf.ln.weight.copy_(torch.from_numpy(d["gamma"]))
        m.cdf.ln.bias.copy_(torch.from_numpy(d["beta"]))
        m.linear.table.copy_(torch.from_numpy(d["table"]))
        m.linear.bias.copy_(torch.from_numpy(d["bias"]))
    x = torch.from_numpy(d["x"]).to(DEV).reshape(4, N // 4, IN).requires_grad_(True)
    y = m(x)
    assert y.shape == (4, N // 4, OUT)
    y.backward(torch.from_numpy(d["go"]).to(DEV).reshape(4, N // 4, OUT))
    r = _run_kernels(d)
    np.testing.assert_array_equal(y.detach().reshape(N, OUT).cpu().numpy(), r["out"])
    np.testing.assert_array_equal(x.grad.reshape(N, IN).cpu().numpy(), r["dx"])
    normwise_close(m.linear.table.grad.cpu().numpy(), r["gt"], 1e-6, "gt")
    normwise_close(m.cdf.ln.weight.grad.cpu().numpy(), r["dg"], 1e-6, "dgamma")
    normwise_close(m.cdf.ln.bias.grad.cpu().numpy(), r["db"], 1e-6, "dbeta")
    normwise_close(m.linear.bias.grad.cpu().numpy(), r["gb"], 1e-6, "dbias")
    assert aiwn_b200.GaussianCDFNorm is type(m.cdf)
