"""The library against the reference's own CUDA extension on the GPU.

`aiwn/layers/indexed_linear_cuda.cu` (the reference's fp32 extension) is
built for sm_100a into baseline/_ref/ by baseline/build_ref_cuda.py; these
tests skip when it is not there.  On inputs in [-1, 1) its bins and
fractions are computed with the same fp32 operations as the reference's eager
path, so forward and table gradient agree.  Its dx keeps the slope term where
the fraction was clamped to [0, 1] (the eager path, followed here, drops it;
cu:117-130 against IL:175-182), so tokens with a clamped fraction are left
out of the dx comparison.
"""
import importlib.util
import os

import numpy as np
import pytest
import torch

from golden_io import normwise_close

from aiwn_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda"
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4
SO = os.path.join(os.path.dirname(__file__), "..", "baseline", "_ref", "indexed_linear_cuda.so")


def _ref_module():
    if not os.path.exists(SO):
        pytest.skip("reference CUDA extension not built (python baseline/build_ref_cuda.py)")
    spec = importlib.util.spec_from_file_location("indexed_linear_cuda", SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _clamped_tokens(x: np.ndarray, K: int, bw: float) -> np.ndarray:
    """Tokens with at least one element whose raw fraction lies outside [0, 1]."""
    f1, fbw = np.float32(1.0), np.float32(bw)
    lo = np.clip(np.trunc((x + f1) / fbw), 0, K - 1).astype(np.float32)
    fr = (x - (np.float32(-1.0) + lo * fbw)) / fbw
    return ((fr < 0) | (fr > 1)).any(axis=1)


@pytest.mark.parametrize("shape", [(8192, 20, 20, 512), (2048, 64, 64, 16), (777, 7, 36, 64)],
                         ids=["c3_shape", "c1_shape", "odd"])
def test_matches_reference_cuda_extension(shape):
    ref = _ref_module()
    N, IN, OUT, K = shape
    bw = 2.0 / K
    g = torch.Generator().manual_seed(N + IN + K)
    x = torch.rand(N, IN, generator=g) * 2 - 1  # [-1, 1): the reference kernels' valid range
    table = torch.randn(K, IN, OUT, generator=g) / IN ** 0.5
    bias = 0.1 * torch.randn(OUT, generator=g)
    go = torch.randn(N, OUT, generator=g)
    xd, td, bd, gd = (t.to(DEV) for t in (x, table, bias, go))

    out = torch.empty(N, OUT, device=DEV)
    _lib.forward(xd, td, bd, out, bw)
    gx = torch.empty_like(xd)
    gt = torch.empty_like(td)
    gb = torch.empty(OUT, device=DEV)
    _lib.backward(gd, xd, td, gx, gt, gb, bw)
    r_out = ref.forward(xd, td, bd, bw)
    r_gx, r_gt = ref.backward(gd, xd, td, bw)
    torch.cuda.synchronize()

    normwise_close(out.cpu().numpy(), r_out.cpu().numpy(), FWD_RTOL, "out vs reference CUDA")
    normwise_close(gt.cpu().numpy(), r_gt.cpu().numpy(), GRAD_RTOL, "gt vs reference CUDA")
    keep = ~_clamped_tokens(x.numpy(), K, bw)
    assert keep.mean() > 0.99
    normwise_close(gx.cpu().numpy()[keep], r_gx.cpu().numpy()[keep], GRAD_RTOL, "gx vs reference CUDA")
    np.testing.assert_allclose(gb.cpu().numpy(), go.sum(0).numpy(), rtol=1e-4, atol=1e-4)
