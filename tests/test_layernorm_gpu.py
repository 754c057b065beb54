"""il_layernorm_forward / il_layernorm_backward (the IndexedGPT blocks'
LayerNorm for d <= 32) against torch.nn.functional.layer_norm and autograd,
fp32, including widths that are not a multiple of 4 (scalar loads)."""
import pytest
import torch
import torch.nn.functional as F

from golden_io import normwise_close

from aiwn_b200.gpt import _LayerNormFn, layer_norm

pytestmark = pytest.mark.gpu

DEV = "cuda"
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4


@pytest.mark.parametrize("d", [16, 8, 20, 32, 7, 1])
def test_layernorm_matches_torch(d):
    g = torch.Generator().manual_seed(d)
    N = 5003
    x = (torch.randn(N, d, generator=g) * 1.7 + 0.4).to(DEV)
    w = (1.0 + 0.3 * torch.randn(d, generator=g)).to(DEV)
    b = (0.2 * torch.randn(d, generator=g)).to(DEV)
    gy = torch.randn(N, d, generator=g).to(DEV)
    eps = 1e-5

    xa, wa, ba = (t.clone().requires_grad_(True) for t in (x, w, b))
    ya = _LayerNormFn.apply(xa, wa, ba, eps)
    ya.backward(gy)
    xr, wr, br = (t.clone().requires_grad_(True) for t in (x, w, b))
    yr = F.layer_norm(xr, (d,), wr, br, eps)
    yr.backward(gy)
    torch.cuda.synchronize()
    normwise_close(ya.detach().cpu().numpy(), yr.detach().cpu().numpy(), FWD_RTOL, "y")
    normwise_close(xa.grad.cpu().numpy(), xr.grad.cpu().numpy(), GRAD_RTOL, "dx")
    normwise_close(wa.grad.cpu().numpy(), wr.grad.cpu().numpy(), GRAD_RTOL, "dgamma")
    normwise_close(ba.grad.cpu().numpy(), br.grad.cpu().numpy(), GRAD_RTOL, "dbeta")


def test_layer_norm_helper_dispatch():
    """3-D input through the module helper; wide rows keep torch's LayerNorm."""
    ln = torch.nn.LayerNorm(16).to(DEV)
    x = torch.randn(4, 33, 16, device=DEV, requires_grad=True)
    y = layer_norm(ln, x)
    assert y.grad_fn is not None and "LayerNormFn" in type(y.grad_fn).__name__
    normwise_close(y.detach().cpu().numpy(), ln(x).detach().cpu().numpy(), FWD_RTOL, "y 3-D")
    wide = torch.nn.LayerNorm(64).to(DEV)
    xw = torch.randn(8, 64, device=DEV)
    assert "LayerNormFn" not in type(layer_norm(wide, xw.requires_grad_(True)).grad_fn).__name__
