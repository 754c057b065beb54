"""il_attention_forward / il_attention_backward (IndexedGPT's narrow-head
causal attention) against the reference's explicit formulation
(transformer_validation.py:264-267): without dropout, and with dropout using
the mask il_attention_dropout_mask reports for the same seed."""
import math

import pytest
import torch
import torch.nn.functional as F

from golden_io import normwise_close

from aiwn_b200 import _lib
from aiwn_b200.gpt import _AttentionFn

pytestmark = pytest.mark.gpu

DEV = "cuda"
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4


def _explicit(q, k, v, H, keep=None, p=0.0):
    """softmax(mask(q k^T / sqrt(D))) [* keep / (1-p)] v on [B, T, H*D] tensors."""
    B, T, C = q.shape
    D = C // H
    qh, kh, vh = (t.view(B, T, H, D).transpose(1, 2) for t in (q, k, v))
    att = (qh @ kh.transpose(-2, -1)) * (1.0 / math.sqrt(D))
    mask = torch.tril(torch.ones(T, T, device=q.device)).view(1, 1, T, T)
    att = F.softmax(att.masked_fill(mask == 0, float("-inf")), dim=-1)
    if keep is not None:
        att = att * keep.float() / (1.0 - p)
    return (att @ vh).transpose(1, 2).contiguous().view(B, T, C)


def _inputs(B, T, H, D, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(B, T, H * D, generator=g).to(DEV) for _ in range(4))
    return q, k, v, do


@pytest.mark.parametrize("shape", [(3, 256, 4, 4), (2, 77, 2, 8), (1, 300, 1, 16), (2, 64, 8, 2), (1, 1, 3, 4)],
                         ids=["config5_head", "odd_T_d8", "d16", "d2", "single_position"])
@pytest.mark.parametrize("p", [0.0, 0.3], ids=["no_dropout", "dropout"])
def test_attention_matches_explicit(shape, p):
    B, T, H, D = shape
    q, k, v, do = _inputs(B, T, H, D, seed=T + D)
    seed = torch.tensor([123456789 + T], dtype=torch.int64, device=DEV)
    keep = None
    if p > 0:
        keep = torch.empty(B, H, T, T, dtype=torch.uint8, device=DEV)
        _lib.attention_dropout_mask(keep, B, T, H, p, seed)
        frac = keep.float().mean().item()
        assert abs(frac - (1 - p)) < 0.05 or B * H * T * T < 1000
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    oa = _AttentionFn.apply(qa, ka, va, H, p, seed)
    oa.backward(do)
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    orf = _explicit(qr, kr, vr, H, keep, p)
    orf.backward(do)
    torch.cuda.synchronize()
    normwise_close(oa.detach().cpu().numpy(), orf.detach().cpu().numpy(), FWD_RTOL, "o")
    for name, a, r in (("dq", qa, qr), ("dk", ka, kr), ("dv", va, vr)):
        got, ref = a.grad.cpu().numpy(), r.grad.cpu().numpy()
        if not ref.any():
            # zero in exact arithmetic (e.g. dq over a single position): rounding noise only
            assert abs(got).max() < 1e-6, name
            continue
        normwise_close(got, ref, GRAD_RTOL, name)


def test_dropout_masks_differ_by_seed_and_repeat_for_a_seed():
    B, T, H = 2, 64, 2
    s1 = torch.tensor([5], dtype=torch.int64, device=DEV)
    s2 = torch.tensor([6], dtype=torch.int64, device=DEV)
    m1, m1b, m2 = (torch.empty(B, H, T, T, dtype=torch.uint8, device=DEV) for _ in range(3))
    _lib.attention_dropout_mask(m1, B, T, H, 0.1, s1)
    _lib.attention_dropout_mask(m1b, B, T, H, 0.1, s1)
    _lib.attention_dropout_mask(m2, B, T, H, 0.1, s2)
    assert torch.equal(m1, m1b)
    assert not torch.equal(m1, m2)
