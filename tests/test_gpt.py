"""IndexedGPT (transformer_validation.py:232-385) built on this package:
state_dict compatibility (CPU), numerics against the reference's own model
(tests/golden/gpt_small.npz, made by tests/golden/make_golden_gpt.py), and
the CUDA-graph training step against eager training (GPU)."""
import os

import numpy as np
import pytest
import torch

from golden_io import normwise_close

from aiwn_b200.buckets import BucketTracker
from aiwn_b200.gpt import GraphedTrainStep, IndexedGPT, get_d_idx

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gpt_small.npz")


def _golden():
    z = np.load(GOLD)
    return {k: z[k] for k in z.files}


def _model(d, dev, dropout=0.0):
    v, bs, nl, nh, ne, K = (int(a) for a in d["cfg"])
    m = IndexedGPT(v, bs, nl, nh, ne, K, dropout=dropout)
    sd = {k[len("param:"):]: torch.from_numpy(a) for k, a in d.items() if k.startswith("param:")}
    m.load_state_dict(sd)
    return m.to(dev)


def test_sizing_matches_reference_formula():
    assert get_d_idx(256, 128, 4) == (16, 8)  # config 5
    assert get_d_idx(64, 16, 4) == (16, 16)
    assert get_d_idx(256, 16, 4) == (64, 64)


def test_state_dict_matches_reference_model():
    d = _golden()
    v, bs, nl, nh, ne, K = (int(a) for a in d["cfg"])
    m = IndexedGPT(v, bs, nl, nh, ne, K, dropout=0.0)
    ours = {k: tuple(t.shape) for k, t in m.state_dict().items()}
    ref = {k[len("param:"):]: a.shape for k, a in d.items() if k.startswith("param:")}
    assert ours == ref


@pytest.mark.gpu
def test_forward_backward_match_reference():
    d = _golden()
    m = _model(d, "cuda")
    x = torch.from_numpy(d["x"]).cuda()
    y = torch.from_numpy(d["y"]).cuda()
    logits, loss = m(x, y)
    loss.backward()
    assert abs(loss.item() - float(d["loss"])) <= 1e-5 * abs(float(d["loss"]))
    normwise_close(logits.detach().cpu().numpy(), d["logits"], 1e-4, "logits")
    for name, p in m.named_parameters():
        got, ref = p.grad.cpu().numpy(), d["grad:" + name]
        if np.abs(ref).max() < 1e-7:
            # zero in exact arithmetic (the key bias: softmax ignores a constant
            # added to every key); both sides hold rounding noise only
            assert np.abs(got).max() < 1e-6, name
            continue
        normwise_close(got, ref, 1e-3, name)


@pytest.mark.gpu
def test_fused_attention_matches_explicit():
    """IndexedAttention's fused form and the reference's explicit masked
    softmax give the same loss and gradients without dropout."""
    d = _golden()
    x = torch.from_numpy(d["x"]).cuda()
    y = torch.from_numpy(d["y"]).cuda()
    m1 = _model(d, "cuda")
    m2 = _model(d, "cuda")
    for blk in m2.transformer["h"]:
        blk.attn.fused = False
    assert all(b.attn.fused for b in m1.transformer["h"])
    _, l1 = m1(x, y)
    _, l2 = m2(x, y)
    l1.backward()
    l2.backward()
    assert abs(l1.item() - l2.item()) <= 1e-5 * abs(l2.item())
    for (name, a), b in zip(m1.named_parameters(), m2.parameters()):
        ga, gb = a.grad.cpu().numpy(), b.grad.cpu().numpy()
        if np.abs(gb).max() < 1e-6:
            continue  # the key bias: zero in exact arithmetic
        normwise_close(ga, gb, 1e-4, name)


@pytest.mark.gpu
def test_graphed_train_step_matches_eager_training():
    d = _golden()
    x = torch.from_numpy(d["x"]).cuda()
    y = torch.from_numpy(d["y"]).cuda()
    bs = x.shape[1]
    eager = _model(d, "cuda")
    graphed = _model(d, "cuda")
    opt_e = torch.optim.AdamW(eager.parameters(), lr=1e-3, weight_decay=1e-2)
    opt_g = torch.optim.AdamW(graphed.parameters(), lr=1e-3, weight_decay=1e-2, capturable=True)
    step = GraphedTrainStep(graphed, opt_g, x.shape[0], bs)
    # construction leaves the model as it was
    for a, b in zip(eager.parameters(), graphed.parameters()):
        assert torch.equal(a, b)
    for it in range(3):
        xi, yi = torch.roll(x, it, 1), torch.roll(y, it, 1)
        opt_e.zero_grad()
        _, le = eager(xi, yi)
        le.backward()
        torch.nn.utils.clip_grad_norm_(eager.parameters(), 1.0)
        opt_e.step()
        lg = step(xi, yi)
        torch.cuda.synchronize()
        assert abs(lg.item() - le.item()) <= 1e-4 * abs(le.item())
    for (name, a), b in zip(eager.named_parameters(), graphed.parameters()):
        ref, got = a.detach().cpu().numpy(), b.detach().cpu().numpy()
        if np.abs(ref).max() < 1e-6:
            # driven only by rounding noise (the key bias's gradient is zero in
            # exact arithmetic, and Adam normalises whatever noise it gets)
            assert np.abs(got).max() < 1e-5, name
            continue
        # table gradients are sums in atomic order (not bitwise reproducible)
        # and Adam's first steps are ~lr * sign(g): entries whose gradient is
        # near zero can step differently, so 1e-3 normwise after three steps
        normwise_close(got, ref, 1e-3, name)


@pytest.mark.gpu
def test_bucket_tracker_on_indexed_gpt():
    d = _golden()
    m = _model(d, "cuda").eval()
    tr = BucketTracker(m.K)
    for layer in m.get_indexed_layers():
        tr.register(layer)
    with torch.no_grad():
        m(torch.from_numpy(d["x"]).cuda())
    x = torch.from_numpy(d["x"])
    n_tok = x.numel()
    # 6 tracked layers per block, in_dim inputs each
    expect = sum(n_tok * l.in_dim for l in m.get_indexed_layers())
    assert tr.counts.sum().item() == expect
    assert 0.0 < tr.entropy() <= 100.0
    tr.remove()
