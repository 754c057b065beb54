"""Torch restatement of the reference's CPU path -- TEST/BENCH INFRASTRUCTURE ONLY.

``IndexedLinear._eager`` (aiwn/layers/indexed_linear.py:173-182) is the
reference's ``--device cpu`` implementation.  Its steps are restated here
with the same ATen operations (so the host cores do the same work the
reference does on CPU), and ``eager_step`` adds autograd's backward, as the
reference's own step benchmark does (aiwn/bench/timing.py:65-72).

Only ``bench.py`` (its ``--impl reference`` arm and ``cpu_baseline`` leg)
uses this module, to time the reference's CPU path beside the GPU kernels.
The parity checker is the C oracle (``oracle/il_oracle.c``).
"""
from __future__ import annotations

import math

import torch


def eager_forward(x: torch.Tensor, table: torch.Tensor, bias: torch.Tensor, bw: float) -> torch.Tensor:
    K = table.shape[0]
    N, IN = x.shape
    lo = ((x + 1) / bw).long().clamp(0, K - 1)
    hi = (lo + 1).clamp(max=K - 1)
    fr = ((x - (-1 + lo.float() * bw)) / bw).clamp(0, 1)
    cols = torch.arange(IN, device=x.device).unsqueeze(0).expand(N, -1)
    w = table[lo, cols] * (1 - fr.unsqueeze(-1)) + table[hi, cols] * fr.unsqueeze(-1)
    return (w * x.unsqueeze(-1)).sum(1) + bias


def eager_step(x, table, bias, go, bw):
    """fwd + bwd of the eager path: returns (out, gx, gt, gb)."""
    xl = x.detach().requires_grad_(True)
    tl = table.detach().requires_grad_(True)
    bl = bias.detach().requires_grad_(True)
    out = eager_forward(xl, tl, bl, bw)
    out.backward(go)
    return out.detach(), xl.grad, tl.grad, bl.grad


def eager_cdf_norm(x, gamma, beta, eps):
    """GaussianCDFNorm.forward (aiwn/layers/indexed_linear_v2.py:33-36), same ATen ops."""
    z = torch.nn.functional.layer_norm(x, (x.shape[-1],), gamma, beta, eps)
    u = 0.5 * (1.0 + torch.erf(z / math.sqrt(2.0)))
    return u * 2.0 - 1.0


def eager_step_v2(x, gamma, beta, eps, table, bias, go, bw):
    """fwd + bwd of IndexedLinearV2's CPU path (prologue, then _eager)."""
    xl = x.detach().requires_grad_(True)
    gl = gamma.detach().requires_grad_(True)
    bl_ = beta.detach().requires_grad_(True)
    tl = table.detach().requires_grad_(True)
    bl = bias.detach().requires_grad_(True)
    out = eager_forward(eager_cdf_norm(xl, gl, bl_, eps), tl, bl, bw)
    out.backward(go)
    return out.detach(), xl.grad, tl.grad, bl.grad


def eager_indexed_gpt(model):
    """Turn an ``aiwn_b200.gpt.IndexedGPT`` into the reference's CPU model: every
    IndexedLinear runs ``_eager``'s ATen ops (``eager_forward``) and the FFN
    takes its unfused ``up(cdf(x))`` route (GaussianCDFNorm is already the
    reference's own two ATen ops).  For the timed CPU baseline only."""
    import torch.nn as nn

    from aiwn_b200.layers import IndexedLinear

    class _EagerIL(IndexedLinear):
        def forward(self, x):
            shape = x.shape
            out = eager_forward(x.reshape(-1, self.in_dim), self.table, self.bias, self.bw)
            return out.reshape(*shape[:-1], self.out_dim)

    for m in model.modules():
        if isinstance(m, IndexedLinear):
            m.__class__ = _EagerIL
    for blk in model.transformer["h"]:
        blk.ffn.up.register_forward_pre_hook(lambda mod, args: None)  # selects the unfused route
    assert isinstance(model, nn.Module)
    return model
