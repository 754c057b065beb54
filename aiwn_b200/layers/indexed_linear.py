"""IndexedLinear on B200 -- drop-in for ``aiwn.layers.indexed_linear``.

Same public surface as the reference module (aiwn/layers/indexed_linear.py):

* ``IndexedLinear(in_d, out_d, K)`` with attributes ``K, bw, in_dim, out_dim,
  table[K, in_d, out_d], bias[out_d]`` and the same initialisation
  (IL:162-171), ``forward`` flattening all leading dimensions (IL:184-191),
  ``flops()`` and ``active_bytes()`` (IL:193-197);
* ``_Fn`` -- the ``torch.autograd.Function`` with the reference's
  ``apply(x, tab, bias, bw)`` signature and 4-tuple backward (IL:100-151);
* ``indexed_dims``, ``indexed_lr``, ``triton_available``, ``TRITON_OK``
  (IL:200-213, IL:18).  ``TRITON_OK`` keeps its name because callers import
  it (aiwn/bench/timing.py:10, aiwn/config.py:25); here it means "the sm_100a
  kernels of libaiwn_il.so are loaded".  No Triton is involved.

The arithmetic is the reference's eager path (IL:173-182) and autograd's
backward of it, computed by the hand-written CUDA kernels behind the C ABI
(include/aiwn_il.h).  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import _lib

TRITON_OK = _lib.available()


class _Fn(torch.autograd.Function):
    """out = IndexedLinear(x) for x[N, IN] (contiguous), tab[K, IN, OUT],
    bias[OUT]; returns fp32 out[N, OUT].  Mirrors aiwn/layers/indexed_linear.py:100-151.
    """

    @staticmethod
    def forward(ctx, x, tab, bias, bw):
        if x.dim() != 2 or tab.dim() != 3 or tab.shape[1] != x.shape[1]:
            raise ValueError(f"_Fn: x {tuple(x.shape)} and table {tuple(tab.shape)} do not match")
        x = x.contiguous()
        tab = tab.contiguous()
        bias = bias.contiguous()
        out = torch.empty(x.shape[0], tab.shape[2], dtype=torch.float32, device=x.device)
        _lib.forward(x, tab, bias, out, bw)
        ctx.save_for_backward(x, tab)
        ctx.bw = bw
        return out

    @staticmethod
    def backward(ctx, go):
        x, tab = ctx.saved_tensors
        go = go.contiguous()
        if go.dtype != torch.float32:
            go = go.float()
        need_x, need_t, need_b = ctx.needs_input_grad[:3]
        gx = torch.empty_like(x) if need_x else None
        gt, gb = grad_pair(tab.shape, (tab.shape[2],), x.device, need_t, need_b)
        if gx is None and gt is None and gb is None:
            return None, None, None, None
        N, IN = x.shape
        K, _, OUT = tab.shape
        ws_n = _lib.workspace_bytes(N, IN, OUT, K, _lib.x_dtype_code(x))
        ws = torch.empty(ws_n, dtype=torch.uint8, device=x.device) if ws_n > 0 else None
        _lib.backward(go, x, tab, gx, gt, gb, ctx.bw, ws)
        return gx, gt, gb, None


class _FnCounts(_Fn):
    """_Fn whose forward also adds the bin occupancy of x into ``counts``
    (int64 [K] on the device) -- the BucketTracker path.  Same backward."""

    @staticmethod
    def forward(ctx, x, tab, bias, bw, counts):
        if x.dim() != 2 or tab.dim() != 3 or tab.shape[1] != x.shape[1]:
            raise ValueError(f"_Fn: x {tuple(x.shape)} and table {tuple(tab.shape)} do not match")
        x = x.contiguous()
        tab = tab.contiguous()
        bias = bias.contiguous()
        out = torch.empty(x.shape[0], tab.shape[2], dtype=torch.float32, device=x.device)
        _lib.forward(x, tab, bias, out, bw, counts=counts)
        ctx.save_for_backward(x, tab)
        ctx.bw = bw
        return out

    @staticmethod
    def backward(ctx, go):
        return (*_Fn.backward(ctx, go), None)


def grad_pair(shape_a, shape_b, device, need_a: bool, need_b: bool):
    """Two fp32 gradient outputs (None where not needed).  When both are
    needed they share one allocation with b right after a, so the library
    zeroes them with one memset instead of two."""
    na, nb = math.prod(shape_a), math.prod(shape_b)
    if need_a and need_b:
        buf = torch.empty(na + nb, dtype=torch.float32, device=device)
        return buf[:na].view(shape_a), buf[na:].view(shape_b)
    a = torch.empty(shape_a, dtype=torch.float32, device=device) if need_a else None
    b = torch.empty(shape_b, dtype=torch.float32, device=device) if need_b else None
    return a, b


class IndexedLinear(nn.Module):
    """Input-indexed linear layer with a K-bucket interpolated weight table."""

    def __init__(self, in_d: int, out_d: int, K: int):
        super().__init__()
        assert K >= 2
        self.K = K
        self.bw = 2.0 / K
        self.in_dim = in_d
        self.out_dim = out_d
        std = math.sqrt(math.sqrt(3.0 / in_d) * (2.0 / K))
        self.table = nn.Parameter(torch.randn(K, in_d, out_d) * std)
        self.bias = nn.Parameter(torch.zeros(out_d))
        # int64 [K] device accumulator that eval-mode forwards add their bin
        # occupancy into (set by BucketTracker.register; None: no counting)
        self._bin_counts = None

    def _eager(self, x: torch.Tensor) -> torch.Tensor:
        """The reference's name for the flattened call (IL:173).  Here it runs
        the same CUDA kernels as ``forward``; CPU tensors raise."""
        return self._apply_fn(x)

    def _apply_fn(self, xf: torch.Tensor) -> torch.Tensor:
        if not xf.is_cuda:
            raise RuntimeError("aiwn_b200.IndexedLinear runs on CUDA (B200) only; got a CPU tensor")
        if not TRITON_OK:
            raise RuntimeError(f"libaiwn_il.so is not built ({_lib.library_path()})")
        counts = self._bin_counts
        if counts is not None and not self.training:
            if counts.device != xf.device:
                raise RuntimeError("the bin-count accumulator is on another device than the input")
            return _FnCounts.apply(xf, self.table, self.bias, self.bw, counts)
        return _Fn.apply(xf, self.table, self.bias, self.bw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, self.in_dim).contiguous()
        out = self._apply_fn(xf)
        return out.reshape(*shape[:-1], self.out_dim)

    def flops(self) -> int:
        return 2 * self.in_dim * self.out_dim

    def active_bytes(self) -> int:
        return 2 * self.in_dim * self.out_dim * 4

    def extra_repr(self) -> str:
        return f"in_dim={self.in_dim}, out_dim={self.out_dim}, K={self.K}"


def indexed_dims(d: int, ff: int, K: int, n_heads: int = 4):
    """(d_idx, ff_idx, h_dn) sizing, identical to aiwn/layers/indexed_linear.py:200-205."""
    s = math.sqrt(K)
    d_idx = max(n_heads, (int(d / s) // n_heads) * n_heads)
    ff_idx = 4 * d_idx
    h_dn = max(1, d_idx // max(1, int(round(s))))
    return d_idx, ff_idx, h_dn


def indexed_lr(base_lr: float, K: int) -> float:
    """Learning-rate scaling of aiwn/layers/indexed_linear.py:208-209."""
    return base_lr * math.sqrt(K / 2)


def triton_available() -> bool:
    """True when the B200 kernels are loaded (name kept from IL:212-213)."""
    return TRITON_OK
