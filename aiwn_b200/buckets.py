"""Bin-occupancy tracking on the GPU -- drop-in for the reference's
``BucketTracker`` (transformer_validation.py:92-123) and
``get_bucket_counts`` (aiwn/experiments/bucket_analysis.py:33-51).

The reference copies every tracked activation to the host and runs
``torch.bincount`` there.  Here the counts are the library's bit-exact bins,
counted in shared memory on the device and added into a 64-bit device
accumulator.  For this package's IndexedLinear the forward kernel itself
counts while it bins (``il_forward_counts``: the layer's eval-mode forwards
add into the tracker's accumulator); other modules get a forward pre-hook
that runs ``il_bin_counts`` on their input.  ``counts`` / ``entropy()`` read
the accumulator back when asked.
"""
from __future__ import annotations

import math

import torch

from . import _lib


class BucketTracker:
    """Counts the bins of the inputs of registered IndexedLinear layers during
    eval-mode forwards.  Same methods and attributes as the reference."""

    def __init__(self, K):
        self.K = K
        self._acc = {}  # device -> int64 [K]
        self.handles = []
        self._fused = []  # IndexedLinear layers that count in their forward kernel

    def _dev_counts(self, dev):
        acc = self._acc.get(dev)
        if acc is None:
            acc = torch.zeros(self.K, dtype=torch.int64, device=dev)
            self._acc[dev] = acc
        return acc

    @property
    def counts(self) -> torch.Tensor:
        """Float CPU tensor [K] of hits per bin, as the reference keeps it."""
        total = torch.zeros(self.K, dtype=torch.float32)
        for acc in self._acc.values():
            total += acc.float().cpu()
        return total

    def reset(self):
        for acc in self._acc.values():
            acc.zero_()

    def register(self, layer):
        from .layers.indexed_linear import IndexedLinear
        if isinstance(layer, IndexedLinear) and layer.K == self.K and layer.table.is_cuda:
            # the layer's forward kernel adds into the accumulator itself
            layer._bin_counts = self._dev_counts(layer.table.device)
            self._fused.append(layer)
            return

        def hook(module, args):
            if not module.training:
                xf = args[0].reshape(-1, module.in_dim).detach()
                _lib.bin_counts(xf.contiguous(), self.K, 2.0 / self.K, self._dev_counts(xf.device))
        self.handles.append(layer.register_forward_pre_hook(hook))

    def entropy(self):
        c = self.counts
        total = c.sum()
        if total == 0:
            return 0.0
        p = c / total
        return -(p * (p + 1e-10).log()).sum().item() / math.log(self.K) * 100

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles.clear()
        for layer in self._fused:
            layer._bin_counts = None
        self._fused.clear()


def get_bucket_counts(layer, x: torch.Tensor, K: int) -> torch.Tensor:
    """Hits per bin (float tensor [K] on x's device) of one forward's inputs to
    ``layer``, over all samples and input dimensions; for an IndexedLinearV2
    the bins are those of its GaussianCDFNorm output."""
    with torch.no_grad():
        in_d = getattr(layer, "in_d", None) or getattr(layer, "in_dim", None) or layer.linear.in_dim
        xf = x.reshape(-1, in_d)
        if hasattr(layer, "cdf"):
            xf = layer.cdf(xf)
        counts = torch.zeros(K, dtype=torch.int64, device=xf.device)
        _lib.bin_counts(xf.contiguous(), K, 2.0 / K, counts)
        return counts.float()
