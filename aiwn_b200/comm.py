"""Gradient exchange over NVLink peer memory for token-parallel training.

``PeerBucket`` is an fp32 buffer of n elements in torch symmetric memory: it
is mapped into every rank's address space, so the library's
``il_allreduce_sum`` kernel can sum it across the GPUs of the node in place
in one launch (for buffers of up to 2^21 elements every value travels to the
reducing rank and back with its call's flag in one 64-bit word, so no fence
or barrier is needed; larger buffers take peer loads and stores between
per-block flag barriers).  The kernel's scratch region (flags and staging
words) follows the data in the same allocation.

    bucket = PeerBucket(n, device, group)   # collective: every rank, same n
    bucket.tensor                            # [n] fp32, this rank's buffer
    bucket.all_reduce(scale=1.0)             # in place, on the current stream

The reference trains on one device; this is the exchange step that
token-parallel training adds (the table and bias gradients of
aiwn/layers/indexed_linear.py:131-151, summed over the ranks' tokens).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def peer_exchange_available(device: torch.device, group=None) -> bool:
    """Whether the peer-memory all-reduce can serve this process group: CUDA
    tensors, an NCCL group and symmetric memory in this torch build.  Every
    rank evaluates the same conditions."""
    if device.type != "cuda" or not dist.is_initialized():
        return False
    if dist.get_backend(group) != "nccl":
        return False
    if dist.get_world_size(group) > 16:
        return False
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except ImportError:
        return False
    return True


class PeerBucket:
    """n fp32 elements in symmetric memory, all-reduced by il_allreduce_sum."""

    def __init__(self, n: int, device, group=None, timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem
        self.n = int(n)
        self.device = torch.device(device)
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.timeout_s = float(timeout_s)
        n_pad = (self.n + 63) // 64 * 64  # the scratch region starts 256-byte aligned
        scratch_words = (_lib.allreduce_scratch_bytes(self.n, self.world) + 3) // 4
        self._raw = symm_mem.empty(n_pad + scratch_words, dtype=torch.float32, device=self.device)
        self._raw.zero_()  # flags and generation counters start at 0 on every rank
        self._handle = symm_mem.rendezvous(self._raw, self.group)
        torch.cuda.synchronize(self.device)
        # every rank's flags are zero before any rank's first signal
        dist.barrier(group=self.group, device_ids=[self.device.index])
        self.tensor = self._raw[: self.n]
        ptrs = [int(p) for p in self._handle.buffer_ptrs]
        off = self._raw.data_ptr() - ptrs[self.rank]  # the same offset in every rank's mapping
        self.bufs = [p + off for p in ptrs]
        self.scratch = [p + off + n_pad * 4 for p in ptrs]
        self._call = _lib.allreduce_caller(self.bufs, self.scratch, self.n, self.rank, self.world, self.timeout_s,
                                           self.device)

    def all_reduce(self, scale: float = 1.0):
        """tensor <- scale * (sum of every rank's tensor), in place, enqueued
        on the current stream (no host synchronisation)."""
        self._call(scale)
