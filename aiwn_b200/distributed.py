"""Multi-GPU IndexedLinear: token parallelism and out_d column sharding.

The reference has no distributed code; this is the B200 node layout for the
layer (one process per GPU, NCCL over NVLink through ``torch.distributed``):

* ``TokenParallelIndexedLinear`` -- every rank holds the whole table and runs
  the layer on its own tokens (the forward needs no collective).  After the
  backward, ``sync_grads()`` all-reduces one contiguous fp32 bucket
  ``[table.grad | bias.grad]``: the table's gradient is the only exchange of
  data-parallel training.  Autograd accumulates the gradients directly into
  the bucket (``.grad`` are views of it), so the all-reduce needs no copies.
  On CUDA ranks of an NCCL group the bucket lives in symmetric memory and the
  library's own peer-memory kernel sums it (``exchange="peer"``, the default
  there: one launch, ~µs, against NCCL's ring/tree latency for this small
  bucket); ``exchange="nccl"`` uses ``dist.all_reduce``.

* ``ColumnShardedIndexedLinear`` -- for tables too large to replicate: rank r
  holds ``table[:, :, cols_r]`` (a contiguous slice of out_d) and computes
  ``y[:, cols_r]`` for all tokens; the full ``y`` is all-gathered.  In the
  backward the table gradient is local, and each rank's partial ``dx`` (its
  columns' contribution) is summed across ranks with an all-reduce.

Both run the same CUDA kernels as ``IndexedLinear`` on each rank.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn

from .layers.indexed_linear import IndexedLinear, _Fn


def token_shard(n_tokens: int, world: int, rank: int) -> slice:
    """Contiguous, balanced token range of `rank` (sizes differ by at most 1)."""
    base, rem = divmod(n_tokens, world)
    start = rank * base + min(rank, rem)
    return slice(start, start + base + (1 if rank < rem else 0))


def column_shard(out_d: int, world: int, rank: int) -> slice:
    """Contiguous, balanced out_d range of `rank`."""
    return token_shard(out_d, world, rank)


class TokenParallelIndexedLinear(nn.Module):
    """Data-parallel IndexedLinear: replicated table, tokens sharded by the
    caller (each rank feeds its own batch), one bucketed gradient all-reduce."""

    def __init__(self, in_d: int, out_d: int, K: int, group=None, average: bool = True,
                 layer: IndexedLinear | None = None, exchange: str = "auto"):
        super().__init__()
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError(f"exchange must be 'auto', 'peer' or 'nccl', not {exchange!r}")
        self.layer = layer if layer is not None else IndexedLinear(in_d, out_d, K)
        self.group = group
        self.average = average
        self.exchange = exchange
        self._bucket = None
        self._peer = None  # PeerBucket when the peer-memory exchange is in use

    @property
    def table(self):
        return self.layer.table

    @property
    def bias(self):
        return self.layer.bias

    def broadcast_parameters(self, src: int = 0):
        """Make every rank start from rank `src`'s table and bias."""
        with torch.no_grad():
            for p in (self.layer.table, self.layer.bias):
                dist.broadcast(p, src, group=self.group)

    def _use_peer(self, device) -> bool:
        if self.exchange == "nccl":
            return False
        from .comm import peer_exchange_available
        ok = peer_exchange_available(device, self.group)
        if self.exchange == "peer" and not ok:
            raise RuntimeError("exchange='peer' needs CUDA ranks of an NCCL group with symmetric memory")
        return ok

    def _ensure_bucket(self):
        t, b = self.layer.table, self.layer.bias
        n = t.numel() + b.numel()
        if self._bucket is None or self._bucket.numel() != n or self._bucket.device != t.device:
            self._peer = None
            if self._use_peer(t.device):
                from .comm import PeerBucket
                self._peer = PeerBucket(n, t.device, self.group)  # collective, zeroed
                self._bucket = self._peer.tensor
            else:
                self._bucket = torch.zeros(n, dtype=torch.float32, device=t.device)
        t.grad = self._bucket[: t.numel()].view_as(t)
        b.grad = self._bucket[t.numel():].view_as(b)
        return self._bucket

    def _grads_attached(self) -> bool:
        """True when table.grad and bias.grad are still the bucket's views."""
        bk = self._bucket
        if bk is None:
            return False
        t, b = self.layer.table, self.layer.bias
        return (t.grad is not None and b.grad is not None and t.grad.data_ptr() == bk.data_ptr()
                and b.grad.data_ptr() == bk.data_ptr() + t.numel() * bk.element_size())

    def zero_grad(self, set_to_none: bool = False):  # noqa: D401 - keeps the bucket alive
        """Zero the gradient bucket (the .grad tensors stay views of it)."""
        self._ensure_bucket().zero_()

    def forward(self, x):
        if not self._grads_attached():
            # First step, or an optimizer's zero_grad(set_to_none=True) (or
            # any other code) detached .grad from the bucket: the bucket holds
            # the previous step's sums, so it starts again from zero.
            self._ensure_bucket().zero_()
        return self.layer(x)

    def sync_grads(self, async_op: bool = False):
        """All-reduce [table.grad | bias.grad] as one buffer (sum, or mean
        over ranks when average=True).  Returns the work handle if async."""
        bucket = self._ensure_bucket() if self._bucket is None else self._bucket
        if self._peer is not None:
            world = dist.get_world_size(self.group)
            self._peer.all_reduce(1.0 / world if self.average else 1.0)
            return None
        op = dist.ReduceOp.AVG if (self.average and _avg_supported(bucket)) else dist.ReduceOp.SUM
        work = dist.all_reduce(bucket, op=op, group=self.group, async_op=async_op)
        if self.average and op == dist.ReduceOp.SUM:
            if async_op:
                work.wait()
            bucket.div_(dist.get_world_size(self.group))
            return None
        return work


def _avg_supported(t: torch.Tensor) -> bool:
    return t.is_cuda and dist.get_backend() == "nccl"


class _GatherColumns(torch.autograd.Function):
    """y_local [N, c_r] -> y [N, out_d] (all-gather along columns); the
    backward returns the local columns of the incoming gradient."""

    @staticmethod
    def forward(ctx, y_local, sizes, group):
        ctx.sizes, ctx.group = sizes, group
        rank = dist.get_rank(group)
        parts = [torch.empty(y_local.shape[0], s, dtype=y_local.dtype, device=y_local.device) for s in sizes]
        dist.all_gather(parts, y_local.contiguous(), group=group)
        ctx.start = sum(sizes[:rank])
        return torch.cat(parts, dim=1)

    @staticmethod
    def backward(ctx, gy):
        rank = dist.get_rank(ctx.group)
        return gy[:, ctx.start: ctx.start + ctx.sizes[rank]].contiguous(), None, None


class _SumDx(torch.autograd.Function):
    """Identity in the forward; all-reduces the input gradient (each rank
    holds the contribution of its own out_d columns)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, gx):
        gx = gx.contiguous()
        dist.all_reduce(gx, group=ctx.group)
        return gx, None


class ColumnShardedIndexedLinear(nn.Module):
    """IndexedLinear with out_d split across the ranks of `group`."""

    def __init__(self, in_d: int, out_d: int, K: int, group=None, gather_output: bool = True,
                 full_table: torch.Tensor | None = None, full_bias: torch.Tensor | None = None):
        super().__init__()
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.group, self.gather_output = group, gather_output
        self.in_dim, self.out_dim, self.K = in_d, out_d, K
        self.bw = 2.0 / K
        self.cols = column_shard(out_d, world, rank)
        self.sizes = [column_shard(out_d, world, r).stop - column_shard(out_d, world, r).start
                      for r in range(world)]
        c = self.cols.stop - self.cols.start
        if full_table is not None:
            t = full_table[:, :, self.cols].contiguous().clone()
        else:
            std = math.sqrt(math.sqrt(3.0 / in_d) * (2.0 / K))
            t = torch.randn(K, in_d, c) * std
        self.table = nn.Parameter(t)
        self.bias = nn.Parameter(full_bias[self.cols].clone() if full_bias is not None else torch.zeros(c))

    def forward(self, x):
        shape = x.shape
        xf = x.reshape(-1, self.in_dim).contiguous()
        if not xf.is_cuda:
            raise RuntimeError("ColumnShardedIndexedLinear runs on CUDA only")
        xf = _SumDx.apply(xf, self.group)
        y = _Fn.apply(xf, self.table, self.bias, self.bw)
        if self.gather_output:
            y = _GatherColumns.apply(y, self.sizes, self.group)
            return y.reshape(*shape[:-1], self.out_dim)
        return y.reshape(*shape[:-1], y.shape[-1])
