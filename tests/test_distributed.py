"""Multi-rank plumbing of aiwn_b200.distributed, as gloo ranks on CPU.

The layer kernels run on CUDA only, so these tests give each rank a CPU
stand-in for the per-rank compute (the reference's eager ops, from the
oracle's torch port) and check the collectives around it: the bucketed
gradient all-reduce of token parallelism, and the column-sharded forward
(all-gather) and backward (dx all-reduce, local table gradient).
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from oracle.eager_port import eager_forward

import aiwn_b200.distributed as D
from aiwn_b200.distributed import (ColumnShardedIndexedLinear, TokenParallelIndexedLinear,
                                   column_shard, token_shard)


def test_token_and_column_shards_cover_exactly():
    for n in (0, 1, 7, 131072, 131073):
        for w in (1, 2, 3, 8):
            parts = [token_shard(n, w, r) for r in range(w)]
            assert parts[0].start == 0 and parts[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1
    assert column_shard(1024, 8, 3) == slice(384, 512)


class _CPULayer(nn.Module):
    """Stand-in for IndexedLinear's per-rank compute: same parameters, eager ops."""

    def __init__(self, IN, OUT, K, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.K, self.bw, self.in_dim, self.out_dim = K, 2.0 / K, IN, OUT
        self.table = nn.Parameter(torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN))
        self.bias = nn.Parameter(torch.randn(OUT, generator=g) * 0.1)

    def forward(self, x):
        return eager_forward(x.reshape(-1, self.in_dim), self.table, self.bias, self.bw)


class _EagerFn(torch.autograd.Function):
    """CPU stand-in for _Fn (same signature), used by the column-shard test."""

    @staticmethod
    def forward(ctx, x, tab, bias, bw):
        with torch.enable_grad():
            xl = x.detach().requires_grad_(True)
            tl = tab.detach().requires_grad_(True)
            bl = bias.detach().requires_grad_(True)
            out = eager_forward(xl, tl, bl, bw)
        ctx.saved = (xl, tl, bl, out)
        return out.detach()

    @staticmethod
    def backward(ctx, go):
        xl, tl, bl, out = ctx.saved
        gx, gt, gb = torch.autograd.grad(out, (xl, tl, bl), go)
        return gx, gt, gb, None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _token_parallel_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        IN, OUT, K, N = 6, 5, 16, 64
        layer = _CPULayer(IN, OUT, K, seed=7)
        m = TokenParallelIndexedLinear(IN, OUT, K, layer=layer, average=False)
        # every rank starts from rank 0's parameters
        if rank != 0:
            with torch.no_grad():
                layer.table.mul_(0).add_(1.0)
        m.broadcast_parameters(0)
        gen = torch.Generator().manual_seed(11)
        x = torch.rand(N, IN, generator=gen) * 2 - 1
        go = torch.randn(N, OUT, generator=gen)
        sh = token_shard(N, world, rank)
        for step in range(2):  # the bucket is reused across steps
            m.zero_grad()
            y = m(x[sh])
            y.backward(go[sh])
            m.sync_grads()
        # single-process reference over all tokens
        ref = _CPULayer(IN, OUT, K, seed=7)
        eager_forward(x, ref.table, ref.bias, ref.bw).backward(go)
        ok = (torch.allclose(layer.table.grad, ref.table.grad, rtol=1e-5, atol=1e-6) and
              torch.allclose(layer.bias.grad, ref.bias.grad, rtol=1e-5, atol=1e-6) and
              layer.table.grad.data_ptr() == m._bucket.data_ptr())
        q.put((rank, ok, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _optimizer_zero_grad_worker(rank, world, port, q):
    """torch optimizers' zero_grad() sets .grad to None by default; the next
    forward must start the gradient bucket from zero, not from the last step."""
    try:
        _init(rank, world, port)
        IN, OUT, K, N = 6, 5, 16, 64
        layer = _CPULayer(IN, OUT, K, seed=7)
        m = TokenParallelIndexedLinear(IN, OUT, K, layer=layer, average=False)
        m.broadcast_parameters(0)
        opt = torch.optim.SGD(m.parameters(), lr=0.0)  # lr 0: parameters stay put, grads are compared
        gen = torch.Generator().manual_seed(13)
        x = torch.rand(N, IN, generator=gen) * 2 - 1
        go = torch.randn(N, OUT, generator=gen)
        sh = token_shard(N, world, rank)
        grads = []
        for step in range(3):
            opt.zero_grad()  # set_to_none=True
            m(x[sh]).backward(go[sh])
            m.sync_grads()
            opt.step()
            grads.append((layer.table.grad.clone(), layer.bias.grad.clone()))
        ref = _CPULayer(IN, OUT, K, seed=7)
        eager_forward(x, ref.table, ref.bias, ref.bw).backward(go)
        ok = all(torch.allclose(gt, ref.table.grad, rtol=1e-5, atol=1e-6) and
                 torch.allclose(gb, ref.bias.grad, rtol=1e-5, atol=1e-6) for gt, gb in grads)
        q.put((rank, ok, None if ok else "gradients accumulated across optimizer.zero_grad()"))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _column_shard_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        D._Fn = _EagerFn  # CPU stand-in for the CUDA autograd function
        IN, OUT, K, N = 4, 10, 8, 33
        full = _CPULayer(IN, OUT, K, seed=3)
        m = ColumnShardedIndexedLinear(IN, OUT, K, full_table=full.table.detach(),
                                       full_bias=full.bias.detach())

        gen = torch.Generator().manual_seed(5)
        x = (torch.rand(N, IN, generator=gen) * 3 - 1.5).requires_grad_(True)
        go = torch.randn(N, OUT, generator=gen)
        xf = x.reshape(-1, IN).contiguous()
        xs = D._SumDx.apply(xf, m.group)
        y_local = D._Fn.apply(xs, m.table, m.bias, m.bw)
        y = D._GatherColumns.apply(y_local, m.sizes, m.group)
        y.backward(go)
        xr = x.detach().clone().requires_grad_(True)
        yr = eager_forward(xr, full.table, full.bias, full.bw)
        yr.backward(go)
        ok = (torch.allclose(y, yr, rtol=1e-5, atol=1e-6) and
              torch.allclose(x.grad, xr.grad, rtol=1e-5, atol=1e-5) and
              torch.allclose(m.table.grad, full.table.grad[:, :, m.cols], rtol=1e-5, atol=1e-6) and
              torch.allclose(m.bias.grad, full.bias.grad[m.cols], rtol=1e-5, atol=1e-6))
        q.put((rank, ok, None))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    results = [q.get(timeout=180) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, ok, err in results:
        assert ok, f"rank {rank}: {err}"


def test_token_parallel_bucket_allreduce_gloo():
    _run(_token_parallel_worker, 2)


def test_token_parallel_optimizer_zero_grad_gloo():
    _run(_optimizer_zero_grad_worker, 2)


def test_column_shard_forward_backward_gloo():
    _run(_column_shard_worker, 2)


def test_rank_failure_surfaces_as_error_not_hang():
    """A rank that raises before the all-reduce: the survivor's collective ends
    with an error within the process-group timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    results = dict(q.get(timeout=90) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert results[1] == "raised"
    assert results[0] in ("error", "raised")


def _failing_worker(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            q.put((rank, "raised"))
            q.close()
            q.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves between steps, nothing in flight
        m = TokenParallelIndexedLinear(3, 2, 4, layer=_CPULayer(3, 2, 4, seed=1), average=False)
        m.zero_grad()
        m(torch.rand(5, 3)).sum().backward()
        try:
            m.sync_grads()
            q.put((rank, "completed"))
        except Exception:
            q.put((rank, "error"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
