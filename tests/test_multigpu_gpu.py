"""Multi-GPU paths on real GPUs: one process per GPU, NCCL, two ranks.

* the library's peer-memory all-reduce (il_allreduce_sum over torch
  symmetric memory, both flag-in-word kernels) against NCCL's all_reduce:
  odd sizes, repeated calls, scaling, CUDA-graph replay; every rank ends
  with the same bits;
* TokenParallelIndexedLinear with either exchange ("peer", "nccl") against
  the oracle on the unsharded batch: out and dx of each rank's tokens, the
  summed table and bias gradients, over two optimizer steps;
* ColumnShardedIndexedLinear (out_d split over the ranks, NCCL all-gather of
  y and all-reduce of dx) against the oracle, at the headline shape and at
  the large-table shape (1024 x 1024, K = 64);
* (one GPU) a bounded wait that runs out: the all-reduce given a peer whose
  flags nothing sets reports IL_ERR_TIMEOUT and the GPU stays usable.

The multi-rank tests skip with fewer than two GPUs: their kernels wait on one
another and must never share a GPU.
"""
import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from golden_io import normwise_close

pytestmark = pytest.mark.gpu
needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs two GPUs (one rank per GPU)")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return torch.device("cuda", rank)


def _finish():
    if dist.is_initialized():
        dist.destroy_process_group()


def _normwise(a, b, rtol):
    """|a - b| <= rtol * (|b| + max|b|) elementwise (golden_io.normwise_close)."""
    try:
        normwise_close(a, b, rtol)
        return True
    except AssertionError:
        return False


def _peer_allreduce_worker(rank, world, port, q):
    try:
        dev = _init(rank, world, port)
        from aiwn_b200 import _lib
        from aiwn_b200.comm import PeerBucket
        errs = []
        for n in (1, 3, 4, 5, 1027, 204820, 1 << 20):
            pb = PeerBucket(n, dev)
            g = torch.Generator(device=dev).manual_seed(1000 * n + rank)
            for rep in range(3):
                src = torch.randn(n, generator=g, device=dev)
                pb.tensor.copy_(src)
                ref = src.clone()
                dist.all_reduce(ref)
                scale = 0.5 if rep == 2 else 1.0
                pb.all_reduce(scale)
                torch.cuda.synchronize()
                if not torch.allclose(pb.tensor, ref * scale, rtol=1e-6, atol=1e-6):
                    errs.append(f"n={n} rep={rep}: max err {(pb.tensor - ref * scale).abs().max().item()}")
                # every rank holds the same bits
                bits = pb.tensor.view(torch.int32).clone()
                bits0 = bits.clone()
                dist.broadcast(bits0, 0)
                if not torch.equal(bits, bits0):
                    errs.append(f"n={n} rep={rep}: ranks disagree")
        # captured once, replayed on fresh data
        n = 204820
        pb = PeerBucket(n, dev)
        pb.tensor.normal_()
        torch.cuda.synchronize()
        pb.all_reduce()  # warm-up outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            pb.all_reduce()
        for rep in range(3):
            src = torch.randn(n, device=dev)
            pb.tensor.copy_(src)
            ref = src.clone()
            dist.all_reduce(ref)
            graph.replay()
            torch.cuda.synchronize()
            if not torch.allclose(pb.tensor, ref, rtol=1e-6, atol=1e-6):
                errs.append(f"graph replay {rep}: max err {(pb.tensor - ref).abs().max().item()}")
        del graph
        _lib.check_device_status(dev)
        q.put((rank, not errs, "; ".join(errs)))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))
    finally:
        _finish()


def _token_parallel_worker(rank, world, port, q):
    try:
        dev = _init(rank, world, port)
        from oracle import oracle
        from aiwn_b200 import IndexedLinear
        from aiwn_b200.distributed import TokenParallelIndexedLinear, token_shard
        IN, OUT, K, N = 20, 20, 512, 8192
        g = torch.Generator().manual_seed(42)
        x = torch.rand(N, IN, generator=g) * 2 - 1
        go = torch.randn(N, OUT, generator=g)
        table = torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)
        bias = torch.randn(OUT, generator=g) * 0.1
        bw = 2.0 / K
        ref_out = oracle.forward(x.numpy(), table.numpy(), bias.numpy(), bw)
        rgx, rgt, rgb = oracle.backward(go.numpy(), x.numpy(), table.numpy(), bw)
        sh = token_shard(N, world, rank)
        errs = []
        for exchange in ("peer", "nccl"):
            layer = IndexedLinear(IN, OUT, K).to(dev)
            m = TokenParallelIndexedLinear(IN, OUT, K, layer=layer, average=False, exchange=exchange)
            with torch.no_grad():
                layer.table.copy_(table if rank == 0 else torch.zeros_like(table))
                layer.bias.copy_(bias if rank == 0 else torch.zeros_like(bias))
            m.broadcast_parameters(0)
            opt = torch.optim.SGD(m.parameters(), lr=0.0)
            for step in range(2):
                opt.zero_grad()
                xs = x[sh].to(dev).requires_grad_(True)
                y = m(xs)
                y.backward(go[sh].to(dev))
                m.sync_grads()
                opt.step()
                torch.cuda.synchronize()
                tag = f"{exchange} step {step}"
                if not _normwise(y.detach().cpu().numpy(), ref_out[sh], 1e-5):
                    errs.append(f"{tag}: out")
                if not _normwise(xs.grad.cpu().numpy(), rgx[sh], 1e-4):
                    errs.append(f"{tag}: dx")
                if not _normwise(layer.table.grad.cpu().numpy(), rgt, 1e-4):
                    errs.append(f"{tag}: dtable")
                if not _normwise(layer.bias.grad.cpu().numpy(), rgb, 1e-4):
                    errs.append(f"{tag}: dbias")
            if exchange == "peer" and m._peer is None:
                errs.append("exchange='peer' did not use the peer bucket")
        q.put((rank, not errs, "; ".join(errs)))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))
    finally:
        _finish()


def _column_shard_worker(rank, world, port, q):
    try:
        dev = _init(rank, world, port)
        from oracle import oracle
        from aiwn_b200.distributed import ColumnShardedIndexedLinear
        errs = []
        # the headline layer's shape with out_d split, and the large-table shape
        for IN, OUT, K, N, xdist in ((20, 40, 512, 4096, "uniform"), (1024, 1024, 64, 256, "clamp_normal")):
            g = torch.Generator().manual_seed(7 + IN)
            if xdist == "uniform":
                x = torch.rand(N, IN, generator=g) * 2 - 1
            else:
                x = (torch.randn(N, IN, generator=g) * 0.5).clamp(-1, 1)
            go = torch.randn(N, OUT, generator=g)
            table = torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)
            bias = torch.randn(OUT, generator=g) * 0.1
            bw = 2.0 / K
            m = ColumnShardedIndexedLinear(IN, OUT, K, full_table=table, full_bias=bias).to(dev)
            xd = x.to(dev).requires_grad_(True)
            y = m(xd)
            y.backward(go.to(dev))
            torch.cuda.synchronize()
            ref_out = oracle.forward(x.numpy(), table.numpy(), bias.numpy(), bw)
            rgx, rgt, rgb = oracle.backward(go.numpy(), x.numpy(), table.numpy(), bw)
            tag = f"{IN}x{OUT} K={K}"
            if not _normwise(y.detach().cpu().numpy(), ref_out, 1e-5):
                errs.append(f"{tag}: out")
            if not _normwise(xd.grad.cpu().numpy(), rgx, 1e-4):
                errs.append(f"{tag}: dx")
            if not _normwise(m.table.grad.cpu().numpy(), rgt[:, :, m.cols], 1e-4):
                errs.append(f"{tag}: dtable of the rank's columns")
            if not _normwise(m.bias.grad.cpu().numpy(), rgb[m.cols], 1e-4):
                errs.append(f"{tag}: dbias of the rank's columns")
        q.put((rank, not errs, "; ".join(errs)))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))
    finally:
        _finish()


def _run(worker, world=2, timeout=600):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    try:
        results = [q.get(timeout=timeout) for _ in ps]
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for rank, ok, err in results:
        assert ok, f"rank {rank}: {err}"


@needs2
@pytest.mark.parametrize("kernel", ["warp", "thread"])
def test_peer_allreduce_matches_nccl(kernel, monkeypatch):
    """Both flag-in-word kernels: one warp per (32 pairs, rank), the default
    for 2, 4 and 8 ranks, and one thread per pair (AIWN_IL_ALLREDUCE=thread)."""
    monkeypatch.setenv("AIWN_IL_ALLREDUCE", kernel)
    _run(_peer_allreduce_worker)


@needs2
def test_token_parallel_two_ranks_match_oracle():
    _run(_token_parallel_worker)


@needs2
def test_column_sharded_two_ranks_match_oracle():
    _run(_column_shard_worker)


@pytest.mark.parametrize("n,kernel", [(4096, "warp"), (4096, "thread"), ((1 << 21) + 4, "warp")],
                         ids=["flags_in_words_warp", "flags_in_words_thread", "two_shot"])
def test_allreduce_wait_runs_out_and_reports(n, kernel, monkeypatch):
    """One GPU, a 2-rank all-reduce whose second 'rank' is a local buffer that
    no kernel ever serves: every bounded wait gives up after 50 ms, the
    status reads IL_ERR_TIMEOUT, and the device keeps working.  Both kernels
    (small buffers: flags in the data words; large: per-block barriers)."""
    from aiwn_b200 import _lib
    monkeypatch.setenv("AIWN_IL_ALLREDUCE", kernel)
    dev = torch.device("cuda", 0)
    sb = _lib.allreduce_scratch_bytes(n, 2)
    bufs = [torch.ones(n + 64, device=dev) for _ in range(2)]
    scratch = [torch.zeros(sb, dtype=torch.uint8, device=dev) for _ in range(2)]
    torch.cuda.synchronize()
    _lib.allreduce_sum([b.data_ptr() for b in bufs], [s.data_ptr() for s in scratch], n, 0, 2, 1.0, 0.05,
                       device=dev)
    with pytest.raises(_lib.ILError, match="bounded wait"):
        _lib.check_device_status(dev)
    # nothing was summed or delivered, and the context is usable
    for b in bufs:
        assert torch.equal(b, torch.ones(n + 64, device=dev))
    _lib.check_device_status(dev)  # the error word was cleared
    y = torch.arange(10.0, device=dev).sum()
    assert y.item() == 45.0
