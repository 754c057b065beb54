"""Host-resident batches through IndexedLinear with copies overlapped.

IndexedLinear treats tokens independently, so a batch that lives in host
memory can be split into chunks whose host-to-device copy, forward/backward
kernels and device-to-host copy run on three CUDA streams in a pipeline:
while chunk c computes, chunk c+1 is being uploaded and chunk c-1's results
are being downloaded.  Table and bias gradients add up exactly over chunks
(they are sums over tokens): ``il_backward_accumulate`` adds every chunk's
into the same sums, so the result equals one call on the whole batch up to
fp32 summation order.

    step = HostPipeline(layer)          # chunk count tuned per batch shape on first use
    step.forward_backward(x_host, go_host, out_host, gx_host)   # pinned tensors

The whole multi-stream step (copies, kernels, per-chunk gradient sums) is
captured once per set of host buffers into a CUDA graph and replayed, so a
step costs one graph launch on the host instead of a few dozen API calls.
This is the path a caller with data in host memory uses; the kernels are the
same as for device tensors.
"""
from __future__ import annotations

import os
import time

import torch

from . import _lib


def _parse_cpulist(text: str) -> set:
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_numa_cpus(device) -> tuple:
    """(NUMA node, CPUs local to it) of a CUDA device's PCI slot, from sysfs;
    (None, None) where the platform does not say."""
    dev = torch.device(device)
    props = torch.cuda.get_device_properties(dev.index if dev.index is not None else torch.cuda.current_device())
    addr = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    base = os.path.join("/sys/bus/pci/devices", addr)
    try:
        with open(os.path.join(base, "numa_node")) as f:
            node = int(f.read().strip())
        with open(os.path.join(base, "local_cpulist")) as f:
            cpus = _parse_cpulist(f.read())
    except (OSError, ValueError):
        return None, None
    return (node if node >= 0 else None), (cpus or None)


def bind_host_to_gpu(device) -> dict:
    """Restrict this process's host threads to the CPUs of the GPU's NUMA
    node, so that pinned host buffers allocated afterwards (first touch) and
    the threads that issue copies sit next to the GPU's PCIe root, and ranks
    of a multi-GPU job spread over the sockets instead of all running on the
    first.  Returns what it did (for the record)."""
    node, cpus = gpu_numa_cpus(device)
    allowed = os.sched_getaffinity(0)
    use = (cpus & allowed) if cpus else None
    if use:
        os.sched_setaffinity(0, use)
        torch.set_num_threads(max(1, min(torch.get_num_threads(), len(use))))
    return {"numa_node": node, "cpus": len(use) if use else len(allowed), "bound": bool(use)}


class HostPipeline:
    """Chunked, stream-overlapped forward(+backward) of an IndexedLinear (or
    TokenParallelIndexedLinear) over pinned host tensors.

    Each chunk gets its own device buffers (x, go, out, dx) as long as the
    whole batch fits ``max_resident_bytes``; then the only ordering between
    chunks is that of each stream, and the upload of chunk c+1 never waits for
    chunk c's results to leave.  Larger batches reuse a ring of slots.

    Copies can be coarser than the compute chunks (``pieces`` < ``chunks``,
    resident batches only): every pinned host<->device copy costs ~9 us of
    copy-engine time beyond its bytes on the hosts measured (two 21 MiB
    copies, one each way, took 0.46 ms; the same bytes in 16 pieces each
    0.72 ms), while the kernels gain from fine chunks.  A piece of several
    chunks is uploaded with one copy per input, its chunks' forwards run,
    its out leaves with one copy while their backwards run, then its dx.
    ``pieces`` is a count of equal pieces or a tuple of chunk counts per
    piece; pieces that shrink towards the end shorten the step's tail (the
    last piece's kernels and download come after the last upload).
    """

    # chunk counts and upload pieces tried when none is given
    TUNE_CHUNKS = (1, 2, 4, 8, 16)
    TUNE_PIECES = (1, 2, 4)
    TUNE_TAPERED = {8: ((4, 2, 1, 1),), 16: ((5, 5, 3, 2, 1), (6, 4, 3, 2, 1))}
    TUNE_MIN_CHUNK = 4096  # tokens
    TUNE_STEPS = 5
    TUNE_FINALISTS = 3

    def __init__(self, layer, chunks: int | None = None, device=None, graphs: bool = True,
                 max_resident_bytes: int = 1 << 30, pieces=None):
        self.layer = layer
        inner = getattr(layer, "layer", layer)
        self.inner = inner
        self.auto = chunks is None
        self.chunks = 1 if chunks is None else max(1, int(chunks))
        # copy pieces: one per chunk unless given; an int must divide the chunk
        # count, a tuple of chunk counts must add up to it
        if pieces is None:
            pieces = self.chunks
        if isinstance(pieces, (tuple, list)):
            sizes = tuple(int(v) for v in pieces)
            if not sizes or min(sizes) < 1 or sum(sizes) != self.chunks:
                raise ValueError(f"piece sizes {sizes} must be >= 1 and add up to chunks ({self.chunks})")
            self.pieces = sizes
        else:
            q = max(1, min(int(pieces), self.chunks))
            if self.chunks % q:
                raise ValueError(f"pieces ({q}) must divide chunks ({self.chunks})")
            self.pieces = q
            sizes = (self.chunks // q,) * q
        self.piece_sizes = sizes
        self._tuned = {}  # (N, in, out, x dtype) -> tuned HostPipeline
        self.device = torch.device(device) if device is not None else inner.table.device
        self.s_h2d = torch.cuda.Stream(self.device)
        self.s_cmp = torch.cuda.Stream(self.device)
        self.s_d2h = torch.cuda.Stream(self.device)
        self.graphs = graphs
        self.max_resident_bytes = int(max_resident_bytes)
        self._bufs = None
        self._ws = None
        self._graph_cache = {}

    def _buffers(self, n, IN, OUT, xdtype):
        key = (n, IN, OUT, xdtype, self.chunks)
        if self._bufs is None or self._bufs[0] != key:
            mk = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt, device=self.device)  # noqa: E731
            xs = torch.empty(0, dtype=xdtype).element_size()
            slot_bytes = n * (2 * IN * xs + 2 * OUT * 4)
            nslots = max(2, min(self.chunks, self.max_resident_bytes // max(slot_bytes, 1)))
            if nslots >= self.chunks:
                # resident: one buffer per kind, chunk c is rows [c*n, (c+1)*n),
                # so that an upload piece can span several chunks
                full = dict(x=mk(self.chunks * n, IN, dt=xdtype), go=mk(self.chunks * n, OUT),
                            out=mk(self.chunks * n, OUT), gx=mk(self.chunks * n, IN, dt=xdtype))
                slots = [{k: v[c * n:(c + 1) * n] for k, v in full.items()} for c in range(self.chunks)]
            else:
                slots = [dict(x=mk(n, IN, dt=xdtype), go=mk(n, OUT), out=mk(n, OUT), gx=mk(n, IN, dt=xdtype))
                         for _ in range(nslots)]
                full = None
            K = self.inner.K
            # the gradients of all chunks add up here (il_backward_accumulate)
            grads = dict(gt_sum=mk(K, IN, OUT), gb_sum=mk(OUT))
            self._bufs = (key, slots, grads, full)
            self._graph_cache.clear()
        return self._bufs[1], self._bufs[2], self._bufs[3]

    def _issue(self, x_host, go_host, out_host, gx_host, table, bias, want_grads):
        """Enqueue the whole pipelined step; joins every side stream back into
        the caller's current stream (so it can be captured as one graph)."""
        inner = self.inner
        N, IN = x_host.shape
        OUT, K = inner.out_dim, inner.K
        n = (N + self.chunks - 1) // self.chunks
        slots, gr, full = self._buffers(n, IN, OUT, x_host.dtype)
        S = len(slots)
        # copy pieces (resident buffers only; a ring copies per chunk)
        sizes = self.piece_sizes if full is not None else (1,) * self.chunks
        ws_n = _lib.workspace_bytes(n, IN, OUT, K, _lib.x_dtype_code(slots[0]["x"]))
        if ws_n and (self._ws is None or self._ws.numel() < ws_n):
            self._ws = torch.empty(ws_n, dtype=torch.uint8, device=self.device)
        cur = torch.cuda.current_stream(self.device)
        if want_grads:
            gr["gt_sum"].zero_()
            gr["gb_sum"].zero_()
        # parameters (and the sums just zeroed) were written on the caller's stream
        for s in (self.s_h2d, self.s_cmp, self.s_d2h):
            s.wait_stream(cur)
        ev = lambda: torch.cuda.Event()  # noqa: E731
        nch = (N + n - 1) // n  # non-empty chunks
        bounds, c0 = [], 0
        for sz in sizes:
            if c0 >= nch:
                break
            bounds.append((c0, min(nch, c0 + sz)))
            c0 += sz
        npieces = len(bounds)
        # per piece (= per chunk in a ring): x_up, go_up, fwd_done, bwd_done, out_down, gx_down
        x_up, go_up, fwd_done, bwd_done, out_down, gx_down = ([ev() for _ in range(npieces)] for _ in range(6))
        for q, (c0, c1) in enumerate(bounds):
            pa, pb = c0 * n, min(N, c1 * n)
            if full is not None:  # resident: one copy per piece, straight into the whole-batch buffers
                xq, goq, outq, gxq = (full[k][pa:pb] for k in ("x", "go", "out", "gx"))
            else:
                sl = slots[q % S]
                xq, goq, outq, gxq = (sl[k][:pb - pa] for k in ("x", "go", "out", "gx"))
            with torch.cuda.stream(self.s_h2d):
                if q >= S:
                    self.s_h2d.wait_event(bwd_done[q - S])  # the slot's inputs are consumed
                xq.copy_(x_host[pa:pb], non_blocking=True)
                x_up[q].record(self.s_h2d)
                goq.copy_(go_host[pa:pb], non_blocking=True)
                go_up[q].record(self.s_h2d)
            # the piece's forwards first, so that its out leaves while the backwards run
            with torch.cuda.stream(self.s_cmp):
                self.s_cmp.wait_event(x_up[q])
                if q >= S:
                    self.s_cmp.wait_event(out_down[q - S])  # the slot's out has left
                for c in range(c0, c1):
                    a, b = (c - c0) * n, min(pb - pa, (c - c0 + 1) * n)
                    _lib.forward(xq[a:b], table, bias, outq[a:b], inner.bw)
                fwd_done[q].record(self.s_cmp)
                self.s_cmp.wait_event(go_up[q])
                if q >= S:
                    self.s_cmp.wait_event(gx_down[q - S])
                for c in range(c0, c1):
                    a, b = (c - c0) * n, min(pb - pa, (c - c0 + 1) * n)
                    _lib.backward(goq[a:b], xq[a:b], table, gxq[a:b], gr["gt_sum"] if want_grads else None,
                                  gr["gb_sum"] if want_grads else None, inner.bw, self._ws if ws_n else None,
                                  accumulate=True)
                bwd_done[q].record(self.s_cmp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(fwd_done[q])
                out_host[pa:pb].copy_(outq, non_blocking=True)
                out_down[q].record(self.s_d2h)
                self.s_d2h.wait_event(bwd_done[q])
                gx_host[pa:pb].copy_(gxq, non_blocking=True)
                gx_down[q].record(self.s_d2h)
        for s in (self.s_h2d, self.s_cmp, self.s_d2h):
            cur.wait_stream(s)
        return gr

    def _tune(self, x_host, go_host, out_host, gx_host):
        """The fastest chunk and piece counts for this batch shape on this
        host: every pinned copy has a fixed cost while every chunk adds the
        kernels' fixed cost, so the best split depends on the machine.  Each
        candidate runs one untimed and TUNE_STEPS timed steps (the fastest
        step counts; gradients stay in the pipeline's own sums); the best
        TUNE_FINALISTS are timed once more and the fastest of all is kept."""
        N = x_host.shape[0]
        cs = [c for c in self.TUNE_CHUNKS if c == 1 or N // c >= self.TUNE_MIN_CHUNK]
        cands = [(c, q) for c in cs for q in sorted(set(self.TUNE_PIECES) | {c}) if q <= c and c % q == 0]
        cands += [(c, t) for c in cs for t in self.TUNE_TAPERED.get(c, ())]
        cur = torch.cuda.current_stream(self.device)

        def make(c, q):
            return HostPipeline(self.layer, chunks=c, device=self.device, graphs=self.graphs,
                                max_resident_bytes=self.max_resident_bytes, pieces=q)

        def timed(p):
            p._run(x_host, go_host, out_host, gx_host, True)
            cur.synchronize()
            best_step = None
            for _ in range(self.TUNE_STEPS):
                t0 = time.perf_counter()
                p._run(x_host, go_host, out_host, gx_host, True)
                cur.synchronize()  # a step ends with its results in host memory
                dt = time.perf_counter() - t0
                best_step = dt if best_step is None else min(best_step, dt)
            return best_step

        times = {}
        for cand in cands:
            p = make(*cand)
            times[cand] = timed(p)
            del p
        for cand in sorted(times, key=times.get)[:self.TUNE_FINALISTS]:
            p = make(*cand)
            times[cand] = min(times[cand], timed(p))
            del p
        return make(*min(times, key=times.get))

    def forward_backward(self, x_host, go_host, out_host, gx_host, accumulate_grads: bool = True):
        """out_host <- layer(x_host); gx_host <- d/dx; table.grad/bias.grad +=.

        All four host tensors must be pinned ([N, in] / [N, out], x dtype
        fp32 or bf16).  Returns when the results are in host memory."""
        for t in (x_host, go_host, out_host, gx_host):
            if not t.is_pinned():
                raise ValueError("HostPipeline needs pinned host tensors (tensor.pin_memory())")
        runner = self
        if self.auto:
            key = (tuple(x_host.shape), tuple(go_host.shape), x_host.dtype)
            runner = self._tuned.get(key)
            if runner is None:
                runner = self._tune(x_host, go_host, out_host, gx_host)
                self._tuned[key] = runner
        gr = runner._run(x_host, go_host, out_host, gx_host, accumulate_grads)
        if accumulate_grads:
            for p, s in ((self.inner.table, gr["gt_sum"]), (self.inner.bias, gr["gb_sum"])):
                if p.grad is None:
                    p.grad = s.clone()
                else:
                    p.grad.add_(s)
        torch.cuda.current_stream(self.device).synchronize()
        return out_host, gx_host

    @property
    def chosen_chunks(self) -> dict:
        """Chunk count in use per batch size N (the tuned ones when auto)."""
        if not self.auto:
            return {"all": self.chunks}
        return {k[0][0]: p.chunks for k, p in self._tuned.items()}

    @property
    def chosen_pieces(self) -> dict:
        """Copy pieces in use per batch size N (the tuned ones when auto): a
        count of equal pieces or a tuple of chunk counts."""
        if not self.auto:
            return {"all": self.pieces}
        return {k[0][0]: p.pieces for k, p in self._tuned.items()}

    def _run(self, x_host, go_host, out_host, gx_host, want_grads: bool):
        """One pipelined step with this instance's chunk count; returns the
        gradient sums (valid once the current stream reaches this point)."""
        inner = self.inner
        table, bias = inner.table.detach(), inner.bias.detach()
        cur = torch.cuda.current_stream(self.device)
        if self.graphs:
            key = (x_host.data_ptr(), go_host.data_ptr(), out_host.data_ptr(), gx_host.data_ptr(),
                   tuple(x_host.shape), x_host.dtype, table.data_ptr(), bias.data_ptr(), bool(want_grads))
            entry = self._graph_cache.get(key)
            if entry is None:
                # one eager step first: the library's per-device setup and the
                # kernels' attributes are then in place before capture
                gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, want_grads)
                cur.synchronize()
                g = torch.cuda.CUDAGraph()
                # captured on torch's side capture stream; replayed on `cur`
                with torch.cuda.graph(g, capture_error_mode="relaxed"):
                    gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, want_grads)
                entry = (g, gr)
                self._graph_cache[key] = entry
            entry[0].replay()
            gr = entry[1]
        else:
            gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, want_grads)
        return gr
