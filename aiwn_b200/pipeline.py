"""Host-resident batches through IndexedLinear with copies overlapped.

IndexedLinear treats tokens independently, so a batch that lives in host
memory can be split into chunks whose host-to-device copy, forward/backward
kernels and device-to-host copy run on three CUDA streams in a pipeline:
while chunk c computes, chunk c+1 is being uploaded and chunk c-1's results
are being downloaded.  Table and bias gradients add up exactly over chunks
(they are sums over tokens), so the result equals one call on the whole
batch up to fp32 summation order.

    step = HostPipeline(layer, chunks=4)
    step.forward_backward(x_host, go_host, out_host, gx_host)   # pinned tensors

The whole multi-stream step (copies, kernels, per-chunk gradient sums) is
captured once per set of host buffers into a CUDA graph and replayed, so a
step costs one graph launch on the host instead of a few dozen API calls.
This is the path a caller with data in host memory uses; the kernels are the
same as for device tensors.
"""
from __future__ import annotations

import torch

from . import _lib


class HostPipeline:
    """Chunked, stream-overlapped forward(+backward) of an IndexedLinear (or
    TokenParallelIndexedLinear) over pinned host tensors."""

    def __init__(self, layer, chunks: int = 4, device=None, graphs: bool = True):
        self.layer = layer
        inner = getattr(layer, "layer", layer)
        self.inner = inner
        self.chunks = max(1, int(chunks))
        self.device = torch.device(device) if device is not None else inner.table.device
        self.s_h2d = torch.cuda.Stream(self.device)
        self.s_cmp = torch.cuda.Stream(self.device)
        self.s_d2h = torch.cuda.Stream(self.device)
        self.graphs = graphs
        self._bufs = None
        self._ws = None
        self._graph_cache = {}

    def _buffers(self, n, IN, OUT, xdtype):
        key = (n, IN, OUT, xdtype)
        if self._bufs is None or self._bufs[0] != key:
            mk = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt, device=self.device)  # noqa: E731
            # two slots per stream stage so chunk c+1 can land while chunk c computes
            slots = [dict(x=mk(n, IN, dt=xdtype), go=mk(n, OUT), out=mk(n, OUT), gx=mk(n, IN, dt=xdtype))
                     for _ in range(2)]
            K = self.inner.K
            # per-chunk gradients and their running sums over the chunks
            grads = dict(gt=mk(K, IN, OUT), gb=mk(OUT), gt_sum=mk(K, IN, OUT), gb_sum=mk(OUT))
            self._bufs = (key, slots, grads)
            self._graph_cache.clear()
        return self._bufs[1], self._bufs[2]

    def _issue(self, x_host, go_host, out_host, gx_host, table, bias, want_grads):
        """Enqueue the whole pipelined step; joins every side stream back into
        the caller's current stream (so it can be captured as one graph)."""
        inner = self.inner
        N, IN = x_host.shape
        OUT, K = inner.out_dim, inner.K
        n = (N + self.chunks - 1) // self.chunks
        slots, gr = self._buffers(n, IN, OUT, x_host.dtype)
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
        up_done = [torch.cuda.Event() for _ in range(2)]
        cmp_done = [torch.cuda.Event() for _ in range(2)]
        down_done = [torch.cuda.Event() for _ in range(2)]
        for c in range(self.chunks):
            a, b = c * n, min(N, (c + 1) * n)
            if a >= b:
                break
            m = b - a
            sl = slots[c & 1]
            with torch.cuda.stream(self.s_h2d):
                if c >= 2:
                    self.s_h2d.wait_event(cmp_done[c & 1])  # slot's inputs consumed
                sl["x"][:m].copy_(x_host[a:b], non_blocking=True)
                sl["go"][:m].copy_(go_host[a:b], non_blocking=True)
                up_done[c & 1].record(self.s_h2d)
            with torch.cuda.stream(self.s_cmp):
                self.s_cmp.wait_event(up_done[c & 1])
                if c >= 2:
                    self.s_cmp.wait_event(down_done[c & 1])  # slot's outputs downloaded
                xs, gos = sl["x"][:m], sl["go"][:m]
                _lib.forward(xs, table, bias, sl["out"][:m], inner.bw)
                _lib.backward(gos, xs, table, sl["gx"][:m], gr["gt"] if want_grads else None,
                              gr["gb"] if want_grads else None, inner.bw, self._ws if ws_n else None)
                if want_grads:
                    gr["gt_sum"].add_(gr["gt"])
                    gr["gb_sum"].add_(gr["gb"])
                cmp_done[c & 1].record(self.s_cmp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(cmp_done[c & 1])
                out_host[a:b].copy_(sl["out"][:m], non_blocking=True)
                gx_host[a:b].copy_(sl["gx"][:m], non_blocking=True)
                down_done[c & 1].record(self.s_d2h)
        for s in (self.s_h2d, self.s_cmp, self.s_d2h):
            cur.wait_stream(s)
        return gr

    def forward_backward(self, x_host, go_host, out_host, gx_host, accumulate_grads: bool = True):
        """out_host <- layer(x_host); gx_host <- d/dx; table.grad/bias.grad +=.

        All four host tensors must be pinned ([N, in] / [N, out], x dtype
        fp32 or bf16).  Returns when the results are in host memory."""
        for t in (x_host, go_host, out_host, gx_host):
            if not t.is_pinned():
                raise ValueError("HostPipeline needs pinned host tensors (tensor.pin_memory())")
        inner = self.inner
        table, bias = inner.table.detach(), inner.bias.detach()
        cur = torch.cuda.current_stream(self.device)
        if self.graphs:
            key = (x_host.data_ptr(), go_host.data_ptr(), out_host.data_ptr(), gx_host.data_ptr(),
                   tuple(x_host.shape), x_host.dtype, table.data_ptr(), bias.data_ptr(), bool(accumulate_grads))
            entry = self._graph_cache.get(key)
            if entry is None:
                # one eager step first: the library's per-device setup and the
                # kernels' attributes are then in place before capture
                gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, accumulate_grads)
                cur.synchronize()
                g = torch.cuda.CUDAGraph()
                # captured on torch's side capture stream; replayed on `cur`
                with torch.cuda.graph(g, capture_error_mode="relaxed"):
                    gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, accumulate_grads)
                entry = (g, gr)
                self._graph_cache[key] = entry
            entry[0].replay()
            gr = entry[1]
        else:
            gr = self._issue(x_host, go_host, out_host, gx_host, table, bias, accumulate_grads)
        if accumulate_grads:
            for p, s in ((inner.table, gr["gt_sum"]), (inner.bias, gr["gb_sum"])):
                if p.grad is None:
                    p.grad = s.clone()
                else:
                    p.grad.add_(s)
        cur.synchronize()
        return out_host, gx_host
