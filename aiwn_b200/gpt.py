"""IndexedGPT on B200 -- the reference's transformer with every projection an
IndexedLinear (transformer_validation.py:232-385), built on this package's
layers, and a training step captured as one CUDA graph.

Module structure, parameter names and initialisation follow the reference
(``transformer.wte / wpe / h[i].{ln1, ln2, attn.{q,k,v,c}_proj, ffn.{cdf,
up, down}} / ln_f``, ``lm_head``), so its state_dicts load unchanged.  The
FFN's GaussianCDFNorm -> up pair runs as one IndexedLinearV2 chain
(``il_cdf_forward``: the prologue fused into the forward when its output fits
one j-range); every other IndexedLinear runs the library's forward and
backward kernels, and the blocks' LayerNorms (d_idx <= 32) run
``il_layernorm_forward`` / ``il_layernorm_backward``.

At the reference's config-5 sizes (n_embd 256, K=128 -> d_idx 16, ff_idx 8;
batch 64 x ctx 256) every kernel is small and the eager step is bound by
launch and host overhead.  ``GraphedTrainStep`` captures forward, backward,
gradient clipping and a capturable AdamW step once and replays them: one
graph launch per step.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .layers import GaussianCDFNorm, IndexedLinear
from .layers.indexed_linear import TRITON_OK, _Fn, grad_pair
from .layers.indexed_linear_v2 import _FnV2


class _LayerNormFn(torch.autograd.Function):
    """LayerNorm over the last dim for d <= 32 through il_layernorm_forward /
    il_layernorm_backward (fp32, one token per thread, rows in registers)."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        n = x2.shape[0]
        y = torch.empty_like(x2)
        mean, rstd = x2.new_empty(n), x2.new_empty(n)
        _lib.layernorm_forward(x2, weight, bias, eps, y, mean, rstd)
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape = shape
        return y.reshape(shape)

    @staticmethod
    def backward(ctx, gy):
        x2, weight, mean, rstd = ctx.saved_tensors
        gy2 = gy.reshape(x2.shape).contiguous()
        dx = torch.empty_like(x2) if ctx.needs_input_grad[0] else None
        dw, db = grad_pair(weight.shape, weight.shape, weight.device, ctx.needs_input_grad[1],
                           ctx.needs_input_grad[2])
        _lib.layernorm_backward(gy2, x2, weight, mean, rstd, dx, dw, db)
        return (dx.reshape(ctx.shape) if dx is not None else None), dw, db, None


class _AttentionFn(torch.autograd.Function):
    """Causal attention of q, k, v [B, T, H*D] through il_attention_forward /
    il_attention_backward (narrow heads, dropout p with a device seed)."""

    @staticmethod
    def forward(ctx, q, k, v, H, p, seed):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        B, T, C = q.shape
        scale = 1.0 / math.sqrt(C // H)
        o = torch.empty_like(q)
        lse = q.new_empty(B, H, T)
        _lib.attention_forward(q, k, v, o, lse, H, scale, p, seed)
        ctx.save_for_backward(q, k, v, o, lse, seed)
        ctx.H, ctx.p, ctx.scale = H, p, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, seed = ctx.saved_tensors
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        _lib.attention_backward(q, k, v, o, do.contiguous(), lse, dq, dk, dv, ctx.H, ctx.scale, ctx.p, seed)
        return dq, dk, dv, None, None, None


def layer_norm(ln: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    """``ln(x)`` with the library's kernels where they apply (fp32 CUDA
    input, one normalised dim of at most 32, affine, no hooks on ``ln``);
    torch's LayerNorm otherwise.  The IndexedGPT blocks' d_idx is 16 at the
    reference's config 5, where torch's backward spends ~77 us per call on
    the gamma/beta reduction of 16-wide rows."""
    if (len(ln.normalized_shape) == 1 and ln.normalized_shape[0] <= 32 and ln.weight is not None
            and ln.bias is not None and x.is_cuda and x.dtype == torch.float32
            and not (ln._forward_pre_hooks or ln._forward_hooks)):
        return _LayerNormFn.apply(x, ln.weight, ln.bias, ln.eps)
    return ln(x)


def get_d_idx(n_embd: int, K: int, n_head: int) -> tuple:
    """(d_idx, ff_idx): n_embd/sqrt(K) and 4*n_embd/K, each rounded down to a
    power of two (d_idx also divisible by n_head), as transformer_validation.py:68-87."""
    raw_d = int(n_embd / math.sqrt(K))
    p2_d = 1 << (raw_d.bit_length() - 1)
    while p2_d % n_head != 0 and p2_d > n_head:
        p2_d >>= 1
    d_idx = max(n_head, p2_d)
    raw_ff = max(4, (4 * n_embd) // K)
    p2_ff = 1 << (raw_ff.bit_length() - 1)
    ff_idx = max(4, p2_ff)
    return d_idx, ff_idx


def _observed(m) -> bool:
    """Whether a layer's own forward must run: forward hooks, or a
    BucketTracker accumulator that the layer's forward kernel adds into."""
    return bool(m._forward_pre_hooks or m._forward_hooks or getattr(m, "_bin_counts", None) is not None)


class IndexedAttention(nn.Module):
    """Causal multi-head attention with IndexedLinear q/k/v/c projections.

    ``fused=True`` computes softmax(mask(q k^T / sqrt(d))) v with dropout
    without [B, H, T, T] tensors in memory: through il_attention_forward /
    backward for fp32 CUDA heads of 2, 4, 8 or 16 features (the dropout seed
    lives on the device and advances every training forward, so CUDA graph
    replays draw new masks), else torch's scaled_dot_product_attention.
    ``fused=False`` keeps the reference's explicit masked-softmax formulation
    (transformer_validation.py:264-267).  They agree to fp32 rounding without
    dropout; with dropout they draw different random masks."""

    def __init__(self, d_idx, n_head, block_size, K, dropout=0.1, fused=True):
        super().__init__()
        assert d_idx % n_head == 0
        self.n_head = n_head
        self.d_idx = d_idx
        self.fused = fused
        self._attn_seed = None  # device int64 [1], drawn from the CUDA generator on first use
        self.q_proj = IndexedLinear(d_idx, d_idx, K)
        self.k_proj = IndexedLinear(d_idx, d_idx, K)
        self.v_proj = IndexedLinear(d_idx, d_idx, K)
        self.c_proj = IndexedLinear(d_idx, d_idx, K)
        self.attn_drop = nn.Dropout(dropout)
        self.resid_drop = nn.Dropout(dropout)
        self.register_buffer("bias", torch.tril(torch.ones(block_size, block_size)).view(1, 1, block_size,
                                                                                          block_size))

    def _qkv(self, h, B, T):
        """q, k, v [B, T, d_idx].  With the fused form and no hooks on the
        projections, one IndexedLinear over the three tables concatenated along
        out_d computes [q | k | v] (each output column depends only on its own
        table column, and dx sums over all of them): one forward and one
        backward instead of three of each."""
        projs = (self.q_proj, self.k_proj, self.v_proj)
        if (self.fused and h.is_cuda and h.dtype == torch.float32 and TRITON_OK
                and not any(_observed(m) for m in projs)):
            tab = torch.cat([m.table for m in projs], dim=2)
            bias = torch.cat([m.bias for m in projs])
            qkv = _Fn.apply(h.contiguous(), tab, bias, self.q_proj.bw).view(B, T, 3 * self.d_idx)
            return qkv.split(self.d_idx, dim=2)
        return tuple(m(h).reshape(B, T, self.d_idx) for m in projs)

    def forward(self, x):
        B, T, C = x.shape
        h = x.reshape(B * T, C)
        q, k, v = self._qkv(h, B, T)
        D = C // self.n_head
        if self.fused and q.is_cuda and q.dtype == torch.float32 and _lib.attention_supported(T, D):
            p = self.attn_drop.p if self.training else 0.0
            if self._attn_seed is None or self._attn_seed.device != q.device:
                self._attn_seed = torch.randint(0, 2 ** 62, (1,), dtype=torch.int64, device=q.device)
            seed = self._attn_seed
            if p > 0.0:
                seed = self._attn_seed.clone()
                self._attn_seed.add_(1)  # on the device: graph replays advance it too
            y = _AttentionFn.apply(q, k, v, self.n_head, p, seed)
            h = self.c_proj(y.reshape(B * T, C)).reshape(B, T, C)
            return self.resid_drop(h)
        k = k.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        q = q.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        v = v.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        if self.fused:
            p = self.attn_drop.p if self.training else 0.0
            y = F.scaled_dot_product_attention(q, k, v, dropout_p=p, is_causal=True)
        else:
            att = (q @ k.transpose(-2, -1)) * (1.0 / math.sqrt(k.size(-1)))
            att = att.masked_fill(self.bias[:, :, :T, :T] == 0, float("-inf"))
            att = self.attn_drop(F.softmax(att, dim=-1))
            y = att @ v
        y = y.transpose(1, 2).contiguous().view(B, T, C)
        h = self.c_proj(y.reshape(B * T, C)).reshape(B, T, C)
        return self.resid_drop(h)


class IndexedFFN(nn.Module):
    """GaussianCDFNorm -> IndexedLinear up -> GELU -> IndexedLinear down."""

    def __init__(self, d_idx, ff_idx, K, dropout=0.1):
        super().__init__()
        self.d_idx = d_idx
        self.ff_idx = ff_idx
        self.cdf = GaussianCDFNorm(d_idx)
        self.up = IndexedLinear(d_idx, ff_idx, K)
        self.down = IndexedLinear(ff_idx, d_idx, K)
        self.act = nn.GELU()
        self.drop = nn.Dropout(dropout)

    def forward(self, x):
        shape = x.shape
        xf = x.reshape(-1, self.d_idx)
        if xf.dtype != torch.float32:
            xf = xf.float()
        if _observed(self.up):
            h = self.up(self.cdf(xf))  # a BucketTracker (hook or counting forward) sees up's input, as in the reference
        else:
            ln = self.cdf.ln
            h = _FnV2.apply(xf, ln.weight, ln.bias, ln.eps, self.up.table, self.up.bias, self.up.bw)
        h = self.act(h)
        h = self.down(h)
        return self.drop(h.reshape(shape))


class IndexedBlock(nn.Module):
    def __init__(self, d_idx, ff_idx, n_head, block_size, K, dropout=0.1, fused_attention=True):
        super().__init__()
        self.ln1 = nn.LayerNorm(d_idx)
        self.ln2 = nn.LayerNorm(d_idx)
        self.attn = IndexedAttention(d_idx, n_head, block_size, K, dropout, fused=fused_attention)
        self.ffn = IndexedFFN(d_idx, ff_idx, K, dropout)

    def forward(self, x):
        x = x + self.attn(layer_norm(self.ln1, x))
        x = x + self.ffn(layer_norm(self.ln2, x))
        return x


class IndexedGPT(nn.Module):
    """GPT with every linear op an IndexedLinear at d_idx (transformer_validation.py:295-385).
    The reference's constructor arguments; ``fused_attention`` (keyword, default
    True) selects IndexedAttention's fused form."""

    def __init__(self, vocab_size, block_size, n_layer, n_head, n_embd, K, dropout=0.1, *,
                 fused_attention=True):
        super().__init__()
        self.block_size = block_size
        self.ffn_type = "indexed"
        self.K = K
        d_idx, ff_idx = get_d_idx(n_embd, K, n_head)
        self.d_idx = d_idx
        self.ff_idx = ff_idx
        self.transformer = nn.ModuleDict({
            "wte": nn.Embedding(vocab_size, d_idx),
            "wpe": nn.Embedding(block_size, d_idx),
            "drop": nn.Dropout(dropout),
            "h": nn.ModuleList([IndexedBlock(d_idx, ff_idx, n_head, block_size, K, dropout, fused_attention)
                                for _ in range(n_layer)]),
            "ln_f": nn.LayerNorm(d_idx),
        })
        self.lm_head = nn.Linear(d_idx, vocab_size, bias=False)
        self._init_weights()
        for m in self.modules():
            if isinstance(m, IndexedLinear):
                nn.init.normal_(m.table, std=0.01)
                nn.init.zeros_(m.bias)
        n = sum(p.numel() for p in self.parameters())
        print(f"  IndexedGPT: n_embd={n_embd}→d_idx={d_idx} ff_idx={ff_idx} K={K} | "
              f"{n / 1e6:.2f}M params | Triton={TRITON_OK}")

    def _init_weights(self):
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, std=0.02)

    def forward(self, idx, targets=None):
        B, T = idx.shape
        x = self.transformer["drop"](self.transformer["wte"](idx) +
                                     self.transformer["wpe"](torch.arange(T, device=idx.device)))
        for block in self.transformer["h"]:
            x = block(x)
        x = layer_norm(self.transformer["ln_f"], x)
        logits = self.lm_head(x)
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.view(-1, logits.size(-1)), targets.view(-1))
        return logits, loss

    def get_indexed_layers(self):
        layers = []
        for blk in self.transformer["h"]:
            layers += [blk.attn.q_proj, blk.attn.k_proj, blk.attn.v_proj, blk.attn.c_proj, blk.ffn.up,
                       blk.ffn.down]
        return layers


class GraphedTrainStep:
    """One training step of ``model`` -- forward, loss, backward,
    clip_grad_norm_(clip), optimizer.step() -- captured once as a CUDA graph
    for a fixed (batch, ctx) and replayed.

        opt = torch.optim.AdamW(model.parameters(), lr, weight_decay=wd, capturable=True)
        step = GraphedTrainStep(model, opt, batch, ctx)
        loss = step(x, y)          # device int64 [batch, ctx]; returns the loss tensor

    The optimizer must be capturable.  Gradients live in the graph's memory
    pool and are overwritten (not accumulated) every step.  Construction runs
    ``warmup`` eager steps (on all-zero tokens) so that the optimizer state and
    the kernels are set up before capture, then puts the parameters back and
    zeroes the optimizer state: the model is unchanged until the first call.
    """

    def __init__(self, model, optimizer, batch_size, block_size, clip: float = 1.0, warmup: int = 3):
        dev = next(model.parameters()).device
        self.model, self.opt, self.clip = model, optimizer, clip
        self.x = torch.zeros(batch_size, block_size, dtype=torch.long, device=dev)
        self.y = torch.zeros(batch_size, block_size, dtype=torch.long, device=dev)
        saved = [p.detach().clone() for p in model.parameters()]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up: optimizer state, autograd, kernel set-up
            for _ in range(warmup):
                self.opt.zero_grad(set_to_none=True)
                _, loss = self.model(self.x, self.y)
                loss.backward()
                torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.clip)
                self.opt.step()
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.no_grad():
            for p, v in zip(model.parameters(), saved):
                p.copy_(v)
            for st in self.opt.state.values():
                for v in st.values():
                    if torch.is_tensor(v):
                        v.zero_()
        self.graph = torch.cuda.CUDAGraph()
        self.opt.zero_grad(set_to_none=True)
        with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
            _, self.loss = self.model(self.x, self.y)
            self.loss.backward()
            torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.clip)
            self.opt.step()

    def __call__(self, x, y):
        self.x.copy_(x, non_blocking=True)
        self.y.copy_(y, non_blocking=True)
        self.graph.replay()
        return self.loss
