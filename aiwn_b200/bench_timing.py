"""Layer timing harness -- drop-in for ``aiwn.bench.timing`` (bench_fn,
bench_layer, aiwn/bench/timing.py:19-95) plus the reference's high-K timing
grid (aiwn/experiments/high_k_sweep.py:55-59) run through this package.

``bench_fn`` and ``bench_layer`` keep the reference's signatures, timing
method (host clock around each call with a device synchronisation on both
sides; median and 95th percentile in ms) and result keys, so a table produced
here reads like the reference's.  The IndexedLinear step goes through ``_Fn``
(the sm_100a kernels), as the reference's does through its own ``_Fn`` when
``TRITON_OK``.

    python -m aiwn_b200.bench_timing --out high_k.csv [--n_warm 20 --n_bench 100]

writes one CSV row per grid point (B, d, K, seq, d_idx, ff_idx, then the
bench_layer keys).  The grid's perplexity columns belong to the reference's
accuracy study (training on text data), which this package does not rebuild.
"""
from __future__ import annotations

import argparse
import csv
import time
from itertools import product

import numpy as np
import torch

from .layers import IndexedLinear, StandardLinear, indexed_dims
from .layers.indexed_linear import TRITON_OK, _Fn

# the reference's high-K grid
K_VALUES = [32, 64, 128, 256, 512]
D_MODELS = [256, 384, 512]
BATCH_SIZES = [32, 64]
SEQ_LENS = [256, 1024, 4096]
N_HEADS = 4


def sync(device: torch.device):
    """Synchronise CUDA if applicable."""
    if device.type == "cuda":
        torch.cuda.synchronize()


def bench_fn(fn, n_warm: int, n_bench: int, device: torch.device):
    """Time ``fn`` with device synchronisation; returns (median_ms, p95_ms)."""
    for _ in range(n_warm):
        fn()
    sync(device)
    times = []
    for _ in range(n_bench):
        sync(device)
        t0 = time.perf_counter()
        fn()
        sync(device)
        times.append((time.perf_counter() - t0) * 1000)
    return float(np.median(times)), float(np.percentile(times, 95))


def bench_layer(layer_std: StandardLinear, layer_idx: IndexedLinear, B: int, IN: int, OUT: int, K: int,
                n_warm: int, n_bench: int, device: torch.device) -> dict:
    """Timing and FLOP metrics of a (StandardLinear, IndexedLinear) pair on B
    rows, with the reference's keys (aiwn/bench/timing.py:38-95)."""
    x_std = torch.randn(B, IN, device=device, requires_grad=True)
    x_idx = torch.empty(B, layer_idx.in_dim, device=device).uniform_(-1, 1).requires_grad_(True)

    fwd_std, _ = bench_fn(lambda: layer_std(x_std), n_warm, n_bench, device)
    fwd_idx, _ = bench_fn(lambda: layer_idx(x_idx), n_warm, n_bench, device)

    def full_std():
        xs = x_std.detach().requires_grad_(True)
        layer_std(xs).sum().backward()

    def full_idx():
        xi = x_idx.detach().requires_grad_(True)
        t = layer_idx.table.detach().requires_grad_(True)
        b = layer_idx.bias.detach().requires_grad_(True)
        _Fn.apply(xi, t, b, layer_idx.bw).sum().backward()

    step_std_ms, _ = bench_fn(full_std, n_warm, n_bench, device)
    step_idx_ms, _ = bench_fn(full_idx, n_warm, n_bench, device)
    flops_std = layer_std.flops()
    flops_idx = layer_idx.flops()
    return {
        "fwd_std_ms": fwd_std,
        "fwd_idx_ms": fwd_idx,
        "fwd_speedup": fwd_std / fwd_idx,
        "step_std_ms": step_std_ms,
        "step_idx_ms": step_idx_ms,
        "step_speedup": step_std_ms / step_idx_ms,
        "flops_std": flops_std,
        "flops_idx": flops_idx,
        "flop_ratio": flops_std / flops_idx,
        "tflops_std": flops_std * B / fwd_std / 1e9,
        "tflops_idx": flops_idx * B / fwd_idx / 1e9,
        "idx_faster_fwd": fwd_idx < fwd_std,
        "idx_faster_step": step_idx_ms < step_std_ms,
        "active_kb": layer_idx.active_bytes() / 1024,
    }


def high_k_grid(device: torch.device, n_warm: int = 20, n_bench: int = 100, fixed_dim: bool = False,
                batches=BATCH_SIZES, d_models=D_MODELS, k_values=K_VALUES, seq_lens=SEQ_LENS):
    """Yields one dict per point of the reference's high-K grid: N = B*seq
    rows through StandardLinear(d, 4d) and IndexedLinear(d_idx, ff_idx, K)
    with indexed_dims' sizing (or d_idx = d with ``fixed_dim``)."""
    for B, d_std, K, seq in product(batches, d_models, k_values, seq_lens):
        if fixed_dim:
            d_idx, ff_idx = d_std, 4 * d_std
        else:
            d_idx, ff_idx, _ = indexed_dims(d_std, 4 * d_std, K, N_HEADS)
        N = B * seq
        layer_std = StandardLinear(d_std, 4 * d_std).to(device)
        layer_idx = IndexedLinear(d_idx, ff_idx, K).to(device)
        r = bench_layer(layer_std, layer_idx, N, d_std, 4 * d_std, K, n_warm, n_bench, device)
        yield {"B": B, "d": d_std, "K": K, "seq": seq, "d_idx": d_idx, "ff_idx": ff_idx, **r}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="high_k.csv")
    ap.add_argument("--n_warm", type=int, default=20)
    ap.add_argument("--n_bench", type=int, default=100)
    ap.add_argument("--fixed_dim", action="store_true")
    args = ap.parse_args()
    if not TRITON_OK or not torch.cuda.is_available():
        raise SystemExit("the timing grid needs the sm_100a kernels and a CUDA device")
    dev = torch.device("cuda")
    rows = []
    with open(args.out, "w", newline="") as f:
        w = None
        for row in high_k_grid(dev, args.n_warm, args.n_bench, args.fixed_dim):
            if w is None:
                w = csv.DictWriter(f, fieldnames=list(row))
                w.writeheader()
            w.writerow(row)
            f.flush()
            rows.append(row)
            print(f"B={row['B']:>3} d={row['d']:>3} K={row['K']:>3} seq={row['seq']:>4} d_idx={row['d_idx']:>3} | "
                  f"fwd {row['fwd_std_ms']:.3f}/{row['fwd_idx_ms']:.3f} ms x{row['fwd_speedup']:.2f} | "
                  f"step {row['step_std_ms']:.3f}/{row['step_idx_ms']:.3f} ms x{row['step_speedup']:.2f}",
                  flush=True)
    sp = np.array([r["step_speedup"] for r in rows])
    print(f"{len(rows)} points; step speedup over StandardLinear: median {np.median(sp):.2f}, "
          f"min {sp.min():.2f}, max {sp.max():.2f}")


if __name__ == "__main__":
    main()
