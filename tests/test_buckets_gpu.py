"""Bin-occupancy counts on the GPU (il_bin_counts, BucketTracker,
get_bucket_counts) against the bincount of the oracle's bit-exact bins."""
import math

import numpy as np
import pytest
import torch

from golden_io import bins_names, load_bins
from oracle import oracle

from aiwn_b200 import IndexedLinear, IndexedLinearV2, _lib
from aiwn_b200.buckets import BucketTracker, get_bucket_counts

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf16_from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("name", bins_names())
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_bin_counts_match_bincount_of_exact_bins(name, dt):
    """Sweeps include +-inf, NaN and |q| >= 2^63 (bin 0); two calls add up."""
    d = load_bins(name)
    K, bw = int(d["K"]), float(d["bw"])
    xs = d[f"x_{dt}"]
    x = (_bf16_from_bits(xs) if dt == "bf16" else torch.from_numpy(xs)).reshape(1, -1).to(DEV)
    ref = np.bincount(d[f"lo_{dt}"].reshape(-1), minlength=K)
    counts = torch.zeros(K, dtype=torch.int64, device=DEV)
    _lib.bin_counts(x, K, bw, counts)
    assert np.array_equal(counts.cpu().numpy(), ref)
    _lib.bin_counts(x, K, bw, counts)
    assert np.array_equal(counts.cpu().numpy(), 2 * ref)


def test_bucket_tracker_counts_eval_forwards_only():
    torch.manual_seed(0)
    K, IN, OUT = 64, 12, 8
    layer = IndexedLinear(IN, OUT, K).to(DEV)
    tr = BucketTracker(K)
    tr.register(layer)
    x = (torch.randn(3, 50, IN) * 0.6).to(DEV)
    layer.train()
    layer(x)
    assert tr.counts.sum() == 0  # the reference counts in eval mode only
    layer.eval()
    with torch.no_grad():
        layer(x)
        layer(x)
    lo, _, _ = oracle.bins(x.reshape(-1, IN).cpu().numpy(), K, 2.0 / K)
    ref = 2 * np.bincount(lo.reshape(-1), minlength=K).astype(np.float32)
    assert np.array_equal(tr.counts.numpy(), ref)
    p = ref / ref.sum()
    want = -(p * np.log(p + 1e-10)).sum() / math.log(K) * 100
    assert abs(tr.entropy() - want) < 1e-3
    tr.remove()
    with torch.no_grad():
        layer(x)
    assert np.array_equal(tr.counts.numpy(), ref)
    tr.reset()
    assert tr.counts.sum() == 0 and tr.entropy() == 0.0


def test_get_bucket_counts_v1_and_v2():
    torch.manual_seed(1)
    K, IN, OUT = 32, 16, 8
    x = (torch.randn(200, IN) * 1.3).to(DEV)
    v1 = IndexedLinear(IN, OUT, K).to(DEV)
    c1 = get_bucket_counts(v1, x, K)
    lo, _, _ = oracle.bins(x.cpu().numpy(), K, 2.0 / K)
    assert np.array_equal(c1.cpu().numpy(), np.bincount(lo.reshape(-1), minlength=K).astype(np.float32))
    v2 = IndexedLinearV2(IN, OUT, K).to(DEV)
    c2 = get_bucket_counts(v2, x, K)
    with torch.no_grad():
        xn = v2.cdf(x).cpu().numpy()
    lo2, _, _ = oracle.bins(xn, K, 2.0 / K)
    assert np.array_equal(c2.cpu().numpy(), np.bincount(lo2.reshape(-1), minlength=K).astype(np.float32))


def test_bin_counts_at_the_largest_k():
    """K = 16384 counters take 64 KB of shared memory per CTA (above the
    default 48 KB dynamic limit)."""
    K = 16384
    bw = 2.0 / K
    g = torch.Generator().manual_seed(77)
    x = torch.rand(4096, 24, generator=g) * 2.2 - 1.1
    lo, _, _ = oracle.bins(x.numpy(), K, bw)
    ref = np.bincount(lo.reshape(-1), minlength=K)
    counts = torch.zeros(K, dtype=torch.int64, device=DEV)
    _lib.bin_counts(x.to(DEV), K, bw, counts)
    assert np.array_equal(counts.cpu().numpy(), ref)


@pytest.mark.parametrize("shape", [(131072, 20, 20, 512, "uniform", "f32"), (131072, 20, 20, 128, "tanh", "bf16"),
                                   (16384, 16, 16, 128, "uniform", "f32"), (3000, 16, 48, 128, "wide", "f32"),
                                   (600, 300, 8, 256, "wide", "f32")],
                         ids=["c3", "c2_bf16", "c5", "qkv_wide", "streamed_table"])
def test_forward_counts_equal_bincount_and_plain_forward(shape):
    """il_forward_counts: the histogram of the forward's own bins (fused into
    the token kernel; the streamed-table shape takes forward + counting pass)
    equals the oracle's bincount, and the output equals il_forward's bit for
    bit."""
    N, IN, OUT, K, xdist, dt = shape
    g = torch.Generator().manual_seed(N + IN + K)
    if xdist == "uniform":
        x = torch.rand(N, IN, generator=g) * 2 - 1
    elif xdist == "tanh":
        x = torch.tanh(torch.randn(N, IN, generator=g))
    else:
        x = torch.rand(N, IN, generator=g) * 3 - 1.5
    if dt == "bf16":
        x = x.to(torch.bfloat16)
    table = torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)
    bias = torch.randn(OUT, generator=g) * 0.1
    xd, td, bd = x.to(DEV), table.to(DEV), bias.to(DEV)
    bw = 2.0 / K
    counts = torch.zeros(K, dtype=torch.int64, device=DEV)
    o1 = torch.empty(N, OUT, device=DEV)
    o2 = torch.empty(N, OUT, device=DEV)
    _lib.forward(xd, td, bd, o1, bw, counts=counts)
    _lib.forward(xd, td, bd, o2, bw)
    assert torch.equal(o1, o2)
    xn = x.contiguous().view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else x.numpy()
    lo, _, _ = oracle.bins(xn, K, bw, x_dtype=dt)
    ref = np.bincount(lo.reshape(-1), minlength=K)
    assert np.array_equal(counts.cpu().numpy(), ref)
    _lib.forward(xd, td, bd, o1, bw, counts=counts)  # accumulates
    assert np.array_equal(counts.cpu().numpy(), 2 * ref)
