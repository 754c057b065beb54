"""The timing harness (drop-in for aiwn.bench.timing) on one small grid point."""
import pytest
import torch

from aiwn_b200 import IndexedLinear, StandardLinear
from aiwn_b200.bench_timing import bench_layer, high_k_grid

pytestmark = pytest.mark.gpu

KEYS = {"fwd_std_ms", "fwd_idx_ms", "fwd_speedup", "step_std_ms", "step_idx_ms", "step_speedup", "flops_std",
        "flops_idx", "flop_ratio", "tflops_std", "tflops_idx", "idx_faster_fwd", "idx_faster_step", "active_kb"}


def test_bench_layer_keys_and_values():
    dev = torch.device("cuda")
    r = bench_layer(StandardLinear(64, 256).to(dev), IndexedLinear(16, 64, 16).to(dev), 512, 64, 256, 16, 1, 3,
                    dev)
    assert set(r) == KEYS
    assert r["fwd_idx_ms"] > 0 and r["step_idx_ms"] > 0
    assert r["flop_ratio"] == (2 * 64 * 256) / (2 * 16 * 64)


def test_high_k_grid_point():
    rows = list(high_k_grid(torch.device("cuda"), 1, 2, batches=[32], d_models=[256], k_values=[64],
                            seq_lens=[256]))
    assert len(rows) == 1 and rows[0]["d_idx"] == 32 and rows[0]["ff_idx"] == 128
