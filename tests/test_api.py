"""Host-side API of the drop-in (no GPU needed)."""
import math

import pytest
import torch

import aiwn_b200
from aiwn_b200 import IndexedLinear, StandardLinear, indexed_dims, indexed_lr
from aiwn_b200.layers import indexed_linear as il


def test_exports_match_reference_names():
    # names imported by the reference's consumers (timing.py:9-10, config.py:25, ...)
    for name in ("IndexedLinear", "indexed_dims", "indexed_lr", "TRITON_OK", "_Fn", "triton_available"):
        assert hasattr(il, name)
    assert hasattr(aiwn_b200.layers, "StandardLinear")


@pytest.mark.parametrize("d,ff,K,expect", [
    (256, 1024, 16, (64, 256, 16)),     # C1 sizing
    (256, 1024, 128, (20, 80, 1)),      # C2 sizing (in=out=20, not ~23)
    (512, 2048, 512, (20, 80, 0 + 1)),  # C3 sizing
    (256, 1024, 4, (128, 512, 64)),
    (64, 256, 2, (44, 176, 44)),
    (8, 32, 512, (4, 16, 1)),           # floor at n_heads
])
def test_indexed_dims_known_answers(d, ff, K, expect):
    assert indexed_dims(d, ff, K) == expect


def test_indexed_dims_matches_formula_grid():
    for d in (32, 64, 100, 256, 512, 1024):
        for K in (2, 3, 4, 16, 64, 100, 128, 512):
            for h in (1, 2, 4, 8):
                s = math.sqrt(K)
                di = max(h, (int(d / s) // h) * h)
                assert indexed_dims(d, 4 * d, K, n_heads=h) == (di, 4 * di, max(1, di // max(1, int(round(s)))))


def test_indexed_lr():
    assert indexed_lr(1e-3, 2) == pytest.approx(1e-3)
    assert indexed_lr(1e-3, 512) == pytest.approx(1e-3 * 16)


def test_ctor_attributes_and_init():
    torch.manual_seed(0)
    m = IndexedLinear(20, 80, 512)
    assert (m.K, m.bw, m.in_dim, m.out_dim) == (512, 2.0 / 512, 20, 80)
    assert m.table.shape == (512, 20, 80) and m.bias.shape == (80,)
    assert m.table.dtype == torch.float32 and torch.all(m.bias == 0)
    std = math.sqrt(math.sqrt(3.0 / 20) * (2.0 / 512))
    assert abs(m.table.std().item() / std - 1) < 0.02
    assert m.flops() == 2 * 20 * 80 and m.active_bytes() == 2 * 20 * 80 * 4
    with pytest.raises(AssertionError):
        IndexedLinear(4, 4, 1)


def test_same_init_stream_as_reference():
    # the reference draws table = randn(K, in, out) * std from the global RNG
    torch.manual_seed(123)
    m = IndexedLinear(8, 6, 16)
    torch.manual_seed(123)
    t = torch.randn(16, 8, 6) * math.sqrt(math.sqrt(3.0 / 8) * (2.0 / 16))
    assert torch.equal(m.table.detach(), t)


def test_state_dict_keys():
    m = IndexedLinear(4, 3, 8)
    assert set(m.state_dict()) == {"table", "bias"}
    s = StandardLinear(4, 3)
    assert set(s.state_dict()) == {"lin.weight", "lin.bias"}
    assert s.flops() == 24


def test_cpu_tensor_raises_no_fallback():
    m = IndexedLinear(4, 3, 8)
    with pytest.raises(RuntimeError):
        m(torch.zeros(2, 4))
    with pytest.raises(RuntimeError):
        m._eager(torch.zeros(2, 4))
