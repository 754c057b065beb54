"""Seeded inputs for the parity tests and the benchmark (CPU generators, so the
oracle and the CUDA kernels see identical bits)."""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Case:
    name: str
    N: int
    IN: int
    OUT: int
    K: int
    xdist: str = "uniform"      # uniform | tanh_normal | clamp_normal | wide
    dtype: str = "f32"          # f32 | bf16
    bias_scale: float = 0.0
    seed: int = 0


# configurations of the benchmark list (sizes at which the oracle finishes in seconds)
CASES = [
    Case("c1_d256_k16", 2048, 64, 64, 16, "uniform", "f32", 0.0, 1),
    Case("c2_d256_k128_bf16", 131072, 20, 20, 128, "tanh_normal", "bf16", 0.1, 2),
    Case("c3_d512_k512", 131072, 20, 20, 512, "uniform", "f32", 0.1, 3),
    Case("c3_refshape_20x80", 131072, 20, 80, 512, "uniform", "f32", 0.1, 4),
    Case("c2_refshape_20x80_bf16", 32768, 20, 80, 128, "tanh_normal", "bf16", 0.1, 5),
    Case("c4_k64_1024_small", 192, 1024, 1024, 64, "clamp_normal", "f32", 0.1, 6),
    Case("c5_q_16x16", 16384, 16, 16, 128, "wide", "f32", 0.1, 7),
    Case("c5_up_16x8", 16384, 16, 8, 128, "uniform", "f32", 0.1, 8),
    Case("c5_down_8x16", 16384, 8, 16, 128, "uniform", "f32", 0.1, 9),
    Case("c5_q_16x16_bf16", 16384, 16, 16, 128, "wide", "bf16", 0.1, 10),
]

# shapes that exercise the edges: tiny dims, odd OUT, non-power-of-two K, x out of range
EDGE_CASES = [
    Case("n1", 1, 20, 20, 512, "uniform", "f32", 0.3, 20),
    Case("n7_in1_out1_k2", 7, 1, 1, 2, "wide", "f32", 0.3, 21),
    Case("out3_k3", 513, 5, 3, 3, "wide", "f32", 0.3, 22),
    Case("out5_k7_bf16", 300, 6, 5, 7, "wide", "bf16", 0.3, 23),
    Case("k100_out12", 1000, 8, 12, 100, "wide", "f32", 0.3, 24),
    Case("k100_out12_bf16", 1000, 8, 12, 100, "wide", "bf16", 0.3, 25),
    Case("in33_out36_k64", 777, 33, 36, 64, "wide", "f32", 0.3, 26),
    Case("out4_k512", 4099, 20, 4, 512, "uniform", "f32", 0.3, 27),
    Case("out132_k16", 999, 7, 132, 16, "wide", "f32", 0.3, 28),
    Case("k3000_out8", 2000, 3, 8, 3000, "uniform", "f32", 0.3, 29),
    Case("out256_k32_jranges", 700, 6, 256, 32, "wide", "f32", 0.3, 30),
    Case("out256_k64_bf16", 500, 8, 256, 64, "wide", "bf16", 0.3, 31),
    Case("out176_k32_jranges", 500, 12, 176, 32, "wide", "f32", 0.3, 34),  # 11 j-ranges of 16 columns
    # out_d 48: the sorted backward's 12-lane groups (IndexedGPT's fused q|k|v projection)
    Case("out48_k128_qkv", 3000, 16, 48, 128, "wide", "f32", 0.3, 36),
    Case("out48_k128_qkv_bf16", 3000, 16, 48, 128, "wide", "bf16", 0.3, 37),
    # too large to keep resident: the streamed forward (partial last column chunk, partial token tile)
    Case("stream_in300_out8_k256", 600, 300, 8, 256, "wide", "f32", 0.3, 32),
    Case("stream_in300_out8_k256_bf16", 600, 300, 8, 256, "wide", "bf16", 0.3, 33),
]


def make_inputs(c: Case):
    """(x, table, bias, go) as CPU tensors; x is bf16 for dtype 'bf16'."""
    g = torch.Generator().manual_seed(1000 + c.seed)
    if c.xdist == "uniform":
        x = torch.rand(c.N, c.IN, generator=g) * 2 - 1
    elif c.xdist == "tanh_normal":
        x = torch.tanh(torch.randn(c.N, c.IN, generator=g))
    elif c.xdist == "clamp_normal":
        x = (torch.randn(c.N, c.IN, generator=g) * 0.5).clamp(-1, 1)
    elif c.xdist == "wide":
        x = torch.rand(c.N, c.IN, generator=g) * 3 - 1.5
    else:
        raise ValueError(c.xdist)
    if c.dtype == "bf16":
        x = x.to(torch.bfloat16)
    table = torch.randn(c.K, c.IN, c.OUT, generator=g) / math.sqrt(c.IN)
    bias = torch.randn(c.OUT, generator=g) * c.bias_scale
    go = torch.randn(c.N, c.OUT, generator=g)
    return x, table, bias, go


def x_numpy(x: torch.Tensor) -> np.ndarray:
    if x.dtype == torch.bfloat16:
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)
    return x.contiguous().numpy()


def to_numpy_grad(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
