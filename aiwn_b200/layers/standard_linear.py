"""StandardLinear -- the nn.Linear comparator of aiwn/layers/standard_linear.py:1-14,
kept (same attribute name ``lin``, so state_dicts match) so that benchmark code
written against the reference imports unchanged."""
import torch.nn as nn


class StandardLinear(nn.Module):
    def __init__(self, in_d: int, out_d: int):
        super().__init__()
        self.lin = nn.Linear(in_d, out_d, bias=True)

    def forward(self, x):
        return self.lin(x)

    def flops(self) -> int:
        return 2 * self.lin.in_features * self.lin.out_features
