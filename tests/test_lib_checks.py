"""The ctypes binding rejects tensors of the wrong dtype, shape or device
before any C call, so a mismatch can never reach a kernel (which trusts the
sizes it is given).  CPU tensors suffice: the checks run before the device
check, and none of these calls launches anything."""
import pytest
import torch

from aiwn_b200 import _lib
from aiwn_b200._lib import ILError

N, IN, OUT, K = 64, 6, 5, 16


def _good():
    x = torch.rand(N, IN) * 2 - 1
    table = torch.randn(K, IN, OUT)
    bias = torch.zeros(OUT)
    out = torch.empty(N, OUT)
    go = torch.randn(N, OUT)
    gx = torch.empty(N, IN)
    gt = torch.empty(K, IN, OUT)
    gb = torch.empty(OUT)
    return x, table, bias, out, go, gx, gt, gb


def test_forward_rejects_mismatches():
    x, table, bias, out, *_ = _good()
    cases = [
        (x.half(), table, bias, out, "dtype"),                       # unsupported x dtype
        (x, table.to(torch.bfloat16), bias, out, "dtype"),           # module .to(bfloat16)
        (x, table.double(), bias, out, "dtype"),
        (x, table, torch.zeros(OUT + 1), out, "shape"),              # bias too long
        (x, table, bias.to(torch.bfloat16), out, "dtype"),
        (x, table, bias, torch.empty(N - 1, OUT), "shape"),          # out too short
        (x, table, bias, torch.empty(N, OUT, dtype=torch.bfloat16), "dtype"),
        (x[:, :IN - 1].contiguous(), table, bias, out, "in_d"),      # x and table disagree
        (x, table.reshape(K, IN * OUT), bias, out, "table"),
    ]
    for xx, tt, bb, oo, what in cases:
        with pytest.raises(ILError, match=what):
            _lib.forward(xx, tt, bb, oo, 2.0 / K)


def test_backward_rejects_mismatches():
    x, table, bias, out, go, gx, gt, gb = _good()
    bad = {
        "go": (torch.randn(N, OUT + 1), "shape"),
        "go_dtype": (go.to(torch.bfloat16), "dtype"),
        "gx": (torch.empty(N, IN, dtype=torch.bfloat16), "dtype"),   # gx must match x's dtype
        "gt": (torch.empty(K, IN, OUT + 1), "shape"),
        "gt_dtype": (gt.half(), "dtype"),
        "gb": (torch.empty(OUT - 1), "shape"),
    }
    for key, (t, what) in bad.items():
        args = dict(go=go, x=x, table=table, gx=gx, gt=gt, gb=gb)
        args[key.split("_")[0]] = t
        with pytest.raises(ILError, match=what):
            _lib.backward(args["go"], args["x"], args["table"], args["gx"], args["gt"], args["gb"], 2.0 / K)
    with pytest.raises(ILError, match="uint8"):
        _lib.backward(go, x, table, gx, gt, gb, 2.0 / K, workspace=torch.empty(4))


def test_valid_cpu_tensors_reach_the_device_check():
    """Correct dtypes and shapes pass the checks and stop at the CUDA check:
    there is no CPU path."""
    x, table, bias, out, go, gx, gt, gb = _good()
    with pytest.raises(ILError, match="CUDA"):
        _lib.forward(x, table, bias, out, 2.0 / K)
    with pytest.raises(ILError, match="CUDA"):
        _lib.backward(go, x, table, gx, gt, gb, 2.0 / K)
    # any gradient may be omitted
    with pytest.raises(ILError, match="CUDA"):
        _lib.backward(go, x, table, None, gt, None, 2.0 / K)


def test_prologue_layernorm_attention_adam_checks():
    x = torch.rand(N, IN)
    g, b = torch.ones(IN), torch.zeros(IN)
    mean, rstd = torch.empty(N), torch.empty(N)
    table = torch.randn(K, IN, OUT)
    with pytest.raises(ILError, match="shape"):
        _lib.cdf_forward(x, torch.ones(IN + 1), b, 1e-5, table, torch.zeros(OUT), torch.empty(N, IN), mean, rstd,
                         torch.empty(N, OUT), 2.0 / K)
    with pytest.raises(ILError, match="shape"):
        _lib.cdf_backward(torch.empty(N, IN), x, g, b, torch.empty(N - 1), rstd, torch.empty(N, IN), None, None)
    with pytest.raises(ILError, match="shape"):
        _lib.layernorm_forward(x, g, b, 1e-5, torch.empty(N, IN + 1), mean, rstd)
    with pytest.raises(ILError, match="dtype"):
        _lib.layernorm_backward(torch.empty(N, IN).double(), x, g, mean, rstd, None, None, None)
    B, T, H, D = 2, 8, 2, 4
    q = torch.randn(B, T, H * D)
    with pytest.raises(ILError, match="shape"):
        _lib.attention_forward(q, q, torch.randn(B, T + 1, H * D), torch.empty_like(q), torch.empty(B, H, T), H,
                               0.5, 0.0, None)
    with pytest.raises(ILError, match="seed"):
        _lib.attention_forward(q, q, q, torch.empty_like(q), torch.empty(B, H, T), H, 0.5, 0.1, None)
    with pytest.raises(ILError, match="same number"):
        _lib.adam_step(torch.zeros(10), torch.zeros(10), torch.zeros(9), torch.zeros(10), 1e-3, 0.9, 0.999,
                       1e-8, 1)


def test_devices_must_agree():
    x, table, bias, out, *_ = _good()
    meta = torch.empty(N, OUT, device="meta")
    with pytest.raises(ILError, match="different devices"):
        _lib.forward(x, table, bias, meta, 2.0 / K)
