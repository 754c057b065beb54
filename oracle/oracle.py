"""CPU oracle for IndexedLinear -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes wrapper over ``il_oracle.c`` (a C restatement of the
reference's eager path, ``aiwn/layers/indexed_linear.py:173-182``, and of
PyTorch autograd's backward of it).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this module, and only as the checker or the timed CPU baseline; the
``aiwn_b200`` package never does.

Parity of this oracle with the reference is pinned by
``tests/test_oracle_golden.py`` against ``tests/golden/*.npz``, which
``tests/golden/make_golden.py`` produced by running the reference itself.

Array conventions: fp32 arrays are ``np.float32``; bf16 arrays are the raw
bit patterns as ``np.uint16`` (``x_dtype="bf16"``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libil_oracle.so")
_lib = None

DT = {"f32": 0, "bf16": 1}


def build(force: bool = False) -> str:
    """Compile ``libil_oracle.so`` with the committed Makefile."""
    src = os.path.join(_HERE, "il_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i64, f64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_int
        lib.il_oracle_bins.argtypes = [vp, ci, i64, i64, i64, f64, vp, vp, vp]
        lib.il_oracle_bins.restype = None
        lib.il_oracle_forward.argtypes = [vp, ci, vp, vp, vp, i64, i64, i64, i64, f64, ci]
        lib.il_oracle_forward.restype = None
        lib.il_oracle_backward.argtypes = [vp, vp, ci, vp, vp, vp, vp, i64, i64, i64, i64, f64, ci]
        lib.il_oracle_backward.restype = ci
        lib.il_oracle_cdf_forward.argtypes = [vp, vp, vp, f64, i64, i64, vp, vp, vp]
        lib.il_oracle_cdf_forward.restype = None
        lib.il_oracle_cdf_backward.argtypes = [vp, vp, vp, vp, f64, i64, i64, vp, vp, vp]
        lib.il_oracle_cdf_backward.restype = ci
        lib.il_oracle_adam.argtypes = [vp, vp, vp, vp, i64, f64, f64, f64, f64, i64]
        lib.il_oracle_adam.restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _x(x, x_dtype):
    return _c(x, np.uint16 if x_dtype == "bf16" else np.float32)


def bins(x, K: int, bw: float, x_dtype: str = "f32"):
    """(lo int32, hi int32, fr fp32), each shaped like x  (reference IL:175-177)."""
    x = _x(x, x_dtype)
    lo = np.empty(x.shape, np.int32)
    hi = np.empty(x.shape, np.int32)
    fr = np.empty(x.shape, np.float32)
    n = x.shape[0] if x.ndim == 2 else 1
    m = x.shape[-1] if x.ndim >= 1 else 1
    _load().il_oracle_bins(_ptr(x), DT[x_dtype], n, m, K, bw, _ptr(lo), _ptr(hi), _ptr(fr))
    return lo, hi, fr


def forward(x, table, bias, bw: float, x_dtype: str = "f32", nthreads: int = 0):
    """fp32 out[N, OUT]  (reference IL:173-182)."""
    x = _x(x, x_dtype)
    table = _c(table, np.float32)
    bias = _c(bias, np.float32)
    N, IN = x.shape
    K, IN2, OUT = table.shape
    assert IN2 == IN and bias.shape == (OUT,)
    out = np.empty((N, OUT), np.float32)
    _load().il_oracle_forward(_ptr(x), DT[x_dtype], _ptr(table), _ptr(bias), _ptr(out),
                              N, IN, OUT, K, bw, nthreads)
    return out


def backward(go, x, table, bw: float, x_dtype: str = "f32", nthreads: int = 0,
             want=("gx", "gt", "gb")):
    """(gx, gt, gb): autograd's gradients of the eager forward.

    gx has x's dtype (uint16 bit patterns for bf16); gt, gb are fp32.
    """
    go = _c(go, np.float32)
    x = _x(x, x_dtype)
    table = _c(table, np.float32)
    N, IN = x.shape
    K, _, OUT = table.shape
    gx = np.empty(x.shape, x.dtype) if "gx" in want else None
    gt = np.empty(table.shape, np.float32) if "gt" in want else None
    gb = np.empty((OUT,), np.float32) if "gb" in want else None
    rc = _load().il_oracle_backward(_ptr(go), _ptr(x), DT[x_dtype], _ptr(table), _ptr(gx),
                                    _ptr(gt), _ptr(gb), N, IN, OUT, K, bw, nthreads)
    if rc != 0:
        raise MemoryError("oracle backward: allocation failed")
    return gx, gt, gb


def cdf_forward(x, gamma, beta, eps: float):
    """(xn, mean, rstd) of the GaussianCDFNorm prologue
    (aiwn/layers/indexed_linear_v2.py:19-37), fp32."""
    x = _c(x, np.float32)
    gamma = _c(gamma, np.float32)
    beta = _c(beta, np.float32)
    N, IN = x.shape
    xn = np.empty_like(x)
    mean = np.empty(N, np.float32)
    rstd = np.empty(N, np.float32)
    _load().il_oracle_cdf_forward(_ptr(x), _ptr(gamma), _ptr(beta), eps, N, IN, _ptr(xn), _ptr(mean), _ptr(rstd))
    return xn, mean, rstd


def cdf_backward(g, x, gamma, beta, eps: float):
    """(dx, dgamma, dbeta): autograd's backward of the prologue given g = dL/dxn."""
    g = _c(g, np.float32)
    x = _c(x, np.float32)
    gamma = _c(gamma, np.float32)
    beta = _c(beta, np.float32)
    N, IN = x.shape
    dx = np.empty_like(x)
    dgamma = np.empty(IN, np.float32)
    dbeta = np.empty(IN, np.float32)
    rc = _load().il_oracle_cdf_backward(_ptr(g), _ptr(x), _ptr(gamma), _ptr(beta), eps, N, IN, _ptr(dx),
                                        _ptr(dgamma), _ptr(dbeta))
    if rc != 0:
        raise MemoryError("oracle cdf backward: allocation failed")
    return dx, dgamma, dbeta


def adam(p, g, m, v, lr, beta1, beta2, eps, step):
    """In-place fp32 Adam step (torch.optim.Adam defaults, single-tensor order)."""
    for a in (p, g, m, v):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    _load().il_oracle_adam(_ptr(p), _ptr(g), _ptr(m), _ptr(v), p.size, lr, beta1, beta2, eps, step)


# ---- bf16 helpers (bit patterns) -------------------------------------------

def f32_to_bf16_bits(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (as torch does)."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)
