"""The C-ABI library loads and exports every symbol include/aiwn_il.h declares;
argument checks that happen before any device work (no GPU needed)."""
import ctypes
import os
import re

import pytest

from aiwn_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "aiwn_il.h")).read()
    return sorted(set(re.findall(r"IL_API\s+[\w\s\*]+?\b(il_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("il_forward", "il_backward", "il_bins", "il_workspace_bytes", "il_adam_step",
              "il_status_string", "il_version", "il_check_device_status", "il_kernel_launches"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.library_path())
    for n in declared_symbols():
        assert hasattr(lib, n), n


def test_version_and_status_strings():
    assert "sm_100a" in _lib.version()
    lib = _lib.load()
    assert lib.il_status_string(0) == b"ok"
    for code in range(1, 10):
        assert lib.il_status_string(code) not in (b"ok", b"unknown status")
    assert lib.il_status_string(999) == b"unknown status"


@pytest.mark.parametrize("args,code", [
    # x_dtype invalid
    (dict(x_dtype=7), 2),
    # K < 2, IN < 1, OUT < 1, N < 0
    (dict(K=1), 1), (dict(IN=0), 1), (dict(OUT=0), 1), (dict(N=-1), 1),
    # bw not positive / not finite
    (dict(bw=0.0), 9), (dict(bw=-1.0), 9), (dict(bw=float("inf")), 9),
    # NULL x with N > 0
    (dict(x=None), 6),
])
def test_forward_argument_checks(args, code):
    lib = _lib.load()
    a = dict(x=ctypes.c_void_p(16), x_dtype=0, N=4, IN=3, OUT=2, K=8, bw=0.25)
    a.update(args)
    rc = lib.il_forward(a["x"], a["x_dtype"], ctypes.c_void_p(16), ctypes.c_void_p(16),
                        ctypes.c_void_p(16), a["N"], a["IN"], a["OUT"], a["K"], a["bw"], None)
    assert rc == code


def test_forward_empty_batch_is_noop():
    lib = _lib.load()
    assert lib.il_forward(None, 0, None, None, None, 0, 3, 2, 8, 0.25, None) == 0


def test_adam_argument_checks():
    lib = _lib.load()
    assert lib.il_adam_step(None, None, None, None, 0, 1e-3, 0.9, 0.999, 1e-8, 1, None) == 0
    assert lib.il_adam_step(None, None, None, None, 4, 1e-3, 0.9, 0.999, 1e-8, 0, None) == 1
    assert lib.il_adam_step(None, None, None, None, 4, 1e-3, 0.9, 0.999, 1e-8, 1, None) == 6


def test_workspace_query_is_host_only():
    n = _lib.workspace_bytes(131072, 20, 20, 512, 0)
    assert n >= 0


def test_cdf_entry_points_argument_checks():
    """il_cdf_forward / il_cdf_backward reject bad arguments before touching a device."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # empty batch: nothing to do
    assert lib.il_cdf_forward(None, None, None, 1e-5, None, None, None, None, None, None, 0, 4, 4, 8, 0.25,
                              None) == 0
    # NULL gamma with N > 0, negative eps, bad K
    assert lib.il_cdf_forward(p, None, p, 1e-5, p, p, p, p, p, p, 4, 4, 4, 8, 0.25, None) == 6
    assert lib.il_cdf_forward(p, p, p, -1.0, p, p, p, p, p, p, 4, 4, 4, 8, 0.25, None) == 9
    assert lib.il_cdf_forward(p, p, p, 1e-5, p, p, p, p, p, p, 4, 4, 4, 1, 0.25, None) == 1
    # in_d beyond the backward's per-block shared-memory sums, NULL inputs
    assert lib.il_cdf_backward(p, p, p, p, p, p, p, p, p, 4, 20000, None) == 1
    assert lib.il_cdf_backward(None, p, p, p, p, p, p, p, p, 4, 8, None) == 6


def test_layernorm_entry_points_argument_checks():
    """il_layernorm_forward / il_layernorm_backward reject bad arguments before touching a device."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.il_layernorm_forward(None, None, None, 1e-5, None, None, None, 0, 16, None) == 0  # empty batch
    assert lib.il_layernorm_forward(p, p, p, 1e-5, p, p, p, 4, 33, None) == 1  # in_d beyond 32
    assert lib.il_layernorm_forward(p, p, p, -1.0, p, p, p, 4, 16, None) == 9  # negative eps
    assert lib.il_layernorm_forward(p, None, p, 1e-5, p, p, p, 4, 16, None) == 6  # NULL gamma
    assert lib.il_layernorm_backward(p, p, p, p, p, p, p, p, 4, 0, None) == 1
    assert lib.il_layernorm_backward(None, p, p, p, p, p, p, p, 4, 16, None) == 6


def test_attention_entry_points_argument_checks():
    """il_attention_* reject unsupported shapes and dropout values before touching a device."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.il_attention_forward(p, p, p, p, p, 2, 256, 4, 3, 0.5, 0.0, None, None) == 1  # D = 3
    assert lib.il_attention_forward(p, p, p, p, p, 2, 2048, 4, 4, 0.5, 0.0, None, None) == 1  # T > 1024
    assert lib.il_attention_forward(p, p, p, p, p, 2, 600, 4, 16, 0.5, 0.0, None, None) == 1  # D = 16, T > 512
    assert lib.il_attention_forward(p, p, p, p, p, 2, 256, 4, 4, 0.5, 1.0, p, None) == 9  # p >= 1
    assert lib.il_attention_forward(p, p, p, p, p, 2, 256, 4, 4, 0.5, 0.1, None, None) == 6  # dropout, no seed
    assert lib.il_attention_backward(p, p, p, p, p, p, p, p, p, 0, 256, 4, 4, 0.5, 0.0, None, None) == 1
    assert _lib.attention_supported(256, 4) and not _lib.attention_supported(256, 5)


def test_bin_counts_argument_checks():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.il_bin_counts(None, 0, 0, 4, 8, 0.25, None, None) == 0
    assert lib.il_bin_counts(p, 0, 4, 4, 8, 0.25, None, None) == 6
    assert lib.il_bin_counts(p, 0, 4, 4, 20000, 2.0 / 20000, p, None) == 1
    assert lib.il_bin_counts(p, 5, 4, 4, 8, 0.25, p, None) == 2
