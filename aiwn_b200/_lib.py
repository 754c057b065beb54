"""ctypes binding of the C ABI in ``include/aiwn_il.h`` (``libaiwn_il.so``).

The shared library is built in-tree by ``python -m aiwn_b200.csrc.build``
(or ``__graft_entry__.build()``).  There is no fallback: if the library is
missing or the tensors are not on a B200, every call raises ``ILError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libaiwn_il.so")
_lib = None
_lock = threading.Lock()

IL_F32, IL_BF16 = 0, 1
_DTYPES = {torch.float32: IL_F32, torch.bfloat16: IL_BF16}


class ILError(RuntimeError):
    """A status other than IL_OK returned by the C ABI."""


def library_path() -> str:
    return _PATH


def load():
    """Load ``libaiwn_il.so`` once and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_PATH):
            raise ILError(f"{_PATH} is not built; run `python aiwn_b200/csrc/build.py`")
        lib = ctypes.CDLL(_PATH)
        vp, i64, f64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_int
        lib.il_status_string.argtypes = [ci]
        lib.il_status_string.restype = ctypes.c_char_p
        lib.il_version.argtypes = []
        lib.il_version.restype = ctypes.c_char_p
        lib.il_forward.argtypes = [vp, ci, vp, vp, vp, i64, i64, i64, i64, f64, vp]
        lib.il_forward.restype = ci
        lib.il_forward_counts.argtypes = [vp, ci, vp, vp, vp, i64, i64, i64, i64, f64, vp, vp]
        lib.il_forward_counts.restype = ci
        lib.il_workspace_bytes.argtypes = [i64, i64, i64, i64, ci]
        lib.il_workspace_bytes.restype = i64
        lib.il_backward.argtypes = [vp, vp, ci, vp, vp, vp, vp, i64, i64, i64, i64, f64, vp, i64, vp]
        lib.il_backward.restype = ci
        lib.il_backward_accumulate.argtypes = lib.il_backward.argtypes
        lib.il_backward_accumulate.restype = ci
        lib.il_bins.argtypes = [vp, ci, i64, i64, i64, f64, vp, vp, vp, vp]
        lib.il_bins.restype = ci
        lib.il_adam_step.argtypes = [vp, vp, vp, vp, i64, f64, f64, f64, f64, i64, vp]
        lib.il_adam_step.restype = ci
        lib.il_cdf_forward.argtypes = [vp, vp, vp, f64, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f64, vp]
        lib.il_cdf_forward.restype = ci
        lib.il_cdf_backward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
        lib.il_cdf_backward.restype = ci
        lib.il_layernorm_forward.argtypes = [vp, vp, vp, f64, vp, vp, vp, i64, i64, vp]
        lib.il_layernorm_forward.restype = ci
        lib.il_layernorm_backward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
        lib.il_layernorm_backward.restype = ci
        lib.il_attention_forward.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, f64, f64, vp, vp]
        lib.il_attention_forward.restype = ci
        lib.il_attention_backward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f64, f64,
                                              vp, vp]
        lib.il_attention_backward.restype = ci
        lib.il_attention_dropout_mask.argtypes = [vp, i64, i64, i64, f64, vp, vp]
        lib.il_attention_dropout_mask.restype = ci
        lib.il_bin_counts.argtypes = [vp, ci, i64, i64, i64, f64, vp, vp]
        lib.il_bin_counts.restype = ci
        lib.il_allreduce_scratch_bytes.argtypes = [i64, ci]
        lib.il_allreduce_scratch_bytes.restype = i64
        lib.il_allreduce_sum.argtypes = [vp, vp, i64, ci, ci, f64, f64, vp]
        lib.il_allreduce_sum.restype = ci
        lib.il_allreduce_sum_noalloc.argtypes = [vp, i64, ci, f64, vp]
        lib.il_allreduce_sum_noalloc.restype = ci
        lib.il_kernel_launches.argtypes = []
        lib.il_kernel_launches.restype = i64
        lib.il_check_device_status.argtypes = [vp]
        lib.il_check_device_status.restype = ci
        _lib = lib
    return _lib


def available() -> bool:
    """True when libaiwn_il.so loads and exports the full ABI."""
    try:
        load()
        return True
    except (ILError, OSError, AttributeError):
        return False


def version() -> str:
    return load().il_version().decode()


def _check(rc: int, what: str):
    if rc != 0:
        raise ILError(f"{what}: {load().il_status_string(rc).decode()} (status {rc})")


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ILError("aiwn_b200 kernels need CUDA tensors; there is no CPU path")
        if t is not None and not t.is_contiguous():
            raise ILError("aiwn_b200 kernels need contiguous tensors")


class _on_device:
    """Make x's device current for the duration of a C call (cheap no-op when
    it already is)."""

    def __init__(self, dev: torch.device):
        self.idx = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *a):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _expect(name: str, t, shape, dtype=torch.float32):
    """Raise ILError unless tensor `t` (skipped when None) has exactly this
    dtype and shape: the C entry points trust every size they are given, so a
    mismatch caught here is one that never reaches a kernel."""
    if t is None:
        return
    if t.dtype != dtype:
        raise ILError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ILError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")


def _same_device(*ts):
    devs = {t.device for t in ts if t is not None}
    if len(devs) > 1:
        raise ILError(f"tensors on different devices: {sorted(str(d) for d in devs)}")


def _layer_shapes(x, table):
    """(N, IN, OUT, K) of an IndexedLinear call, checking x [N, IN] against
    table [K, IN, OUT]."""
    if x.dim() != 2:
        raise ILError(f"x must be [N, in_d], got shape {tuple(x.shape)}")
    if table.dim() != 3:
        raise ILError(f"table must be [K, in_d, out_d], got shape {tuple(table.shape)}")
    N, IN = x.shape
    K, tin, OUT = table.shape
    if tin != IN:
        raise ILError(f"x has in_d {IN} but the table has {tin}")
    _expect("table", table, (K, IN, OUT))
    return N, IN, OUT, K


def x_dtype_code(x: torch.Tensor) -> int:
    try:
        return _DTYPES[x.dtype]
    except KeyError:
        raise ILError(f"x dtype {x.dtype} is not supported (float32 or bfloat16)") from None


def forward(x, table, bias, out, bw: float, counts=None):
    """out[N, OUT] (fp32) <- IndexedLinear forward of x[N, IN]; with
    ``counts`` (int64 [K] on the device) the bin occupancy of x is added into
    it by the same launch where the kernel allows."""
    _same_device(x, table, bias, out, counts)
    N, IN, OUT, K = _layer_shapes(x, table)
    x_dtype_code(x)
    _expect("bias", bias, (OUT,))
    _expect("out", out, (N, OUT))
    _expect("counts", counts, (K,), torch.int64)
    _need_cuda(x, table, bias, out, counts)
    lib = load()
    with _on_device(x.device):
        if counts is None:
            _check(lib.il_forward(_p(x), x_dtype_code(x), _p(table), _p(bias), _p(out),
                                  N, IN, OUT, K, float(bw), _stream(x.device)), "il_forward")
        else:
            _check(lib.il_forward_counts(_p(x), x_dtype_code(x), _p(table), _p(bias), _p(out),
                                         N, IN, OUT, K, float(bw), _p(counts), _stream(x.device)),
                   "il_forward_counts")
    return out


def workspace_bytes(N, IN, OUT, K, x_dtype: int) -> int:
    return int(load().il_workspace_bytes(N, IN, OUT, K, x_dtype))


def backward(go, x, table, gx, gt, gb, bw: float, workspace=None, accumulate: bool = False):
    """gx / gt / gb (any may be None) <- gradients of the forward; with
    ``accumulate`` gt and gb are added into instead of overwritten."""
    _same_device(go, x, table, gx, gt, gb, workspace)
    N, IN, OUT, K = _layer_shapes(x, table)
    xdt = x_dtype_code(x)
    _expect("go", go, (N, OUT))
    _expect("gx", gx, (N, IN), x.dtype)
    _expect("gt", gt, (K, IN, OUT))
    _expect("gb", gb, (OUT,))
    if workspace is not None and workspace.dtype != torch.uint8:
        raise ILError("workspace must be a uint8 tensor")
    if workspace_bytes(N, IN, OUT, K, xdt) > (0 if workspace is None else workspace.numel()):
        raise ILError("workspace missing or smaller than workspace_bytes()")
    _need_cuda(go, x, table, gx, gt, gb, workspace)
    lib = load()
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    fn, name = (lib.il_backward_accumulate, "il_backward_accumulate") if accumulate else (lib.il_backward,
                                                                                           "il_backward")
    with _on_device(x.device):
        _check(fn(_p(go), _p(x), x_dtype_code(x), _p(table), _p(gx), _p(gt), _p(gb), N, IN, OUT, K, float(bw),
                  _p(workspace), ws_bytes, _stream(x.device)), name)


def cdf_forward(x, gamma, beta, eps: float, table, bias, xn, mean, rstd, out, bw: float):
    """IndexedLinearV2 forward: xn <- GaussianCDFNorm(x), out <- IndexedLinear(xn);
    also the per-token LayerNorm mean and rstd.  fp32 x [N, IN]."""
    _same_device(x, gamma, beta, table, bias, xn, mean, rstd, out)
    if x.dtype != torch.float32:
        raise ILError("il_cdf_forward takes fp32 x")
    N, IN, OUT, K = _layer_shapes(x, table)
    for name, t, shp in (("gamma", gamma, (IN,)), ("beta", beta, (IN,)), ("bias", bias, (OUT,)),
                         ("xn", xn, (N, IN)), ("mean", mean, (N,)), ("rstd", rstd, (N,)), ("out", out, (N, OUT))):
        _expect(name, t, shp)
    _need_cuda(x, gamma, beta, table, bias, xn, mean, rstd, out)
    lib = load()
    with _on_device(x.device):
        _check(lib.il_cdf_forward(_p(x), _p(gamma), _p(beta), float(eps), _p(table), _p(bias), _p(xn), _p(mean),
                                  _p(rstd), _p(out), N, IN, OUT, K, float(bw), _stream(x.device)),
               "il_cdf_forward")
    return out


def cdf_backward(gxn, x, gamma, beta, mean, rstd, dx, dgamma, dbeta):
    """dx / dgamma / dbeta (any may be None) <- backward of the GaussianCDFNorm prologue."""
    _same_device(gxn, x, gamma, beta, mean, rstd, dx, dgamma, dbeta)
    if x.dim() != 2:
        raise ILError(f"x must be [N, in_d], got shape {tuple(x.shape)}")
    N, IN = x.shape
    for name, t, shp in (("gxn", gxn, (N, IN)), ("x", x, (N, IN)), ("gamma", gamma, (IN,)), ("beta", beta, (IN,)),
                         ("mean", mean, (N,)), ("rstd", rstd, (N,)), ("dx", dx, (N, IN)), ("dgamma", dgamma, (IN,)),
                         ("dbeta", dbeta, (IN,))):
        _expect(name, t, shp)
    _need_cuda(gxn, x, gamma, beta, mean, rstd, dx, dgamma, dbeta)
    lib = load()
    with _on_device(x.device):
        _check(lib.il_cdf_backward(_p(gxn), _p(x), _p(gamma), _p(beta), _p(mean), _p(rstd), _p(dx), _p(dgamma),
                                   _p(dbeta), N, IN, _stream(x.device)), "il_cdf_backward")


def layernorm_forward(x, gamma, beta, eps: float, y, mean, rstd):
    """y <- LayerNorm(x; gamma, beta, eps) over the last dim (fp32 x [N, IN],
    IN <= 32); also the per-row mean and rstd [N]."""
    _same_device(x, gamma, beta, y, mean, rstd)
    if x.dim() != 2:
        raise ILError(f"x must be [N, in_d], got shape {tuple(x.shape)}")
    N, IN = x.shape
    for name, t, shp in (("x", x, (N, IN)), ("gamma", gamma, (IN,)), ("beta", beta, (IN,)), ("y", y, (N, IN)),
                         ("mean", mean, (N,)), ("rstd", rstd, (N,))):
        _expect(name, t, shp)
    _need_cuda(x, gamma, beta, y, mean, rstd)
    lib = load()
    with _on_device(x.device):
        _check(lib.il_layernorm_forward(_p(x), _p(gamma), _p(beta), float(eps), _p(y), _p(mean), _p(rstd), N, IN,
                                        _stream(x.device)), "il_layernorm_forward")
    return y


def layernorm_backward(gy, x, gamma, mean, rstd, dx, dgamma, dbeta):
    """dx / dgamma / dbeta (any may be None) <- backward of layernorm_forward."""
    _same_device(gy, x, gamma, mean, rstd, dx, dgamma, dbeta)
    if x.dim() != 2:
        raise ILError(f"x must be [N, in_d], got shape {tuple(x.shape)}")
    N, IN = x.shape
    for name, t, shp in (("gy", gy, (N, IN)), ("x", x, (N, IN)), ("gamma", gamma, (IN,)), ("mean", mean, (N,)),
                         ("rstd", rstd, (N,)), ("dx", dx, (N, IN)), ("dgamma", dgamma, (IN,)), ("dbeta", dbeta, (IN,))):
        _expect(name, t, shp)
    _need_cuda(gy, x, gamma, mean, rstd, dx, dgamma, dbeta)
    lib = load()
    with _on_device(x.device):
        _check(lib.il_layernorm_backward(_p(gy), _p(x), _p(gamma), _p(mean), _p(rstd), _p(dx), _p(dgamma),
                                         _p(dbeta), N, IN, _stream(x.device)), "il_layernorm_backward")


def attention_supported(T: int, D: int) -> bool:
    """Whether il_attention_* take heads of D features over T positions."""
    return D in (2, 4, 8, 16) and 1 <= T <= (512 if D == 16 else 1024)


def _attn_shapes(q, H: int):
    if q.dim() != 3 or H < 1 or q.shape[2] % H != 0:
        raise ILError(f"q must be [B, T, H*D] with H={H} dividing the last dimension, got {tuple(q.shape)}")
    _expect("q", q, tuple(q.shape))
    return q.shape


def _expect_seed(seed, p: float):
    if seed is None:
        if p > 0:
            raise ILError("dropout p > 0 needs a device seed tensor")
        return
    if seed.dtype not in (torch.int64, torch.uint64) or seed.numel() < 1:
        raise ILError("seed must be an int64 device tensor of at least one element")


def attention_forward(q, k, v, o, lse, H: int, scale: float, p: float, seed):
    """o <- causal attention of fp32 q, k, v [B, T, H*D] (dropout p, device
    int64 seed [1]); lse [B, H, T] for the backward."""
    _same_device(q, k, v, o, lse, seed)
    B, T, C = _attn_shapes(q, H)
    for name, t in (("k", k), ("v", v), ("o", o)):
        _expect(name, t, (B, T, C))
    _expect("lse", lse, (B, H, T))
    _expect_seed(seed, p)
    _need_cuda(q, k, v, o, lse, seed)
    lib = load()
    with _on_device(q.device):
        _check(lib.il_attention_forward(_p(q), _p(k), _p(v), _p(o), _p(lse), B, T, H, C // H, float(scale),
                                        float(p), _p(seed), _stream(q.device)), "il_attention_forward")
    return o


def attention_backward(q, k, v, o, do, lse, dq, dk, dv, H: int, scale: float, p: float, seed):
    """dq, dk, dv <- backward of attention_forward given do = dL/do."""
    _same_device(q, k, v, o, do, lse, dq, dk, dv, seed)
    B, T, C = _attn_shapes(q, H)
    for name, t in (("k", k), ("v", v), ("o", o), ("do", do), ("dq", dq), ("dk", dk), ("dv", dv)):
        _expect(name, t, (B, T, C))
    _expect("lse", lse, (B, H, T))
    _expect_seed(seed, p)
    _need_cuda(q, k, v, o, do, lse, dq, dk, dv, seed)
    lib = load()
    with _on_device(q.device):
        _check(lib.il_attention_backward(_p(q), _p(k), _p(v), _p(o), _p(do), _p(lse), _p(dq), _p(dk), _p(dv), B, T,
                                         H, C // H, float(scale), float(p), _p(seed), _stream(q.device)),
               "il_attention_backward")


def attention_dropout_mask(keep, B: int, T: int, H: int, p: float, seed):
    """keep [B, H, T, T] uint8 <- the dropout mask attention_forward uses."""
    _same_device(keep, seed)
    _expect("keep", keep, (B, H, T, T), torch.uint8)
    _expect_seed(seed, 1.0)
    _need_cuda(keep, seed)
    lib = load()
    with _on_device(keep.device):
        _check(lib.il_attention_dropout_mask(_p(keep), B, T, H, float(p), _p(seed), _stream(keep.device)),
               "il_attention_dropout_mask")


def bin_counts(x, K: int, bw: float, counts):
    """counts[K] (int64, device) += occupancy of the bins of x[..., IN]."""
    _same_device(x, counts)
    if counts.dtype != torch.int64 or counts.numel() != K:
        raise ILError("bin_counts needs an int64 counts tensor of K elements")
    x_dtype_code(x)
    _need_cuda(x, counts)
    x2 = x.reshape(-1, x.shape[-1])
    lib = load()
    with _on_device(x.device):
        _check(lib.il_bin_counts(_p(x2), x_dtype_code(x2), x2.shape[0], x2.shape[1], K, float(bw), _p(counts),
                                 _stream(x.device)), "il_bin_counts")
    return counts


def bins(x, K: int, bw: float):
    """(lo int32, hi int32, fr fp32) of every element of x[N, IN]."""
    _need_cuda(x)
    x2 = x.reshape(x.shape[0] if x.dim() > 1 else 1, -1)
    lo = torch.empty(x2.shape, dtype=torch.int32, device=x.device)
    hi = torch.empty_like(lo)
    fr = torch.empty(x2.shape, dtype=torch.float32, device=x.device)
    with _on_device(x.device):
        _check(load().il_bins(_p(x2), x_dtype_code(x), x2.shape[0], x2.shape[1], K, float(bw),
                              _p(lo), _p(hi), _p(fr), _stream(x.device)), "il_bins")
    return lo.reshape(x.shape), hi.reshape(x.shape), fr.reshape(x.shape)


def adam_step(p, g, m, v, lr, beta1, beta2, eps, step: int):
    _same_device(p, g, m, v)
    for t in (p, g, m, v):
        if t.dtype != torch.float32:
            raise ILError("il_adam_step works on fp32 tensors")
        if t.numel() != p.numel():
            raise ILError("il_adam_step: p, g, m and v must have the same number of elements")
    _need_cuda(p, g, m, v)
    with _on_device(p.device):
        _check(load().il_adam_step(_p(p), _p(g), _p(m), _p(v), p.numel(), float(lr), float(beta1),
                                   float(beta2), float(eps), int(step), _stream(p.device)),
               "il_adam_step")


def allreduce_scratch_bytes(n: int, world: int) -> int:
    """Bytes of the per-rank scratch region allreduce_sum needs for n
    elements over `world` ranks."""
    b = int(load().il_allreduce_scratch_bytes(int(n), int(world)))
    if b < 0:
        raise ILError(f"allreduce_scratch_bytes: invalid n={n} or world={world}")
    return b


def allreduce_sum(bufs, scratch, n: int, rank: int, world: int, scale: float = 1.0, timeout_s: float = 10.0,
                  device=None):
    """In-place all-reduce (sum x scale) of n fp32 elements over `world`
    GPUs: bufs / scratch are every rank's buffer and scratch region
    addresses as mapped in this process (peer memory), 256-byte aligned."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    allreduce_caller(bufs, scratch, n, rank, world, timeout_s, dev)(scale)


def allreduce_caller(bufs, scratch, n: int, rank: int, world: int, timeout_s: float, device):
    """A function scale -> None that runs allreduce_sum with these fixed
    buffers on the current stream of `device`, with the address arrays built
    once (the per-call host cost is one C call)."""
    if len(bufs) != world or len(scratch) != world:
        raise ILError("allreduce_sum needs one buffer and one scratch address per rank")
    dev = torch.device(device)
    arr = ctypes.c_uint64 * world
    b, f = arr(*[int(p) for p in bufs]), arr(*[int(p) for p in scratch])
    pb, pf = ctypes.cast(b, ctypes.c_void_p), ctypes.cast(f, ctypes.c_void_p)
    fn = load().il_allreduce_sum
    n, rank, world, timeout_s = int(n), int(rank), int(world), float(timeout_s)

    def call(scale: float = 1.0):
        with _on_device(dev):
            rc = fn(pb, pf, n, rank, world, float(scale), timeout_s, _stream(dev))
        if rc:
            _check(rc, "il_allreduce_sum")

    call.keep = (b, f)  # the arrays live as long as the function
    return call


def kernel_launches() -> int:
    """Kernels launched by libaiwn_il.so in this process so far."""
    return int(load().il_kernel_launches())


def check_device_status(dev=None):
    dev = torch.device("cuda", torch.cuda.current_device()) if dev is None else dev
    with _on_device(dev):
        _check(load().il_check_device_status(_stream(dev)), "device status")
