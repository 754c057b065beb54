"""il_allreduce_sum_noalloc -- the all-reduce for callers that cannot
allocate device memory (it keeps its scratch in a static array compiled into
the library) -- against the allocating entry point il_allreduce_sum, through
the C ABI, two calls in a row each.

One process drives every GPU here, as such a caller would: the new entry
point enqueues all ranks of a call itself; the allocating one is called once
per rank, each on its own device, with a torch-allocated scratch region per
device.  With one GPU the comparison runs at world 1 (the static scratch is
set up, summed into and copied back); with two GPUs also at world 2, across
the GPUs.  This file is collected
last, so a failure here stops a `-x` run only after every other test ran.
"""
import ctypes

import pytest
import torch

from aiwn_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL = 1e-6  # the all-reduce tolerance of the multi-GPU tests


def _arr(vals):
    return (ctypes.c_uint64 * len(vals))(*[int(v) for v in vals])


def _streams(world):
    return [torch.cuda.current_stream(torch.device("cuda", p)) for p in range(world)]


def _run_allocating(bufs, n, scale, world):
    """il_allreduce_sum, one call per rank on its device (scratch from torch)."""
    lib = _lib.load()
    sb = _lib.allreduce_scratch_bytes(n, world)
    scratch = [torch.zeros(sb, dtype=torch.uint8, device=f"cuda:{p}") for p in range(world)]
    for p in range(world):
        torch.cuda.synchronize(p)
    b, s = _arr([t.data_ptr() for t in bufs]), _arr([t.data_ptr() for t in scratch])
    for p, st in enumerate(_streams(world)):
        with torch.cuda.device(p):
            rc = lib.il_allreduce_sum(ctypes.cast(b, ctypes.c_void_p), ctypes.cast(s, ctypes.c_void_p), n, p, world,
                                      scale, 10.0, ctypes.c_void_p(st.cuda_stream))
        assert rc == 0, lib.il_status_string(rc)
    for p in range(world):
        torch.cuda.synchronize(p)
        _lib.check_device_status(torch.device("cuda", p))


def _run_noalloc(bufs, n, scale, world):
    lib = _lib.load()
    b = _arr([t.data_ptr() for t in bufs])
    st = _arr([s.cuda_stream for s in _streams(world)])
    rc = lib.il_allreduce_sum_noalloc(ctypes.cast(b, ctypes.c_void_p), n, world, scale,
                                      ctypes.cast(st, ctypes.c_void_p))
    assert rc == 0, lib.il_status_string(rc)
    for p in range(world):
        torch.cuda.synchronize(p)
        _lib.check_device_status(torch.device("cuda", p))


@pytest.mark.parametrize("world", [1, 2])
def test_noalloc_allreduce_matches_allocating_entry_point(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for call, (n, scale) in enumerate([(204820, 1.0), (100003, 0.5)]):  # two calls in a row
        g = torch.Generator().manual_seed(17 + call)
        src = [torch.randn(n, generator=g) for _ in range(world)]
        mine = [src[p].to(f"cuda:{p}") for p in range(world)]
        theirs = [src[p].to(f"cuda:{p}") for p in range(world)]
        _run_noalloc(mine, n, scale, world)
        _run_allocating(theirs, n, scale, world)
        want = sum(src) * scale
        for p in range(world):
            got, ref = mine[p].cpu(), theirs[p].cpu()
            assert torch.allclose(got, ref, rtol=RTOL, atol=RTOL), f"call {call} rank {p}"
            assert torch.allclose(got, want, rtol=RTOL, atol=RTOL), f"call {call} rank {p} vs host sum"


def test_noalloc_allreduce_rejects_sizes_beyond_its_static_scratch():
    lib = _lib.load()
    t = torch.zeros(8, device="cuda:0")
    b = _arr([t.data_ptr()])
    st = _arr([torch.cuda.current_stream(torch.device("cuda", 0)).cuda_stream])
    rc = lib.il_allreduce_sum_noalloc(ctypes.cast(b, ctypes.c_void_p), (1 << 18) + 1, 1, 1.0,
                                      ctypes.cast(st, ctypes.c_void_p))
    assert lib.il_status_string(rc).decode() == "invalid shape"
    rc = lib.il_allreduce_sum_noalloc(ctypes.cast(b, ctypes.c_void_p), 8, 9, 1.0,
                                      ctypes.cast(st, ctypes.c_void_p))
    assert lib.il_status_string(rc).decode() == "invalid shape"
