"""Parity of the CUDA kernels (through the C ABI) with the oracle and with the
golden vectors of the reference.

Tolerances (normwise, see golden_io.normwise_close): forward 1e-5 relative in
fp32 and 2e-2 with bf16 x; fp32 gradients 1e-4; bf16 gx 2e-2.  Bins are
bit-exact.
"""
import math

import numpy as np
import pytest
import torch

from golden_io import bins_names, case_names, load_bins, load_case, normwise_close, same_bits
from il_cases import CASES, EDGE_CASES, make_inputs, to_numpy_grad, x_numpy
from oracle import oracle

import aiwn_b200
from aiwn_b200 import IndexedLinear, _Fn, _lib

pytestmark = pytest.mark.gpu

FWD_RTOL = {"f32": 1e-5, "bf16": 2e-2}
GRAD_RTOL = 1e-4
BF16_GX_RTOL = 2e-2
DEV = "cuda"


def _bf16_from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def run_ours(x, table, bias, go, bw):
    """forward + backward through _Fn (the reference's autograd.Function API)."""
    xg = x.to(DEV).requires_grad_(True)
    tg = table.to(DEV).requires_grad_(True)
    bg = bias.to(DEV).requires_grad_(True)
    out = _Fn.apply(xg, tg, bg, bw)
    out.backward(go.to(DEV))
    torch.cuda.synchronize()
    return out.detach(), xg.grad, tg.grad, bg.grad


def check_against_oracle(c, x, table, bias, go):
    bw = 2.0 / c.K
    out, gx, gt, gb = run_ours(x, table, bias, go, bw)
    assert out.dtype == torch.float32 and gx.dtype == x.dtype
    xn = x_numpy(x)
    ref = oracle.forward(xn, table.numpy(), bias.numpy(), bw, x_dtype=c.dtype)
    normwise_close(out.cpu().numpy(), ref, FWD_RTOL[c.dtype], f"{c.name} out")
    rgx, rgt, rgb = oracle.backward(go.numpy(), xn, table.numpy(), bw, x_dtype=c.dtype)
    normwise_close(to_numpy_grad(gx), rgx, BF16_GX_RTOL if c.dtype == "bf16" else GRAD_RTOL, f"{c.name} gx")
    normwise_close(gt.cpu().numpy(), rgt, GRAD_RTOL, f"{c.name} gt")
    normwise_close(gb.cpu().numpy(), rgb, GRAD_RTOL, f"{c.name} gb")
    lo, hi, fr = _lib.bins(x.to(DEV), c.K, bw)
    rlo, rhi, rfr = oracle.bins(xn, c.K, bw, x_dtype=c.dtype)
    assert np.array_equal(lo.cpu().numpy(), rlo) and np.array_equal(hi.cpu().numpy(), rhi)
    assert same_bits(fr.cpu().numpy(), rfr)


@pytest.mark.parametrize("paths", [("auto", "auto"), ("token", "sorted"), ("cluster", "gather")],
                         ids=["auto", "pinned", "alt"])
@pytest.mark.parametrize("c", CASES + EDGE_CASES, ids=lambda c: c.name)
def test_parity_vs_oracle(c, paths, monkeypatch):
    """auto: the library's own choice (cluster forward for rows of >= 32
    outputs at K <= 64, else one token per lane; bin-sorted backward) wherever there is a
    plan; pinned: the token forward and the sorted backward wherever they have
    a plan; alt: the cluster forward and the gather backward with per-token
    table-gradient reductions."""
    monkeypatch.setenv("AIWN_IL_FORWARD", paths[0])
    monkeypatch.setenv("AIWN_IL_BACKWARD", paths[1])
    x, table, bias, go = make_inputs(c)
    check_against_oracle(c, x, table, bias, go)


TC_CASES = [c for c in CASES + EDGE_CASES
            if c.OUT % 16 == 0 and c.OUT <= 256 and c.K >= 16 and (c.K & (c.K - 1)) == 0 and (c.IN * c.K) % 32 == 0]


@pytest.mark.parametrize("c", TC_CASES, ids=lambda c: c.name)
def test_tensor_core_forward_vs_oracle(c, monkeypatch):
    """The tcgen05 hat-basis forward (3xTF32, accumulator in tensor memory),
    pinned with AIWN_IL_FORWARD=tc, on every listed shape it takes."""
    monkeypatch.setenv("AIWN_IL_FORWARD", "tc")
    x, table, bias, _ = make_inputs(c)
    out = torch.empty(c.N, c.OUT, device=DEV)
    _lib.forward(x.to(DEV), table.to(DEV), bias.to(DEV), out, 2.0 / c.K)
    ref = oracle.forward(x_numpy(x), table.numpy(), bias.numpy(), 2.0 / c.K, x_dtype=c.dtype)
    normwise_close(out.cpu().numpy(), ref, FWD_RTOL[c.dtype], f"{c.name} out (tc)")


def test_tensor_core_forward_nonfinite_and_partial_tile(monkeypatch):
    """Tokens with +-inf or NaN inputs take the plain formula in the
    epilogue; 300 tokens end in a partial 128-token tile."""
    monkeypatch.setenv("AIWN_IL_FORWARD", "tc")
    g = torch.Generator().manual_seed(5)
    N, IN, OUT, K = 300, 8, 32, 16
    x = torch.rand(N, IN, generator=g) * 2.4 - 1.2
    x[3, 1] = float("inf")
    x[4, 0] = float("-inf")
    x[7, 5] = float("nan")
    x[299, 2] = float("inf")
    table = torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)
    bias = torch.randn(OUT, generator=g) * 0.1
    out = torch.empty(N, OUT, device=DEV)
    _lib.forward(x.to(DEV), table.to(DEV), bias.to(DEV), out, 2.0 / K)
    ref = oracle.forward(x.numpy(), table.numpy(), bias.numpy(), 2.0 / K)
    normwise_close(out.cpu().numpy(), ref, FWD_RTOL["f32"], "tc non-finite")


@pytest.mark.parametrize("fwd", ["auto", "token"], ids=["wide_fwd", "stream_fwd"])
def test_c4_parity_at_the_bench_launch_size(fwd, monkeypatch):
    """The large-table configuration at the size one GPU runs in the bench:
    16384 tokens, in_d = out_d = 1024, K = 64, x = clamp(N(0, 0.5), -1, 1).
    Exercises the forward that the library picks there (one warp per token,
    streamed table) and the streamed per-lane forward (AIWN_IL_FORWARD=token
    falls through to it), and the sorted backward's 128-column j-ranges with
    atomically added dx at that launch shape; every output and gradient is
    compared with the oracle."""
    from il_cases import Case
    monkeypatch.setenv("AIWN_IL_FORWARD", fwd)
    c = Case("c4_bench_launch", 16384, 1024, 1024, 64, "clamp_normal", "f32", 0.1, 40)
    x, table, bias, go = make_inputs(c)
    check_against_oracle(c, x, table, bias, go)


def _wide_cases():
    from il_cases import Case
    listed = [c for c in CASES + EDGE_CASES if c.OUT % 64 == 0 and c.K <= 128 and (c.K & (c.K - 1)) == 0]
    return listed + [
        Case("wide_in1020_out128_k64", 333, 1020, 128, 64, "wide", "f32", 0.3, 41),  # entry-block tail
        Case("wide_in9_out384_k128", 1000, 9, 384, 128, "wide", "f32", 0.3, 42),     # one column per stage
        Case("wide_in24_out128_k16_bf16", 2049, 24, 128, 16, "wide", "bf16", 0.3, 43),
        Case("wide_in1_out128_k2", 5, 1, 128, 2, "wide", "f32", 0.3, 44),
        Case("wide_in64_out256_k32_n7000", 7000, 64, 256, 32, "clamp_normal", "f32", 0.3, 45),
        # 64-wide j-ranges: two tokens per warp step
        Case("wide64_in64_out64_k16_n7000", 7000, 64, 64, 16, "uniform", "f32", 0.3, 46),
        Case("wide64_in20_out192_k64", 999, 20, 192, 64, "wide", "f32", 0.3, 47),
        Case("wide64_in7_out64_k128_bf16", 333, 7, 64, 128, "wide", "bf16", 0.3, 48),
    ]


@pytest.mark.parametrize("c", _wide_cases(), ids=lambda c: c.name)
def test_wide_forward_vs_oracle(c, monkeypatch):
    """The warp-per-token forward (out_d a multiple of 64, K <= 128), pinned
    with AIWN_IL_FORWARD=wide: 128- and 64-wide j-ranges, partial token
    tiles, entry blocks past in_d, 1..8 input columns per stage, bf16 x."""
    monkeypatch.setenv("AIWN_IL_FORWARD", "wide")
    x, table, bias, _ = make_inputs(c)
    out = torch.empty(c.N, c.OUT, device=DEV)
    _lib.forward(x.to(DEV), table.to(DEV), bias.to(DEV), out, 2.0 / c.K)
    ref = oracle.forward(x_numpy(x), table.numpy(), bias.numpy(), 2.0 / c.K, x_dtype=c.dtype)
    normwise_close(out.cpu().numpy(), ref, FWD_RTOL[c.dtype], f"{c.name} out (wide)")


@pytest.mark.parametrize("OUT", [256, 64])
def test_wide_forward_matches_streamed_forward_bitwise(OUT, monkeypatch):
    """Same products in the same order: the warp-per-token forward (128- and
    64-wide j-ranges) and the per-lane token forward give identical bits,
    non-finite inputs included."""
    g = torch.Generator().manual_seed(9)
    N, IN, K = 1500, 40, 64
    x = torch.rand(N, IN, generator=g) * 2.4 - 1.2
    x[3, 1] = float("inf")
    x[4, 0] = float("-inf")
    x[7, 5] = float("nan")
    table = (torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)).to(DEV)
    bias = (torch.randn(OUT, generator=g) * 0.1).to(DEV)
    xd = x.to(DEV)
    outs = {}
    for path in ("wide", "token"):
        monkeypatch.setenv("AIWN_IL_FORWARD", path)
        outs[path] = torch.empty(N, OUT, device=DEV)
        _lib.forward(xd, table, bias, outs[path], 2.0 / K)
    a, b = outs["wide"].cpu().numpy(), outs["token"].cpu().numpy()
    assert same_bits(a, b)
    ref = oracle.forward(x.numpy(), table.cpu().numpy(), bias.cpu().numpy(), 2.0 / K)
    normwise_close(a, ref, FWD_RTOL["f32"], "wide non-finite")


@pytest.mark.parametrize("name", case_names())
def test_parity_vs_golden(name):
    d = load_case(name)
    dt = d["x_dtype"]
    x = _bf16_from_bits(d["x"]) if dt == "bf16" else torch.from_numpy(d["x"])
    out, gx, gt, gb = run_ours(x, torch.from_numpy(d["table"]), torch.from_numpy(d["bias"]),
                               torch.from_numpy(d["go"]), d["bw"])
    normwise_close(out.cpu().numpy(), d["out"], FWD_RTOL["f32"], "out")
    normwise_close(to_numpy_grad(gx), d["gx"], BF16_GX_RTOL if dt == "bf16" else GRAD_RTOL, "gx")
    normwise_close(gt.cpu().numpy(), d["gt"], GRAD_RTOL, "gt")
    normwise_close(gb.cpu().numpy(), d["gb"], GRAD_RTOL, "gb")


@pytest.mark.parametrize("name", bins_names())
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_bins_bit_exact_vs_golden(name, dt):
    d = load_bins(name)
    xb = d[f"x_{dt}"]
    x = _bf16_from_bits(xb) if dt == "bf16" else torch.from_numpy(xb)
    lo, hi, fr = _lib.bins(x.to(DEV), d["K"], d["bw"])
    assert np.array_equal(lo.cpu().numpy(), d[f"lo_{dt}"])
    assert same_bits(fr.cpu().numpy(), d[f"fr_{dt}"])


def test_forward_deterministic_and_token_independent():
    """Full C3 size: bitwise-identical reruns, and the output of a token does
    not depend on which other tokens share the launch."""
    c = CASES[2]
    x, table, bias, _ = make_inputs(c)
    x, table, bias = x.to(DEV), table.to(DEV), bias.to(DEV)
    bw = 2.0 / c.K
    o1 = torch.empty(c.N, c.OUT, device=DEV)
    o2 = torch.empty_like(o1)
    _lib.forward(x, table, bias, o1, bw)
    _lib.forward(x, table, bias, o2, bw)
    assert torch.equal(o1, o2)
    cut = 50001
    oa = torch.empty(cut, c.OUT, device=DEV)
    ob = torch.empty(c.N - cut, c.OUT, device=DEV)
    _lib.forward(x[:cut].contiguous(), table, bias, oa, bw)
    _lib.forward(x[cut:].contiguous(), table, bias, ob, bw)
    assert torch.equal(torch.cat([oa, ob]), o1)


def test_dtable_is_additive_over_token_chunks():
    c = CASES[2]
    x, table, bias, go = make_inputs(c)
    x, table, go = x.to(DEV), table.to(DEV), go.to(DEV)
    bw = 2.0 / c.K
    gt = torch.empty_like(table)
    _lib.backward(go, x, table, None, gt, None, bw, _ws(c, x))
    parts = torch.zeros_like(table)
    for a, b in ((0, 40000), (40000, 90001), (90001, c.N)):
        g = torch.empty_like(table)
        xs = x[a:b].contiguous()
        _lib.backward(go[a:b].contiguous(), xs, table, None, g, None, bw, _ws(c, xs))
        parts += g
    normwise_close(parts.cpu().numpy(), gt.cpu().numpy(), GRAD_RTOL, "dtable chunks")


def _ws(c, x):
    n = _lib.workspace_bytes(x.shape[0], c.IN, c.OUT, c.K, _lib.x_dtype_code(x))
    return torch.empty(n, dtype=torch.uint8, device=DEV) if n else None


def test_module_flattens_leading_dims_and_backprops():
    torch.manual_seed(0)
    m = IndexedLinear(20, 80, 512).to(DEV)
    with torch.no_grad():
        m.bias.normal_()
    x = (torch.rand(2, 3, 50, 20, device=DEV) * 2 - 1).requires_grad_(True)
    y = m(x)
    assert y.shape == (2, 3, 50, 80) and y.dtype == torch.float32
    go = torch.randn_like(y)
    y.backward(go)
    xf = x.detach().reshape(-1, 20).cpu().numpy()
    ref = oracle.forward(xf, m.table.detach().cpu().numpy(), m.bias.detach().cpu().numpy(), m.bw)
    normwise_close(y.detach().reshape(-1, 80).cpu().numpy(), ref, 1e-5, "module out")
    rgx, rgt, rgb = oracle.backward(go.reshape(-1, 80).cpu().numpy(), xf, m.table.detach().cpu().numpy(), m.bw)
    normwise_close(x.grad.reshape(-1, 20).cpu().numpy(), rgx, GRAD_RTOL, "module gx")
    normwise_close(m.table.grad.cpu().numpy(), rgt, GRAD_RTOL, "module gt")
    normwise_close(m.bias.grad.cpu().numpy(), rgb, GRAD_RTOL, "module gb")
    assert aiwn_b200.TRITON_OK and aiwn_b200.triton_available()


def test_grad_subsets_follow_needs_input_grad():
    c = CASES[0]
    x, table, bias, go = make_inputs(c)
    xg = x.to(DEV)
    tg = table.to(DEV).requires_grad_(True)
    out = _Fn.apply(xg, tg, bias.to(DEV), 2.0 / c.K)
    out.backward(go.to(DEV))
    _, rgt, _ = oracle.backward(go.numpy(), x.numpy(), table.numpy(), 2.0 / c.K)
    normwise_close(tg.grad.cpu().numpy(), rgt, GRAD_RTOL, "gt only")


def test_adam_step_matches_torch():
    g = torch.Generator().manual_seed(5)
    p0 = torch.randn(513 * 20 * 20 + 3, generator=g)
    grads = [torch.randn(p0.shape, generator=g) for _ in range(3)]
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.Adam([ref], lr=1e-2, foreach=False)
    p = p0.to(DEV)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    for k, gr in enumerate(grads, start=1):
        ref.grad = gr.clone()
        opt.step()
        _lib.adam_step(p, gr.to(DEV), m, v, 1e-2, 0.9, 0.999, 1e-8, k)
    torch.cuda.synchronize()
    normwise_close(p.cpu().numpy(), ref.detach().numpy(), 1e-6, "adam")


def test_device_status_clean():
    _lib.check_device_status()


def test_backward_accumulate_adds_into_grads():
    """il_backward_accumulate: gt / gb grow by the gradients of each call
    (chunks of a batch sum to the whole batch's); dx is written per call."""
    c = CASES[2]
    x, table, bias, go = make_inputs(c)
    bw = 2.0 / c.K
    out, gx, gt, gb = run_ours(x, table, bias, go, bw)
    x, table, go = x.to(DEV), table.to(DEV), go.to(DEV)
    h = x.shape[0] // 3
    gt_acc = torch.full_like(gt, 0.5)
    gb_acc = torch.full_like(gb, -0.25)
    gx_acc = torch.empty_like(gx)
    for a, b in ((0, h), (h, x.shape[0])):
        _lib.backward(go[a:b], x[a:b], table, gx_acc[a:b], gt_acc, gb_acc, bw, accumulate=True)
    torch.cuda.synchronize()
    normwise_close(gt_acc.cpu().numpy() - 0.5, gt.cpu().numpy(), GRAD_RTOL, "accumulated gt")
    normwise_close(gb_acc.cpu().numpy() + 0.25, gb.cpu().numpy(), GRAD_RTOL, "accumulated gb")
    normwise_close(gx_acc.cpu().numpy(), gx.cpu().numpy(), 1e-6, "dx of the chunks")


@pytest.mark.parametrize("chunks,pieces,resident", [(5, None, True), (5, None, False), (None, None, True),
                                                    (6, 2, True), (8, 1, True), (6, 3, False),
                                                    (7, (3, 2, 1, 1), True), (6, (1, 4, 1), False)],
                         ids=["per_chunk_buffers", "slot_ring", "tuned_chunks", "pieces_of_3_chunks",
                              "one_upload", "ring_ignores_pieces", "tapered_pieces", "ring_ignores_tapered"])
@pytest.mark.parametrize("graphs", [True, False])
def test_host_pipeline_matches_whole_batch_call(graphs, chunks, pieces, resident):
    """HostPipeline (chunked, copies overlapped on three streams, replayed
    from a CUDA graph or issued eagerly; device buffers per chunk or a ring
    of two reused slots; uploads per chunk or in pieces of several chunks)
    gives the same out / dx as one call on the whole batch and the same
    summed grads."""
    from aiwn_b200.pipeline import HostPipeline
    c = CASES[2]
    x, table, bias, go = make_inputs(c)
    N = 50003
    x, go = x[:N].contiguous(), go[:N].contiguous()
    m = IndexedLinear(c.IN, c.OUT, c.K).to(DEV)
    with torch.no_grad():
        m.table.copy_(table)
        m.bias.copy_(bias)
    xh, goh = x.pin_memory(), go.pin_memory()
    outh = torch.empty(N, c.OUT).pin_memory()
    gxh = torch.empty(N, c.IN).pin_memory()
    pipe = HostPipeline(m, chunks=chunks, graphs=graphs, max_resident_bytes=(1 << 30) if resident else 1,
                        pieces=pieces)
    for _ in range(2):  # second call reuses the buffers (and the graph); grads accumulate
        pipe.forward_backward(xh, goh, outh, gxh)
    torch.cuda.synchronize()
    out, gx, gt, gb = run_ours(x, table, bias, go, 2.0 / c.K)
    normwise_close(outh.numpy(), out.cpu().numpy(), 1e-6, "pipeline out")
    normwise_close(gxh.numpy(), gx.cpu().numpy(), 1e-6, "pipeline gx")
    normwise_close(m.table.grad.cpu().numpy(), 2 * gt.cpu().numpy(), GRAD_RTOL, "pipeline gt")
    normwise_close(m.bias.grad.cpu().numpy(), 2 * gb.cpu().numpy(), GRAD_RTOL, "pipeline gb")
    if chunks is None:
        assert pipe.chosen_chunks[N] in HostPipeline.TUNE_CHUNKS
        q, c_ = pipe.chosen_pieces[N], pipe.chosen_chunks[N]
        if isinstance(q, tuple):
            assert sum(q) == c_
        else:
            assert c_ % q == 0
