"""IndexedLinear benchmark on B200: fwd and fwd+bwd tokens/s, % of HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c3]

One step = one forward + backward of IndexedLinear over the configuration's
token batch (B*seq tokens per GPU; weak scaling across GPUs: with N>1 every
rank processes its own batch and the [table | bias] gradient bucket is
all-reduced over NCCL each step, the data-parallel exchange of training).
Rank 0 prints one JSON line.  Inputs rotate over enough sets that the bytes
read per step are not L2-resident (>126 MB per rotation).

--impl reference times the reference's own CPU path (its eager PyTorch ops,
restated in oracle/eager_port.py) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "fwd & fwd+bwd tokens/s at K=128/512, seq=4096; % of HBM roofline"
L2_BYTES = 126 * 2**20

# The benchmark configurations (d, K, B, seq as the reference's high_k sweep
# names them; in_d = out_d = indexed_dims(d, 4d, K)[0]).
CONFIGS = {
    "c3": dict(desc="high-K headline: IndexedLinear(20, 20, K=512) fwd+bwd, d=512 B=32 seq=4096, "
                    "x~U(-1,1) fp32, table~N(0,1/in_d)", d=512, K=512, B=32, seq=4096, IN=20, OUT=20,
               xdist="uniform", dtype="f32"),
    "c2": dict(desc="sweep point: IndexedLinear(20, 20, K=128) fwd+bwd, d=256 B=32 seq=4096, "
                    "x=tanh(N(0,1)) bf16, fp32 table", d=256, K=128, B=32, seq=4096, IN=20, OUT=20,
               xdist="tanh_normal", dtype="bf16"),
    "c1": dict(desc="IndexedLinear(64, 64, K=16) fwd+bwd, d=256 B=8 seq=256, x~U(-1,1) fp32",
               d=256, K=16, B=8, seq=256, IN=64, OUT=64, xdist="uniform", dtype="f32"),
    "c3ref": dict(desc="reference benchmark shape IndexedLinear(20, 80, K=512), B=32 seq=4096 fp32",
                  d=512, K=512, B=32, seq=4096, IN=20, OUT=80, xdist="uniform", dtype="f32"),
    "c4": dict(desc="IndexedLinear(1024, 1024, K=64), 16384 tokens per GPU, x=clamp(N(0,0.5)) fp32",
               d=1024, K=64, B=2, seq=8192, IN=1024, OUT=1024, xdist="clamp_normal", dtype="f32"),
    "c3v2": dict(desc="IndexedLinearV2(20, 20, K=512): GaussianCDFNorm prologue fused into the forward, "
                      "fwd+bwd, d=512 B=32 seq=4096, x~N(0.3, 1.7^2) fp32", d=512, K=512, B=32, seq=4096, IN=20,
                 OUT=20, xdist="normal", dtype="f32", v2=True),
    "c5gpt": dict(desc="config 5: IndexedGPT training step (4 layers, n_embd 256 -> d_idx 16, ff_idx 8, 4 heads, "
                       "K=128, vocab 65, ctx 256, batch 64), fp32, AdamW + clip, CUDA-graph replay",
                  d=256, K=128, B=64, seq=256, IN=16, OUT=16, xdist="uniform", dtype="f32", gpt=True),
    "c5": dict(desc="IndexedGPT projection shape IndexedLinear(16, 16, K=128), batch 64 x ctx 256 "
                    "(16384 tokens), x~U(-1,1) fp32", d=256, K=128, B=64, seq=256, IN=16, OUT=16,
               xdist="uniform", dtype="f32"),
    "c5qkv": dict(desc="IndexedGPT fused q|k|v projection IndexedLinear(16, 48, K=128), batch 64 x ctx 256 "
                       "(16384 tokens), x~U(-1,1) fp32", d=256, K=128, B=64, seq=256, IN=16, OUT=48,
                  xdist="uniform", dtype="f32"),
    "c1big": dict(desc="IndexedLinear(64, 64, K=16) at 131072 tokens (the C1 layer, large batch), x~U(-1,1) fp32",
                  d=256, K=16, B=32, seq=4096, IN=64, OUT=64, xdist="uniform", dtype="f32"),
}


def arm_config(cfg):
    """The `config` object of the JSON line: identical in both arms (the
    workload and its sizes only; how an arm runs it goes in top-level keys)."""
    return {"workload": cfg["desc"], "K": cfg["K"], "in_d": cfg["IN"], "out_d": cfg["OUT"],
            "tokens_per_gpu": cfg["B"] * cfg["seq"], "d": cfg["d"], "B": cfg["B"], "seq": cfg["seq"]}


def cpu_model() -> str:
    """The host CPU's model name (first `model name` line of /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(N, IN, OUT, K, sx):
    """Compulsory HBM bytes: x, out, table, bias for the forward; go, x, table
    re-read and dx, dtable, dbias written for the backward."""
    fwd = N * IN * sx + N * OUT * 4 + K * IN * OUT * 4 + OUT * 4
    bwd = N * OUT * 4 + N * IN * sx + K * IN * OUT * 4 + N * IN * sx + K * IN * OUT * 4 + OUT * 4
    return fwd, bwd


def make_x(N, IN, xdist, dtype, gen, device):
    if xdist == "uniform":
        x = torch.rand(N, IN, generator=gen, device=device) * 2 - 1
    elif xdist == "tanh_normal":
        x = torch.tanh(torch.randn(N, IN, generator=gen, device=device))
    elif xdist == "normal":
        x = torch.randn(N, IN, generator=gen, device=device) * 1.7 + 0.3
    else:
        x = (torch.randn(N, IN, generator=gen, device=device) * 0.5).clamp(-1, 1)
    return x.to(torch.bfloat16) if dtype == "bf16" else x


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed loops run."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for k, name in enumerate(names):
                    if r[5 + k].strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        sm.sort()
        # samples under load: the top half of the SM clock distribution is the
        # timed region (the sampler also sees the idle edges around it)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


# ---------------------------------------------------------------------------
# reference arm: the reference's eager CPU path on the host cores
# ---------------------------------------------------------------------------

def cpu_step_fn(cfg, g):
    """The reference's CPU fwd+bwd step for this config (its eager ops,
    restated in oracle/eager_port.py): IndexedLinear, or IndexedLinearV2."""
    from oracle.eager_port import eager_step, eager_step_v2
    IN, OUT, K = cfg["IN"], cfg["OUT"], cfg["K"]
    bw = 2.0 / K
    table = torch.randn(K, IN, OUT, generator=g) / math.sqrt(IN)
    bias = torch.zeros(OUT)
    if cfg.get("v2"):
        gamma = 1.0 + 0.1 * torch.randn(IN, generator=g)
        beta = 0.1 * torch.randn(IN, generator=g)
        return lambda x, go: eager_step_v2(x, gamma, beta, 1e-5, table, bias, go, bw)
    return lambda x, go: eager_step(x, table, bias, go, bw)


def run_reference(args, cfg, world, rank):
    if rank != 0:
        return None
    if cfg.get("gpt"):
        b = gpt_cpu_baseline(cfg, seconds=max(5.0, min(60.0, 2.0 * (args.steps + args.warmup))))
        return {"metric": METRIC, "value": b["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": arm_config(cfg), "cpu_baseline": b, "e2e": {"value": b["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                           "d2h_bytes_per_step": 0}}
    torch.set_num_threads(os.cpu_count() or 1)
    N, IN, OUT, K = cfg["B"] * cfg["seq"], cfg["IN"], cfg["OUT"], cfg["K"]
    g = torch.Generator().manual_seed(0)
    step = cpu_step_fn(cfg, g)
    # size the per-step token sample so the whole run stays within ~2 minutes
    probe = 1024
    x = make_x(probe, IN, cfg["xdist"], cfg["dtype"], g, "cpu")
    go = torch.randn(probe, OUT, generator=g)
    step(x, go)
    t = time.perf_counter()
    step(x, go)
    per_tok = (time.perf_counter() - t) / probe
    budget = 100.0 / max(1, args.steps + args.warmup)
    n_s = int(min(N, max(256, budget / max(per_tok, 1e-12))))
    n_s = max(256, (n_s // 256) * 256)
    x = make_x(n_s, IN, cfg["xdist"], cfg["dtype"], g, "cpu")
    go = torch.randn(n_s, OUT, generator=g)
    for _ in range(args.warmup):
        step(x, go)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(x, go)
    dt = (time.perf_counter() - t0) / args.steps
    v = n_s / dt
    cores = torch.get_num_threads()
    sample = (f"{n_s} of the {N} tokens of the workload per step (fwd+bwd of the reference's "
              f"eager ops, restated in oracle/eager_port.py), {cores} threads")
    module = None if cfg.get("v2") else reference_module_cpu(cfg, x, go, min(args.steps, 3))
    return {
        "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if cfg["dtype"] == "bf16" else "f32", "data": "synthetic",
        "impl": "reference",
        "config": arm_config(cfg), "x_dtype": cfg["dtype"],
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "cpu_model": cpu_model(), "kind": "port",
                         "sample": sample, "reference_module": module},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_module_cpu(cfg, x, go, steps):
    """The same CPU step through the reference's own module, installed
    unchanged in baseline/_ref (its IndexedLinear.forward takes _eager on CPU
    tensors, aiwn/layers/indexed_linear.py:173-190, and autograd does the
    backward): a check that the timed port runs at the reference's speed."""
    if steps < 1 or not os.path.isdir(os.path.join(REF_PKG, "aiwn")):
        return None
    try:
        sys.path.insert(0, REF_PKG)
        try:
            import aiwn.layers.indexed_linear as ref_il
        finally:
            sys.path.remove(REF_PKG)
        m = ref_il.IndexedLinear(cfg["IN"], cfg["OUT"], cfg["K"])
        xr = x.float().clone().requires_grad_(True)

        def step():
            m.zero_grad(set_to_none=True)
            xr.grad = None
            m(xr).backward(go)

        step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        dt = (time.perf_counter() - t0) / steps
        return {"value": x.shape[0] / dt, "unit": "tokens/s", "steps": steps,
                "code": "baseline/_ref aiwn.layers.indexed_linear.IndexedLinear on CPU tensors, fwd+bwd"}
    except Exception as e:  # reported, never fatal
        return {"unavailable": repr(e)[:200]}


REF_CUDA_SO = os.path.join(ROOT, "baseline", "_ref", "indexed_linear_cuda.so")


def reference_gpu(cfg, x, table, bias, go, reps=3):
    """The reference's own CUDA extension (aiwn/layers/indexed_linear_cuda.cu,
    built for sm_100a by baseline/build_ref_cuda.py) timed on the same
    device-resident inputs: its forward, and its backward (dx and dtable; it
    has no dbias).  Reported beside the result, not as it.  Its kernels take
    fp32 x in [-1, 1] only (the low bin is not clamped), so other inputs are
    not run."""
    if cfg["dtype"] != "f32" or cfg["xdist"] != "uniform":
        return {"unavailable": "the reference's CUDA extension takes fp32 x in [-1, 1] only"}
    if not os.path.exists(REF_CUDA_SO):
        return {"unavailable": "not built here (python baseline/build_ref_cuda.py)"}
    import importlib.util
    spec = importlib.util.spec_from_file_location("indexed_linear_cuda", REF_CUDA_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    bw = 2.0 / cfg["K"]

    def timed(fn):
        fn()  # warm-up
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()  # the extension launches on the legacy default stream, torch's current one here
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    ms_f = timed(lambda: mod.forward(x, table, bias, bw))
    ms_b = timed(lambda: mod.backward(go, x, table, bw))
    n = x.shape[0]
    return {"source": "aiwn/layers/indexed_linear_cuda.cu, built for sm_100a", "fwd_ms": ms_f, "bwd_ms": ms_b,
            "fwd_tokens_per_s": n / (ms_f * 1e-3), "fwd_bwd_tokens_per_s": n / ((ms_f + ms_b) * 1e-3),
            "reps": reps, "inputs": "the bench's first x/go set, device-resident"}


REF_PKG = os.path.join(ROOT, "baseline", "_ref")


def reference_triton(cfg, x, table, bias, go, reps=3):
    """The reference's own GPU path: ``aiwn.layers.indexed_linear._Fn``
    (Triton forward IL:23-39 + bias add, Triton dx IL:41-60, one-hot einsum
    dtable IL:131-149, go.sum(0) dbias), installed unchanged into
    baseline/_ref by baseline/install_ref.py and timed on the same
    device-resident inputs as this library.  Reported beside the result, not
    as it.  fp32 x only: its backward allocates fp32 one-hot tensors of x's
    dtype and cannot run bf16."""
    if cfg["dtype"] != "f32":
        return {"unavailable": "the reference's Triton backward takes fp32 x only"}
    if not os.path.isdir(os.path.join(REF_PKG, "aiwn")):
        return {"unavailable": "reference package not installed (python baseline/install_ref.py)"}
    try:
        sys.path.insert(0, REF_PKG)
        try:
            import aiwn.layers.indexed_linear as ref_il
        finally:
            sys.path.remove(REF_PKG)
        if not ref_il.TRITON_OK:
            return {"unavailable": "triton did not import in the reference module"}
        bw = 2.0 / cfg["K"]
        xr = x.detach().clone().requires_grad_(True)
        tr = table.detach().clone().requires_grad_(True)
        br = bias.detach().clone().requires_grad_(True)

        def fwd():
            with torch.no_grad():
                return ref_il._Fn.apply(xr, tr, br, bw)

        def fwd_bwd():
            out = ref_il._Fn.apply(xr, tr, br, bw)
            return torch.autograd.grad(out, (xr, tr, br), go)

        def timed(fn):
            fn()  # warm-up (and Triton's JIT compile)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / reps

        ms_f = timed(fwd)
        ms_fb = timed(fwd_bwd)
        n = x.shape[0]
        return {"source": "aiwn.layers.indexed_linear._Fn (Triton), the reference package in baseline/_ref",
                "fwd_ms": ms_f, "fwd_bwd_ms": ms_fb, "fwd_tokens_per_s": n / (ms_f * 1e-3),
                "fwd_bwd_tokens_per_s": n / (ms_fb * 1e-3), "reps": reps,
                "inputs": "the bench's first x/go set, device-resident"}
    except Exception as e:  # the comparator must not take the bench line down with it
        torch.cuda.synchronize()
        return {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    finally:
        torch.cuda.empty_cache()


def cpu_baseline(cfg, seconds=12.0):
    """The reference's CPU path on a bounded sample of the workload."""
    torch.set_num_threads(os.cpu_count() or 1)
    IN, OUT = cfg["IN"], cfg["OUT"]
    g = torch.Generator().manual_seed(0)
    step = cpu_step_fn(cfg, g)
    n_s = 4096 if IN * OUT <= 4096 else 32
    x = make_x(n_s, IN, cfg["xdist"], cfg["dtype"], g, "cpu")
    go = torch.randn(n_s, OUT, generator=g)
    step(x, go)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        step(x, go)
        done += 1
    dt = (time.perf_counter() - t0) / done
    cores = torch.get_num_threads()
    return {"value": n_s / dt, "unit": "tokens/s", "cores": cores, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{done} fwd+bwd steps of {n_s} tokens (reference eager ops{', V2 chain' if cfg.get('v2') else ''}, "
                      f"oracle/eager_port.py) in {seconds:.0f} s on {cores} threads"}


def host_copy_probe(dev, world, local, mib=32, reps=4, trials=3):
    """Pinned host <-> device copy rates of this rank (GB/s) for `mib`-MiB
    copies, host to device alone, device to host alone and both at once, with
    every rank copying at the same time (a barrier before each pattern), the
    best of `trials`: the host-side limit of the end-to-end leg."""
    n = mib * 2**20 // 4
    h_src = torch.empty(n, dtype=torch.float32).pin_memory()
    h_dst = torch.empty(n, dtype=torch.float32).pin_memory()
    d_a = torch.empty(n, device=dev)
    d_b = torch.empty(n, device=dev)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    def timed(up, down):
        sync()
        t0 = time.perf_counter()
        for _ in range(reps):
            if up:
                with torch.cuda.stream(s_up):
                    d_a.copy_(h_src, non_blocking=True)
            if down:
                with torch.cuda.stream(s_down):
                    h_dst.copy_(d_b, non_blocking=True)
        torch.cuda.synchronize(dev)
        return (time.perf_counter() - t0) / reps

    timed(True, True)
    nbytes = n * 4
    t_up = min(timed(True, False) for _ in range(trials))
    t_down = min(timed(False, True) for _ in range(trials))
    t_both = min(timed(True, True) for _ in range(trials))
    return {"copy_mib": mib, "h2d_gbs": nbytes / t_up / 1e9, "d2h_gbs": nbytes / t_down / 1e9,
            "both_gbs": 2 * nbytes / t_both / 1e9, "ranks_copying": world}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def v2_bytes(N, IN, OUT, K):
    """Compulsory HBM bytes of IndexedLinearV2: the forward reads x, writes xn,
    mean, rstd and out; the backward reads go, xn, x, mean, rstd and writes
    gxn (read back), dx, dtable, dbias, dgamma, dbeta."""
    tab = K * IN * OUT * 4
    fwd = N * IN * 4 * 2 + N * 8 + N * OUT * 4 + tab + OUT * 4 + IN * 8
    bwd = N * OUT * 4 + N * IN * 4 + tab + N * IN * 4 * 2 + tab + OUT * 4 + N * IN * 4 * 2 + N * 8 + IN * 8
    return fwd, bwd


def run_ours_v2(args, cfg, world, rank, local):
    """IndexedLinearV2: fused prologue + forward, sorted backward on xn, prologue backward."""
    from aiwn_b200 import IndexedLinearV2, _lib
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N, IN, OUT, K = cfg["B"] * cfg["seq"], cfg["IN"], cfg["OUT"], cfg["K"]
    bw = 2.0 / K
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    per_set = N * IN * 4 * 3 + N * OUT * 4 * 2
    n_sets = max(2, min(16, math.ceil(2 * L2_BYTES / per_set)))
    xs = [make_x(N, IN, cfg["xdist"], "f32", gen, dev) for _ in range(n_sets)]
    gos = [torch.randn(N, OUT, generator=gen, device=dev) for _ in range(n_sets)]
    outs = [torch.empty(N, OUT, device=dev) for _ in range(n_sets)]
    xns = [torch.empty(N, IN, device=dev) for _ in range(n_sets)]
    dxs = [torch.empty(N, IN, device=dev) for _ in range(n_sets)]
    gxn = torch.empty(N, IN, device=dev)
    mean, rstd = torch.empty(N, device=dev), torch.empty(N, device=dev)
    table = torch.randn(K, IN, OUT, generator=gen, device=dev) / math.sqrt(IN)
    gamma = 1.0 + 0.1 * torch.randn(IN, generator=gen, device=dev)
    beta = 0.1 * torch.randn(IN, generator=gen, device=dev)
    if world > 1:
        import torch.distributed as dist
        for t in (table, gamma, beta):
            dist.broadcast(t, 0)
    bias = torch.zeros(OUT, device=dev)
    nb = K * IN * OUT + OUT + 2 * IN
    bucket = torch.empty(nb, device=dev)  # [dtable | dbias | dgamma | dbeta]
    gt = bucket[: K * IN * OUT].view(K, IN, OUT)
    gb = bucket[K * IN * OUT: K * IN * OUT + OUT]
    dg = bucket[K * IN * OUT + OUT: K * IN * OUT + OUT + IN]
    db = bucket[K * IN * OUT + OUT + IN:]

    def fwd(i):
        _lib.cdf_forward(xs[i], gamma, beta, 1e-5, table, bias, xns[i], mean, rstd, outs[i], bw)

    def bwd(i):
        _lib.backward(gos[i], xns[i], table, gxn, gt, gb, bw)
        _lib.cdf_backward(gxn, xs[i], gamma, beta, mean, rstd, dxs[i], dg, db)

    def step(k):
        i = k % n_sets
        fwd(i)
        bwd(i)
        if world > 1:
            torch.distributed.all_reduce(bucket)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def time_calls(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync_all()
        e0.record()
        for k in range(reps):
            fn(k)
        e1.record()
        sync_all()
        return max_over_ranks(e0.elapsed_time(e1) / reps)

    clocks = ClockSampler(local) if rank == 0 else None
    for k in range(max(3, args.warmup)):
        step(k)
    sync_all()
    if clocks:
        clocks.start()
    launches0 = _lib.kernel_launches()
    ms_step = time_calls(step, args.steps)
    launches = _lib.kernel_launches() - launches0
    reps = max(args.steps, 20)
    ms_fwd = time_calls(lambda k: fwd(k % n_sets), reps)
    ms_bwd = time_calls(lambda k: (fwd(k % n_sets), bwd(k % n_sets)), reps) - ms_fwd

    # end to end through the module: pinned host x / go in, out / dx out
    m = IndexedLinearV2(IN, OUT, K).to(dev)
    with torch.no_grad():
        m.linear.table.copy_(table)
        m.cdf.ln.weight.copy_(gamma)
        m.cdf.ln.bias.copy_(beta)
    xh = [x.cpu().pin_memory() for x in xs[:2]]
    goh = [g.cpu().pin_memory() for g in gos[:2]]
    outh = [torch.empty(N, OUT).pin_memory() for _ in range(2)]
    dxh = [torch.empty(N, IN).pin_memory() for _ in range(2)]

    def e2e_step(k):
        i = k % 2
        m.zero_grad(set_to_none=False)
        xd = xh[i].to(dev, non_blocking=True).requires_grad_(True)
        y = m(xd)
        y.backward(goh[i].to(dev, non_blocking=True))
        if world > 1:
            for p_ in m.parameters():
                torch.distributed.all_reduce(p_.grad)
        outh[i].copy_(y.detach(), non_blocking=True)
        dxh[i].copy_(xd.grad, non_blocking=True)

    for k in range(3):
        e2e_step(k)
    ms_e2e = time_calls(e2e_step, max(10, min(args.steps, 100)))
    clk = clocks.stop() if clocks else None
    if rank != 0:
        return None
    hbm, peak_kind = peaks()
    b_fwd, b_bwd = v2_bytes(N, IN, OUT, K)
    dom = ("forward", ms_fwd, b_fwd) if ms_fwd >= ms_bwd else ("backward", ms_bwd, b_bwd)
    achieved = dom[2] / (dom[1] * 1e-3) / 1e9
    res = {
        "metric": METRIC, "value": world * N / (ms_step * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": arm_config(cfg), "x_dtype": "f32",
        "parallelism": f"token-parallel dp{world}" + (" + NCCL all-reduce of the gradients" if world > 1 else ""),
        "l2": f"inputs rotate over {n_sets} sets ({n_sets * per_set / 2**20:.0f} MiB > L2)",
        "fwd_tokens_per_s": world * N / (ms_fwd * 1e-3),
        "fwd_bwd_tokens_per_s": world * N / (ms_step * 1e-3),
        "ms": {"fwd": ms_fwd, "bwd": ms_bwd, "fwd_bwd": ms_step},
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": dom[2]},
        "e2e": {"value": world * N / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": N * (IN + OUT) * 4,
                "d2h_bytes_per_step": N * (IN + OUT) * 4,
                "api": "aiwn_b200.IndexedLinearV2 forward+backward through autograd; pinned host x/go copied in, "
                       "out/dx copied back each step"},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg)
    return res


GPT_CFG = dict(vocab_size=65, block_size=256, n_layer=4, n_head=4, n_embd=256, K=128, dropout=0.1)


def _zipf_tokens(n, vocab, gen, device):
    """Seeded synthetic token stream: Zipf(1.1) over the vocabulary."""
    w = 1.0 / torch.arange(1, vocab + 1, dtype=torch.float64) ** 1.1
    return torch.multinomial(w / w.sum(), n, replacement=True, generator=gen).to(device)


def _gpt_batches(n_batches, B, T, vocab, gen, device):
    data = _zipf_tokens(n_batches * B * (T + 1), vocab, gen, "cpu").view(n_batches, B, T + 1)
    return data[:, :, :T].contiguous().to(device), data[:, :, 1:].contiguous().to(device)


def gpt_cpu_baseline(cfg, seconds=12.0):
    """The reference's CPU training step (its eager ops) on a bounded batch."""
    from oracle.eager_port import eager_indexed_gpt
    from aiwn_b200.gpt import IndexedGPT
    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    m = eager_indexed_gpt(IndexedGPT(**GPT_CFG))
    opt = torch.optim.AdamW(m.parameters(), lr=3e-4 * math.sqrt(GPT_CFG["K"] / 2), weight_decay=1e-2)
    g = torch.Generator().manual_seed(0)
    Bs = 4
    x, y = _gpt_batches(1, Bs, GPT_CFG["block_size"], GPT_CFG["vocab_size"], g, "cpu")

    def step():
        opt.zero_grad()
        _, loss = m(x[0], y[0])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0)
        opt.step()

    step()
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        step()
        done += 1
    dt = (time.perf_counter() - t0) / done
    n = Bs * GPT_CFG["block_size"]
    cores = torch.get_num_threads()
    return {"value": n / dt, "unit": "tokens/s", "cores": cores, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{done} training steps of batch {Bs} x ctx {GPT_CFG['block_size']} (the reference's eager "
                      f"ops: IndexedLinear._eager restated in oracle/eager_port.py) in {seconds:.0f} s on {cores} threads"}


def run_ours_gpt(args, cfg, world, rank, local):
    """Config 5: IndexedGPT training steps, graph-replayed and eager."""
    from aiwn_b200 import _lib
    from aiwn_b200.gpt import GraphedTrainStep, IndexedGPT
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, T = cfg["B"], GPT_CFG["block_size"]
    torch.manual_seed(1234)
    lr = 3e-4 * math.sqrt(GPT_CFG["K"] / 2)
    gen = torch.Generator().manual_seed(99 + rank)
    nb = 8
    xs, ys = _gpt_batches(nb, B, T, GPT_CFG["vocab_size"], gen, dev)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def time_calls(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync_all()
        e0.record()
        for k in range(reps):
            fn(k)
        e1.record()
        sync_all()
        return max_over_ranks(e0.elapsed_time(e1) / reps)

    model = IndexedGPT(**GPT_CFG).to(dev)
    if world > 1:
        for p_ in model.parameters():
            torch.distributed.broadcast(p_.data, 0)
    opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=1e-2, capturable=True)
    if world > 1:
        # data-parallel: the gradient all-reduce goes inside the captured step
        def _allreduce_hook(p_):
            torch.distributed.all_reduce(p_.grad)
            p_.grad.div_(world)
        for p_ in model.parameters():
            p_.register_post_accumulate_grad_hook(_allreduce_hook)
    graphed = GraphedTrainStep(model, opt, B, T)

    def step(k):
        graphed(xs[k % nb], ys[k % nb])

    clocks = ClockSampler(local) if rank == 0 else None
    for k in range(max(3, args.warmup)):
        step(k)
    sync_all()
    if clocks:
        clocks.start()
    launches0 = _lib.kernel_launches()
    ms_step = time_calls(step, args.steps)
    launches = _lib.kernel_launches() - launches0  # host counter: launches happened at capture

    # the same step without graph replay (eager), for comparison
    model_e = IndexedGPT(**GPT_CFG).to(dev)
    opt_e = torch.optim.AdamW(model_e.parameters(), lr=lr, weight_decay=1e-2)

    def eager_step(k):
        opt_e.zero_grad()
        _, loss = model_e(xs[k % nb], ys[k % nb])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model_e.parameters(), 1.0)
        opt_e.step()

    for k in range(3):
        eager_step(k)
    eager_launch0 = _lib.kernel_launches()
    ms_eager = time_calls(eager_step, max(10, min(args.steps, 50)))
    eager_launches = (_lib.kernel_launches() - eager_launch0) / max(10, min(args.steps, 50))

    # end to end: host token batch in (pinned), loss value out
    xh = xs.cpu().pin_memory()
    yh = ys.cpu().pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step(k):
        loss = graphed(xh[k % nb].to(dev, non_blocking=True), yh[k % nb].to(dev, non_blocking=True))
        loss_h.copy_(loss, non_blocking=True)

    ms_e2e = time_calls(e2e_step, max(10, min(args.steps, 100)))
    clk = clocks.stop() if clocks else None
    if rank != 0:
        return None
    n_tok = B * T
    res = {
        "metric": METRIC, "value": world * n_tok / (ms_step * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Zipf(1.1) token stream)",
        "config": arm_config(cfg), "x_dtype": "f32",
        "parallelism": f"data-parallel dp{world}" + (" (gradient all-reduce in the graph)" if world > 1 else ""),
        "l2": "model and activations fit L2; steps rotate over 8 token batches",
        "train_step_tokens_per_s": world * n_tok / (ms_step * 1e-3),
        "eager_step_tokens_per_s": world * n_tok / (ms_eager * 1e-3),
        "ms": {"train_step_graph": ms_step, "train_step_eager": ms_eager},
        "roofline": None,
        "e2e": {"value": world * n_tok / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": 2 * n_tok * 8,
                "d2h_bytes_per_step": 4,
                "api": "aiwn_b200.gpt.GraphedTrainStep: host int64 token batches copied in, loss copied out"},
        "gpu_launches": int(eager_launches * args.steps),
        "gpu_launches_note": "library kernels per eager step x steps (graph replays launch the same kernels "
                             "without host calls)",
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = gpt_cpu_baseline(cfg)
    return res


def run_ours_column(args, cfg, world, rank, local):
    """out_d column-sharded layout (tables too large to replicate): every rank
    holds table[:, :, cols_r] and runs the whole global batch (B*seq tokens
    per GPU, times the number of GPUs) on its columns.  Step: forward on the
    local columns, NCCL all-gather of y, backward on the local columns
    (local table gradient), NCCL all-reduce of the partial dx."""
    from aiwn_b200 import _lib
    from aiwn_b200.distributed import column_shard
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N1, IN, OUT, K = cfg["B"] * cfg["seq"], cfg["IN"], cfg["OUT"], cfg["K"]
    N = N1 * world
    cols = column_shard(OUT, world, rank)
    c = cols.stop - cols.start
    if OUT % world:
        raise SystemExit("--layout column needs out_d divisible by the GPU count")
    bw = 2.0 / K
    gen = torch.Generator(device=dev).manual_seed(1234)  # every rank draws the same global batch
    x = make_x(N, IN, cfg["xdist"], cfg["dtype"], gen, dev)
    table = (torch.randn(K, IN, OUT, generator=gen, device=dev) / math.sqrt(IN))[:, :, cols].contiguous()
    bias = torch.zeros(c, device=dev)
    go = torch.randn(N, c, generator=gen, device=dev)
    y = torch.empty(N, c, device=dev)
    y_all = torch.empty(world * N * c, device=dev)  # rank-major column blocks
    dx = torch.empty_like(x)
    gt = torch.empty_like(table)
    gb = torch.empty(c, device=dev)

    def fwd():
        _lib.forward(x, table, bias, y, bw)
        if world > 1:
            torch.distributed.all_gather_into_tensor(y_all, y)

    def bwd():
        _lib.backward(go, x, table, dx, gt, gb, bw)
        if world > 1:
            torch.distributed.all_reduce(dx)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def timed(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync_all()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        sync_all()
        v = e0.elapsed_time(e1) / reps
        if world > 1:
            t = torch.tensor([v], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            v = float(t.item())
        return v

    for _ in range(max(3, args.warmup)):
        fwd()
        bwd()
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    launches0 = _lib.kernel_launches()
    ms_step = timed(lambda: (fwd(), bwd()), args.steps)
    launches = _lib.kernel_launches() - launches0
    ms_fwd_local = timed(lambda: _lib.forward(x, table, bias, y, bw), args.steps)
    ms_bwd_local = timed(lambda: _lib.backward(go, x, table, dx, gt, gb, bw), args.steps)
    clk = clocks.stop() if clocks else None
    if rank != 0:
        return None
    return {
        "metric": METRIC, "value": N / (ms_step * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if cfg["dtype"] == "bf16" else "f32",
        "data": "synthetic", "config": arm_config(cfg), "x_dtype": cfg["dtype"],
        "layout": f"out_d column-sharded over {world} GPUs: {c} columns and all {N} tokens per GPU",
        "parallelism": f"column shard cs{world}" + (" + NCCL all-gather of y, all-reduce of dx" if world > 1 else ""),
        "ms": {"fwd_bwd": ms_step, "fwd_local": ms_fwd_local, "bwd_local": ms_bwd_local,
               "collectives": ms_step - ms_fwd_local - ms_bwd_local},
        "fwd_bwd_tokens_per_s": N / (ms_step * 1e-3),
        "e2e": None, "e2e_note": "the column layout is measured on device-resident inputs only",
        "gpu_launches": launches, "clocks": clk,
    }


def run_ours(args, cfg, world, rank, local):
    if args.layout == "column":
        return run_ours_column(args, cfg, world, rank, local)
    if cfg.get("gpt"):
        return run_ours_gpt(args, cfg, world, rank, local)
    if cfg.get("v2"):
        return run_ours_v2(args, cfg, world, rank, local)
    from aiwn_b200 import IndexedLinear, _lib
    from aiwn_b200.distributed import TokenParallelIndexedLinear
    from aiwn_b200.pipeline import HostPipeline, bind_host_to_gpu
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # host threads and pinned buffers of the e2e leg next to this GPU (the CPU
    # baseline legs below restore all CPUs)
    cpus_all = os.sched_getaffinity(0)
    numa = bind_host_to_gpu(dev)
    N, IN, OUT, K = cfg["B"] * cfg["seq"], cfg["IN"], cfg["OUT"], cfg["K"]
    bw = 2.0 / K
    sx = 2 if cfg["dtype"] == "bf16" else 4
    xdt = _lib.x_dtype_code(torch.empty(0, dtype=torch.bfloat16 if sx == 2 else torch.float32))
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    per_set = N * IN * sx * 2 + N * OUT * 4 * 2  # x, dx, go, out
    n_sets = max(2, min(16, math.ceil(2 * L2_BYTES / per_set)))
    xs = [make_x(N, IN, cfg["xdist"], cfg["dtype"], gen, dev) for _ in range(n_sets)]
    gos = [torch.randn(N, OUT, generator=gen, device=dev) for _ in range(n_sets)]
    outs = [torch.empty(N, OUT, device=dev) for _ in range(n_sets)]
    gxs = [torch.empty_like(x) for x in xs]
    table = torch.randn(K, IN, OUT, generator=gen, device=dev) / math.sqrt(IN)
    if world > 1:
        import torch.distributed as dist
        dist.broadcast(table, 0)
    bias = torch.zeros(OUT, device=dev)
    # [gt | gb], all-reduced as one buffer: in symmetric memory, summed by the
    # library's peer-memory kernel (--exchange peer), or by NCCL
    peer = None
    if world > 1 and args.exchange == "peer":
        from aiwn_b200.comm import PeerBucket
        peer = PeerBucket(K * IN * OUT + OUT, dev)
        bucket = peer.tensor
    else:
        bucket = torch.empty(K * IN * OUT + OUT, device=dev)
    gt = bucket[: K * IN * OUT].view(K, IN, OUT)
    gb = bucket[K * IN * OUT:]
    ws_n = _lib.workspace_bytes(N, IN, OUT, K, xdt)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)

    def exchange():
        if peer is not None:
            peer.all_reduce(1.0)
        else:
            torch.distributed.all_reduce(bucket)

    def step(k):
        i = k % n_sets
        _lib.forward(xs[i], table, bias, outs[i], bw)
        _lib.backward(gos[i], xs[i], table, gxs[i], gt, gb, bw, ws if ws_n else None)
        if world > 1:
            exchange()

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local) if rank == 0 else None

    # The timed calls replay CUDA graphs, one per input set, captured from the
    # same library calls: a small layer's kernels run for less time than one
    # Python call takes to check and enqueue them, so eager timing would
    # measure the host.  The NCCL exchange stays eager (no NCCL in graphs).
    use_graphs = peer is not None or world == 1

    def graphed(fn):
        if not use_graphs:
            return fn, None
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn(0)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graphs, l0 = [], _lib.kernel_launches()
        for k in range(n_sets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn(k)
            graphs.append(g)
        per_call = (_lib.kernel_launches() - l0) / n_sets
        return (lambda k: graphs[k % n_sets].replay()), per_call

    for k in range(max(3, args.warmup)):
        step(k)
    sync_all()
    launches0 = _lib.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all()
    ev0.record()
    for k in range(args.steps):
        step(k)
    ev1.record()
    sync_all()
    eager_launches = _lib.kernel_launches() - launches0
    ms_step_eager = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)

    step_g, step_launches = graphed(step)
    for k in range(max(3, args.warmup)):
        step_g(k)
    sync_all()
    if clocks:
        clocks.start()
    sync_all()
    ev0.record()
    for k in range(args.steps):
        step_g(k)
    ev1.record()
    sync_all()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    launches = int(round(step_launches * args.steps)) if step_launches is not None else eager_launches

    # per-call device time of the forward and of the backward (same stream)
    def time_calls(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync_all()
        e0.record()
        for k in range(reps):
            fn(k)
        e1.record()
        sync_all()
        return max_over_ranks(e0.elapsed_time(e1) / reps)

    reps = max(args.steps, 20)
    fwd_g, _ = graphed(lambda k: _lib.forward(xs[k % n_sets], table, bias, outs[k % n_sets], bw))
    bwd_g, _ = graphed(lambda k: _lib.backward(gos[k % n_sets], xs[k % n_sets], table, gxs[k % n_sets],
                                               gt, gb, bw, ws if ws_n else None))
    ms_fwd = time_calls(fwd_g, reps)
    ms_bwd = time_calls(bwd_g, reps)

    # training step with the fused Adam update of table and bias
    m_t, v_t = torch.zeros_like(bucket), torch.zeros_like(bucket)
    params = torch.cat([table.reshape(-1), bias])

    def train_step(k):
        step(k)
        _lib.adam_step(params, bucket, m_t, v_t, 1e-3, 0.9, 0.999, 1e-8, k + 1)

    ms_train = time_calls(train_step, reps)
    del step_g, fwd_g, bwd_g

    # the same step without the gradient all-reduce (multi-GPU runs): the
    # difference is the exchange step's cost
    ms_noar = ms_nccl = None
    if world > 1:
        def step_local(k):
            i = k % n_sets
            _lib.forward(xs[i], table, bias, outs[i], bw)
            _lib.backward(gos[i], xs[i], table, gxs[i], gt, gb, bw, ws if ws_n else None)
        local_g, _ = graphed(step_local)
        ms_noar = time_calls(local_g, reps)
        del local_g
        if peer is not None:
            # the same step with NCCL's all-reduce of a plain bucket, for comparison
            nb = torch.empty_like(bucket)
            gtn, gbn = nb[: K * IN * OUT].view(K, IN, OUT), nb[K * IN * OUT:]

            def step_nccl(k):
                i = k % n_sets
                _lib.forward(xs[i], table, bias, outs[i], bw)
                _lib.backward(gos[i], xs[i], table, gxs[i], gtn, gbn, bw, ws if ws_n else None)
                torch.distributed.all_reduce(nb)
            for k in range(3):
                step_nccl(k)
            ms_nccl = time_calls(step_nccl, reps)

    # end to end through the public module API, host buffers, copies inside
    m = TokenParallelIndexedLinear(IN, OUT, K, layer=IndexedLinear(IN, OUT, K),
                                   exchange="peer" if (world > 1 and args.exchange == "peer") else "nccl").to(dev)
    with torch.no_grad():
        m.table.copy_(table)
    xh = [x.cpu().pin_memory() for x in xs[:2]]
    goh = [g.cpu().pin_memory() for g in gos[:2]]
    outh = [torch.empty(N, OUT).pin_memory() for _ in range(2)]
    gxh = [torch.empty(N, IN, dtype=xs[0].dtype).pin_memory() for _ in range(2)]
    # chunk count tuned by the pipeline on its first call (the untimed warm-up)
    pipe = HostPipeline(m)

    def e2e_step(k):
        i = k % 2
        m.zero_grad()
        pipe.forward_backward(xh[i], goh[i], outh[i], gxh[i])
        if world > 1:
            m.sync_grads()

    for k in range(3):
        e2e_step(k)
    e2e_reps = max(10, min(args.steps, 200))
    ms_e2e = time_calls(e2e_step, e2e_reps)
    clk = clocks.stop() if clocks else None
    host_bw = host_copy_probe(dev, world, local)

    if rank != 0:
        return None
    hbm, peak_kind = peaks()
    b_fwd, b_bwd = algorithmic_bytes(N, IN, OUT, K, sx)
    dom = ("forward", ms_fwd, b_fwd) if ms_fwd >= ms_bwd else ("backward", ms_bwd, b_bwd)
    achieved = dom[2] / (dom[1] * 1e-3) / 1e9
    traffic = None
    onchip = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        tj = json.load(open(tp))
        traffic = tj.get(f"{args.config}:{dom[0]}")
        wf = tj.get(f"{args.config}:{dom[0]}:lsu_wavefronts_per_sm")
        if wf:
            # the pipe that binds the kernel: L1 data-pipe wavefronts per SM (ncu)
            # at one per SM clock, against the launch's CUDA-event time
            mhz = (clk or {}).get("sm_mhz") or 1965.0
            floor_us = wf / mhz
            onchip = {"bound": "l1_data_pipe", "wavefronts_per_sm": wf, "sm_mhz": mhz, "floor_us": floor_us,
                      "achieved_us": dom[1] * 1e3, "frac": floor_us / (dom[1] * 1e3),
                      "source": "profiles/traffic.json (ncu l1tex__data_pipe_lsu_wavefronts, one launch)"}
    res = {
        "metric": METRIC,
        "value": world * N / (ms_step * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if sx == 2 else "f32", "data": "synthetic",
        "config": arm_config(cfg), "x_dtype": cfg["dtype"],
        "parallelism": f"token-parallel dp{world}" + (
            (" + peer-memory all-reduce of [dtable|dbias] (il_allreduce_sum, NVLink)" if peer is not None
             else " + NCCL all-reduce of [dtable|dbias]") if world > 1 else ""),
        "l2": f"inputs rotate over {n_sets} sets of x/go/out/dx ({n_sets * per_set / 2**20:.0f} MiB > L2)",
        "fwd_tokens_per_s": world * N / (ms_fwd * 1e-3),
        "fwd_bwd_tokens_per_s": world * N / (ms_step * 1e-3),
        "train_step_tokens_per_s": world * N / (ms_train * 1e-3),
        "ms": {"fwd": ms_fwd, "bwd": ms_bwd, "fwd_bwd": ms_step, "train_step_adam": ms_train,
               "fwd_bwd_eager": ms_step_eager},
        "timing": ("CUDA-graph replays of the library calls, one graph per input set; fwd_bwd_eager: "
                   "the same calls from Python" if use_graphs else "eager library calls"),
        **({"fwd_bwd_without_allreduce": {"tokens_per_s": world * N / (ms_noar * 1e-3), "ms": ms_noar}}
           if ms_noar is not None else {}),
        **({"fwd_bwd_nccl_allreduce": {"tokens_per_s": world * N / (ms_nccl * 1e-3), "ms": ms_nccl,
                                        "timing": "eager (compare with ms.fwd_bwd_eager)"}}
           if ms_nccl is not None else {}),
        "hbm_roofline_frac": {
            "fwd": b_fwd / (ms_fwd * 1e-3) / 1e9 / hbm,
            "fwd_bwd": (b_fwd + b_bwd) / (ms_step * 1e-3) / 1e9 / hbm,
        },
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": dom[2], "onchip_ceiling": onchip},
        "e2e": {"value": world * N / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": xh[0].numel() * xh[0].element_size() + goh[0].numel() * 4,
                "d2h_bytes_per_step": N * OUT * 4 + gxh[0].numel() * gxh[0].element_size(),
                "api": "aiwn_b200.pipeline.HostPipeline over TokenParallelIndexedLinear: forward+backward "
                       f"of pinned host x/go into pinned host out/dx, {pipe.chosen_chunks.get(N)} chunks, "
                       f"{pipe.chosen_pieces.get(N)} upload pieces "
                       "(tuned on the first call) with copies overlapped, replayed as one CUDA graph "
                       "(+gradient all-reduce when N>1)"},
        "gpu_launches": launches,
        "clocks": clk,
    }
    res["e2e"]["host_binding"] = numa
    res["e2e"]["host_copy_rates_rank0"] = host_bw
    moved = res["e2e"]["h2d_bytes_per_step"] + res["e2e"]["d2h_bytes_per_step"]
    # the step's copies alone at the rate measured with every rank copying both ways
    res["e2e"]["copy_floor_ms"] = moved / (host_bw["both_gbs"] * 1e9) * 1e3
    res["e2e"]["copy_floor_frac"] = res["e2e"]["copy_floor_ms"] / ms_e2e
    os.sched_setaffinity(0, cpus_all)
    if world == 1 and not args.no_reference_gpu:
        res["reference_gpu"] = reference_gpu(cfg, xs[0], table, bias, gos[0])
        res["reference_triton"] = reference_triton(cfg, xs[0], table, bias, gos[0])
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="gradient all-reduce at N>1: the library's peer-memory kernel or NCCL")
    ap.add_argument("--layout", choices=["token", "column"], default="token",
                    help="token: replicated table, tokens sharded (default); column: out_d column-sharded")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own CUDA extension (when built)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            res = run_reference(args, cfg, world, rank)
        else:
            res = run_ours(args, cfg, world, rank, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
