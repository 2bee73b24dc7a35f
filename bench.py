#!/usr/bin/env python
"""Benchmark of the fused softmax-weighted embedding readout, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference|reference-gpu]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload (the headline): bf16, N=16384 tokens, K=2560, V=152064, D=64,
bias ~ N(0, 0.02), Bernoulli(0.9) 0/1 per-token weight, z_loss_weight=1e-4, MSE loss,
fwd+bwd through the public API (``swvr_b200.softmax_readout_mse``).  Inputs are seeded
synthetic tensors with the config's distributions (no dataset is involved); W ~ N(0, 1/K)
is read as variance 1/K (std K^-1/2).  W, E and b are drawn whole from one seed and each rank
keeps its vocabulary shard (V/N rows, ``swvr_b200.vocab_parallel``), so every N runs the same
problem (strong scaling) and the ``checksums`` of the JSON line (loss, gradient norms summed
over ranks) agree across N.  W alone (778 MB bf16) is larger than the 126 MB L2, so every
step streams from HBM; no extra L2 flush is needed.

One JSON line on rank 0.  ``value`` is the whole job's algorithmic TFLOP/s,
F_algo = 6 N V (K + D) per step (the backward score recompute is not counted).  At N=1 the
line also carries ``reference_gpu``: the reference library's own GPU path (cuBLAS + its
Triton kernels, unmodified, from the offline install under baseline/_ref) timed in the same
process on the same inputs, with its checksums.

``--impl reference`` is the reference arm: the reference library's own CPU path
(``swvr.softmax_readout_mse`` on CPU tensors, swvr/chunked.py:82-151) on the host cores, one
bounded vocabulary slice of the workload per step; without the install it times the numpy
restatement of that path (oracle/swvr_oracle.py) instead and says so (``kind: "port"``).
``--impl reference-gpu`` prints the reference GPU path's own line.
"""
import argparse
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # N, K, V, D; bias; weight (Bernoulli p); z_loss_weight; lead: h's leading dims;
    # raw: the (O, LSE) op with a torch MSE on top; target "erows": E[randint] + N(0, 0.01)
    "c1": dict(N=16384, K=1024, V=152064, D=16, bias=False, weight=None, z=0.0, lead=(8, 2048)),
    "c2": dict(N=16384, K=2560, V=152064, D=64, bias=True, weight=0.9, z=1e-4),
    "c3": dict(N=8192, K=4096, V=128256, D=128, bias=False, weight=None, z=0.0, raw=True, target="erows"),
    # the headline shape with the widest embedding the tensor-core kernels take
    "d256": dict(N=16384, K=2560, V=152064, D=256, bias=True, weight=0.9, z=1e-4),
    # large batch under activation checkpointing (the readout's forward re-runs in the backward),
    # meant for 2/4/8 GPUs; F_exec counts the re-run, F_algo does not
    "c4": dict(N=131072, K=4096, V=152064, D=64, bias=True, weight=None, z=0.0, lead=(32, 4096), checkpoint=True),
    # profiling size for ncu --set full captures: the c2 kernels on a cut (W 168 MB > L2)
    "prof": dict(N=4096, K=2560, V=32768, D=64, bias=True, weight=0.9, z=1e-4),
    # fp32 operands (exact path: CUDA-core SIMT kernels here, cuBLAS fp32 without TF32 in the
    # reference) at a mid size, to compare the two fp32 paths on one box
    "fp32": dict(N=4096, K=1024, V=32768, D=64, bias=True, weight=0.9, z=1e-4, dtype="fp32"),
}


def param_dtype(c):
    return torch.float32 if c.get("dtype") == "fp32" else torch.bfloat16


def metric_name(args, c):
    """BASELINE.json's metric for the headline config; the same metric at another config's shape."""
    if args.config == "c2":
        return "fwd+bwd TFLOP/s (algorithmic 6NV(K+D)) at N=16k,K=2560,V=152k,D=64"
    return f"fwd+bwd TFLOP/s (algorithmic 6NV(K+D)) at N={c['N']},K={c['K']},V={c['V']},D={c['D']} ({args.config})"


def workload(args, c):
    if c.get("raw"):
        what = "softmax_readout (O, LSE) + torch MSE on O against E[randint] + N(0, 0.01), fwd+bwd"
    else:
        what = "softmax_readout_mse fwd+bwd"
    if c.get("checkpoint"):
        what += " under activation checkpointing"
    return f"{args.config}: {what}"


def config_dict(args, c, world):
    return {"workload": workload(args, c), "N": c["N"], "K": c["K"], "V": c["V"], "D": c["D"],
            "h_shape": [*(c.get("lead") or (c["N"],)), c["K"]], "bias": c["bias"], "weight": c["weight"],
            "z_loss_weight": c["z"], "chunk_size": args.chunk or 8192,
            "parallelism": f"vocab-sharded x{world}" if world > 1 else "single GPU",
            "l2": f"inputs larger than L2 (W {c['V'] * c['K'] * 2 / 1e6:.0f} MB); no flush"}


def f_exec(c):
    """Executed FLOPs per step: F_algo plus the backward's score recompute (and the checkpoint re-run)."""
    N, V, K, D = c["N"], c["V"], c["K"], c["D"]
    return 8.0 * N * V * K + 6.0 * N * V * D + (2.0 * N * V * (K + D) if c.get("checkpoint") else 0.0)


def f_algo(c, V=None):
    V = c["V"] if V is None else V
    return 6.0 * c["N"] * V * (c["K"] + c["D"])


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 1590.0, 1400.0, "fallback"


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each tensor-core
# kernel at the named config on one GPU with the default chunk, from a one-pass capture of one
# launch of this build:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum \
#       --clock-control none -k regex:<kernel> -s 1 -c 1 \
#       python bench.py --steps 2 --warmup 3 --no-cpu-baseline --no-reference-gpu
# Other configs, chunk sizes or GPU counts report null.
CAPTURED_TRAFFIC_GB = {("c2", "gemm_kernel"): 2.956, ("c2", "bwd_scores_kernel"): 0.987,
                       ("c2", "fwd_kernel"): 3.259}


def load_reference():
    """The reference library (pengzhangzhi/swvr, unmodified) from its offline install under
    baseline/_ref, imported under the module name ``swvr_reference`` so that it can never be
    mistaken for this repository's ``swvr`` import alias.  None when it is not installed."""
    mod = sys.modules.get("swvr_reference")
    if mod is not None:
        return mod
    pkg = os.path.join(ROOT, "baseline", "_ref", "swvr")
    init = os.path.join(pkg, "__init__.py")
    if not os.path.exists(init):
        return None
    spec = importlib.util.spec_from_file_location("swvr_reference", init, submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["swvr_reference"] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception:
        del sys.modules["swvr_reference"]
        raise
    return mod


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms; ``summary`` keeps the samples
    taken between ``mark_start`` and ``mark_end`` (the timed region).  ``__enter__`` waits for the
    first sample so that even a short timed region is covered."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        # nvidia-smi numbers GPUs by PCI order, which need not match CUDA's: select by UUID
        try:
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.gpu = str(device.index)
        self.proc = None
        self.t0 = self.t1 = None
        log_dir = os.environ.get("SWVR_BENCH_LOG_DIR") or tempfile.gettempdir()
        self.out = os.path.join(log_dir, f"clocks_bench_{os.getpid()}_{id(self)}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.out), exist_ok=True)
            self.f = open(self.out, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", self.gpu, "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            deadline = time.time() + 10.0
            while time.time() < deadline and self.proc.poll() is None and os.path.getsize(self.out) == 0:
                time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)  # one more sample after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()
        return False

    @staticmethod
    def _when(stamp):
        import datetime
        try:
            return datetime.datetime.strptime(stamp, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.out) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 10 and parts[2].isdigit():
                    rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = []
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if (w := self._when(r[0])) is not None and self.t0 - 0.1 <= w <= self.t1 + 0.1]
        window = inside or rows
        sm = [int(r[2]) for r in window]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in window for n, v in zip(names, r[6:10]) if v.lower() == "active"})
        power = [float(r[4]) for r in window if r[4].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(window[0][3]), "samples": len(window),
                "in_timed_region": bool(inside),
                "power_w_max": max(power) if power else None, "reasons": reasons}


def make_inputs(c, device, rank, world):
    """Seeded synthetic inputs.  W, E and b are drawn whole from one seed on every rank and each
    rank keeps its vocabulary shard, so all N run the same problem; h, target and weight are
    replicated.  h (and target, weight) carry the config's leading dims."""
    from swvr_b200.vocab_parallel import shard_range
    N, K, V, D = c["N"], c["K"], c["V"], c["D"]
    lead = tuple(c.get("lead") or (N,))
    v0, v1 = shard_range(V, world, rank)
    dt = param_dtype(c)
    g = torch.Generator(device=device).manual_seed(1234)
    W_full = (K ** -0.5 * torch.randn(V, K, generator=g, device=device)).to(dt)
    E_full = (0.02 * torch.randn(V, D, generator=g, device=device)).to(dt)
    b_full = (0.02 * torch.randn(V, generator=g, device=device)).to(dt) if c["bias"] else None
    gs = torch.Generator(device=device).manual_seed(99)
    h = torch.randn(N, K, generator=gs, device=device).to(dt).view(*lead, K)
    if c.get("target") == "erows":
        ids = torch.randint(0, V, (N,), generator=gs, device=device)
        t = E_full[ids].float() + 0.01 * torch.randn(N, D, generator=gs, device=device)
    else:
        t = 0.02 * torch.randn(N, D, generator=gs, device=device)
    t = t.view(*lead, D)
    w = (torch.rand(N, generator=gs, device=device) < c["weight"]).float().view(lead) if c["weight"] else None
    W = W_full[v0:v1].clone().requires_grad_(True)
    E = E_full[v0:v1].clone().requires_grad_(True)
    b = b_full[v0:v1].clone().requires_grad_(True) if b_full is not None else None
    del W_full, E_full, b_full
    return h.requires_grad_(True), W, E, b, t, w, v1 - v0


def make_step(c, readout_api, W, E, b, chunk):
    """One fwd+bwd of the workload through ``readout_api`` (a module with ``softmax_readout`` and
    ``softmax_readout_mse``); returns a function (h, target, weight) -> loss."""
    params = [x for x in (W, E, b) if x is not None]

    def loss_of(x, tt, ww):
        if c.get("raw"):
            O, _lse = readout_api.softmax_readout(x, W, E, b, chunk_size=chunk)
            return torch.nn.functional.mse_loss(O, tt.to(O.dtype))
        return readout_api.softmax_readout_mse(x, W, E, tt, b, weight=ww, z_loss_weight=c["z"], chunk_size=chunk)

    def step(hh, tt, ww):
        for p in params:
            p.grad = None
        hh.grad = None
        if c.get("checkpoint"):
            loss = torch.utils.checkpoint.checkpoint(loss_of, hh, tt, ww, use_reentrant=False)
        else:
            loss = loss_of(hh, tt, ww)
        loss.backward()
        return loss

    return step


class _VocabParallelAPI:
    """The vocabulary-sharded entry points under the single-GPU names (for make_step)."""

    def __init__(self, group=None):
        from swvr_b200 import vocab_parallel as vp
        self.vp, self.group = vp, group

    def softmax_readout(self, h, W, E, b, chunk_size=None):
        return self.vp.softmax_readout_vocab_parallel(h, W, E, b, chunk_size=chunk_size, group=self.group)

    def softmax_readout_mse(self, h, W, E, t, b, weight=None, z_loss_weight=0.0, chunk_size=None):
        return self.vp.softmax_readout_mse_vocab_parallel(h, W, E, t, b, weight=weight, z_loss_weight=z_loss_weight,
                                                          chunk_size=chunk_size, group=self.group)


def checksums(loss, h, W, E, b, world):
    """Loss and gradient norms of one step, the shard norms summed over ranks (one tiny
    all-reduce, outside every timed region).  h's gradient is replicated."""
    sq = lambda x: (x.grad.float().norm() ** 2).double() if x is not None and x.grad is not None \
        else torch.zeros((), dtype=torch.float64, device=h.device)
    local = torch.stack([sq(W), sq(E), sq(b)])
    if world > 1:
        dist.all_reduce(local)
    dW2, dE2, db2 = local.tolist()
    out = {"loss": float(loss), "dh_norm": float(h.grad.float().norm()) if h.grad is not None else None,
           "dW_norm": math.sqrt(dW2), "dE_norm": math.sqrt(dE2)}
    if b is not None:
        out["db_norm"] = math.sqrt(db2)
    return {k: (float(f"{v:.7g}") if isinstance(v, float) else v) for k, v in out.items()}


def checksum_agreement(a, b):
    """Largest relative difference between two checksum dicts over their common keys."""
    keys = [k for k in a if k in b and a[k] is not None and b[k] is not None]
    return max((abs(a[k] - b[k]) / max(abs(b[k]), 1e-30) for k in keys), default=None)


def run_ours(args, c, rank, world, device):
    import swvr_b200 as swvr
    from swvr_b200 import _native
    from swvr_b200 import vocab_parallel as vp

    h, W, E, b, t, w, Vr = make_inputs(c, device, rank, world)
    api = swvr if world == 1 else _VocabParallelAPI()
    step = make_step(c, api, W, E, b, args.chunk)
    params = [x for x in (h, W, E, b) if x is not None]

    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        step(h, t, w)
    torch.cuda.synchronize(device)
    _native.check_device_error()
    for p in params:  # peak memory above the inputs, including the gradient buffers (as bench/bench.py:35-38)
        p.grad = None
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    base = torch.cuda.memory_allocated(device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # ---------------------------------------------------------------- device-resident timing
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    loss = None
    with ClockSampler(device) as clocks:
        barrier()
        clocks.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            loss = step(h, t, w)
        ev1.record(stream)
        barrier()
        clocks.mark_end()
    ms = ev0.elapsed_time(ev1) / args.steps
    peak_gib = (torch.cuda.max_memory_allocated(device) - base) / 2 ** 30
    _native.check_device_error()
    sums = checksums(loss.detach(), h, W, E, b, world)

    # per-kernel breakdown: the same steps again under the library's launch accounting, which
    # brackets every launch with CUDA events on its stream (kept out of the timed loop above:
    # an event between two launches would also stop a kernel from starting while its
    # predecessor drains)
    barrier()
    with _native.profile() as prof:
        for _ in range(args.steps):
            step(h, t, w)
        barrier()
    _native.check_device_error()

    # ---------------------------------------------------------------- end to end (host buffers)
    h_host = h.detach().cpu().pin_memory()
    t_host = t.cpu().pin_memory()
    w_host = w.cpu().pin_memory() if w is not None else None
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    h_dev = torch.empty_like(h).requires_grad_(False)
    t_dev = torch.empty_like(t)
    w_dev = torch.empty_like(w) if w is not None else None
    h2d = h_host.numel() * h_host.element_size() + t_host.numel() * 4 + (w_host.numel() * 4 if w is not None else 0)
    if world > 1:  # each rank copies a 1/world row slab; NVLink all-gathers the rest
        h2d = -(-h2d // world)

    def e2e_step():
        hd = vp.replicate_from_host(h_host, device)
        td = vp.replicate_from_host(t_host, device)
        wd = vp.replicate_from_host(w_host, device) if w_host is not None else None
        loss = step(hd.detach().requires_grad_(True), td, wd)
        loss_host.copy_(loss.detach(), non_blocking=True)

    # One GPU: the inputs are double-buffered and step i + 1's are copied on a side stream while
    # step i computes (as a training loop prefetches its next batch); every copy, the first
    # included, runs inside the timed region.
    copy_stream = torch.cuda.Stream(device)
    bufs = [(h_dev, t_dev, w_dev), (torch.empty_like(h_dev), torch.empty_like(t_dev),
                                     torch.empty_like(w_dev) if w_dev is not None else None)]
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]

    def issue_copy(i):
        hb, tb, wb = bufs[i % 2]
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[i % 2])  # the step that last read this buffer is done
            hb.copy_(h_host, non_blocking=True)
            tb.copy_(t_host, non_blocking=True)
            if wb is not None:
                wb.copy_(w_host, non_blocking=True)
            copied[i % 2].record(copy_stream)

    def e2e_run(n):
        if world > 1:
            for _ in range(n):
                e2e_step()
            return
        copy_stream.wait_stream(stream)
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            stream.wait_event(copied[i % 2])
            hb, tb, wb = bufs[i % 2]
            loss = step(hb.detach().requires_grad_(True), tb, wb)
            loss_host.copy_(loss.detach(), non_blocking=True)
            consumed[i % 2].record(stream)

    e2e_run(2)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as e2e_clocks:
        barrier()
        e2e_clocks.mark_start()
        e0.record(stream)
        e2e_run(args.steps)
        e1.record(stream)
        barrier()
        e2e_clocks.mark_end()
    ms_e2e = e0.elapsed_time(e1) / args.steps

    # max over ranks
    t_local = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    ms, ms_e2e = t_local.tolist()
    return dict(ms=ms, ms_e2e=ms_e2e, prof=prof.result, clocks=clocks.summary(), e2e_clocks=e2e_clocks.summary(),
                peak_gib=peak_gib, h2d=h2d,
                loss=float(loss_host), Vr=Vr, checksums=sums)


def kernel_flops(name, c, Vr, launches_per_step, chunk):
    """Algorithmic FLOPs one launch of a kernel performs (per rank)."""
    N, K, D = c["N"], c["K"], c["D"]
    if name == "fwd_kernel":
        return 2.0 * N * Vr * (K + D) * (2.0 if c.get("checkpoint") else 1.0) / launches_per_step
    if name == "gemm_kernel":       # dh and dW of one chunk: 4 N C K per chunk, summed over the shard
        return 4.0 * N * Vr * K / launches_per_step
    if name == "bwd_scores_kernel":  # dP and dE (the S recompute is not algorithmic)
        return 4.0 * N * Vr * D / launches_per_step
    return None


# ------------------------------------------------------------------ the reference's GPU path

def run_reference_gpu(args, c, device):
    """The reference library's own GPU path (its custom ops over cuBLAS and Triton), unmodified,
    from the offline install in baseline/_ref, on the same inputs and step as ours, one GPU.
    Returns a dict (ms, TFLOP/s, peak memory, clocks, checksums) or {"unavailable": why}."""
    try:
        ref = load_reference()
    except Exception as e:  # noqa: BLE001 - report, do not fail the bench
        return {"unavailable": f"importing the reference failed: {type(e).__name__}: {e}"}
    if ref is None:
        return {"unavailable": "no offline install of the reference under baseline/_ref"}
    h, W, E, b, t, w, _ = make_inputs(c, device, 0, 1)
    step = make_step(c, ref, W, E, b, args.chunk)
    for _ in range(max(args.warmup, 2)):
        step(h, t, w)
    torch.cuda.synchronize(device)
    for x in (h, W, E, b):
        if x is not None:
            x.grad = None
    torch.cuda.reset_peak_memory_stats(device)
    mem0 = torch.cuda.memory_allocated(device)
    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    loss = None
    with ClockSampler(device) as clocks:
        torch.cuda.synchronize(device)
        clocks.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            loss = step(h, t, w)
        ev1.record(stream)
        torch.cuda.synchronize(device)
        clocks.mark_end()
    ms = ev0.elapsed_time(ev1) / args.steps
    out = {"ms_per_step": round(ms, 3), "value": round(f_algo(c) / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "peak_mem_gib": round((torch.cuda.max_memory_allocated(device) - mem0) / 2 ** 30, 3),
           "clocks": clocks.summary(), "checksums": checksums(loss.detach(), h, W, E, b, 1),
           "reference_version": getattr(ref, "__version__", None),
           "what": "swvr (unmodified, baseline/_ref): its public API on the same inputs, cuBLAS + Triton"}
    del h, W, E, b, t, w, loss, step
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ the reference's CPU path

def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuSample:
    """One bounded sample of the workload on the host cores: the full token batch against a
    slice of ``rows`` vocabulary rows, fwd + bwd + loss.  Runs the reference library's own CPU
    path (``kind`` "reference") when its offline install is present, else the numpy
    restatement of that path (``kind`` "port")."""

    def __init__(self, c, rows, threads):
        self.c, self.rows, self.threads = c, rows, threads
        try:
            self.ref = load_reference()
        except Exception:  # noqa: BLE001
            self.ref = None
        self.kind = "reference" if self.ref is not None else "port"
        N, K, D = c["N"], c["K"], c["D"]
        lead = tuple(c.get("lead") or (N,))
        g = torch.Generator().manual_seed(0)
        dt = param_dtype(c)
        self.h = torch.randn(N, K, generator=g).to(dt).view(*lead, K)
        self.W = (K ** -0.5 * torch.randn(rows, K, generator=g)).to(dt)
        self.E = (0.02 * torch.randn(rows, D, generator=g)).to(dt)
        self.b = (0.02 * torch.randn(rows, generator=g)).to(dt) if c["bias"] else None
        if c.get("target") == "erows":
            ids = torch.randint(0, rows, (N,), generator=g)
            self.t = (self.E[ids].float() + 0.01 * torch.randn(N, D, generator=g)).view(*lead, D)
        else:
            self.t = (0.02 * torch.randn(N, D, generator=g)).view(*lead, D)
        self.w = (torch.rand(N, generator=g) < c["weight"]).float().view(lead) if c["weight"] else None

    def describe(self):
        c = self.c
        src = ("the reference library's own CPU path (swvr.softmax_readout_mse on CPU tensors, "
               "swvr/chunked.py:82-151, from baseline/_ref)" if self.kind == "reference"
               else "the numpy restatement of swvr's chunked path (oracle/swvr_oracle.py; the reference "
                    "install was not found)")
        return (f"vocabulary slice of {self.rows} of {c['V']} rows against all N={c['N']} tokens "
                f"(K={c['K']}, D={c['D']}), {'fp32' if c.get('dtype') == 'fp32' else 'bf16'} inputs, chunk 8192, "
                f"fwd+bwd+loss: {src}; "
                f"{self.threads} threads")

    def run(self):
        """Seconds for one fwd+bwd of the sample."""
        if self.kind == "port":
            return self._run_port()
        torch.set_num_threads(self.threads)
        ref, c = self.ref, self.c
        h = self.h.detach().requires_grad_(True)
        W = self.W.detach().requires_grad_(True)
        E = self.E.detach().requires_grad_(True)
        b = self.b.detach().requires_grad_(True) if self.b is not None else None
        t0 = time.perf_counter()
        if c.get("raw"):
            O, _ = ref.softmax_readout(h, W, E, b)
            loss = torch.nn.functional.mse_loss(O, self.t)
        else:
            loss = ref.softmax_readout_mse(h, W, E, self.t, b, weight=self.w, z_loss_weight=c["z"])
        loss.backward()
        return time.perf_counter() - t0

    def _run_port(self):
        from oracle import swvr_oracle as orc
        c = self.c
        f = lambda x: None if x is None else x.float().numpy().reshape(-1, x.shape[-1]) if x.dim() > 1 \
            else x.float().numpy().reshape(-1)
        h, W, E, b, t = f(self.h), f(self.W), f(self.E), f(self.b), f(self.t)
        w = None if self.w is None else self.w.numpy().reshape(-1)
        t0 = time.perf_counter()
        cdt = "fp32" if c.get("dtype") == "fp32" else "bf16"
        O, lse = orc.chunked_forward(h, W, E, b, 1.0, 8192, cdt)
        z = 0.0 if c.get("raw") else c["z"]
        orc.mse_forward(O, lse, t, w, "mean", z)
        gO, glse, _, _ = orc.mse_backward(O, lse, t, w, "mean", z)
        orc.chunked_backward(gO, glse, h, W, E, b, O, lse, 1.0, 8192, cdt)
        return time.perf_counter() - t0


def sized_cpu_sample(c, target_s, threads):
    """A CpuSample whose one fwd+bwd takes about target_s seconds (a 256-row probe sizes it)."""
    probe = CpuSample(c, 256, threads)
    probe.run()  # first call pays one-off costs
    dt = probe.run()
    rows = int(min(c["V"], max(256, 256 * target_s / max(dt, 1e-3))) // 256 * 256) or 256
    return probe if rows == 256 else CpuSample(c, rows, threads)


def run_reference_arm(args, c, rank, world):
    """--impl reference: the reference's own CPU path on the host cores (rank 0 only; the other
    ranks of a torchrun launch exit without work)."""
    if rank != 0:
        return
    threads = cpu_threads()
    torch.set_num_threads(threads)  # torchrun sets OMP_NUM_THREADS=1 for every rank
    smp = sized_cpu_sample(c, max(1.0, min(8.0, 150.0 / max(args.steps + args.warmup, 1))), threads)
    for _ in range(args.warmup):
        smp.run()
    times = [smp.run() for _ in range(args.steps)]
    sec = sum(times) / len(times)
    value = f_algo(c, smp.rows) / sec / 1e12
    line = {
        "metric": metric_name(args, c),
        "value": round(value, 4), "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1),
        "ms_per_step_scope": "one step = one bounded sample (cpu_baseline.sample); a whole-vocabulary step "
                             f"would take about {sec * c['V'] / smp.rows:.0f} s",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": ("fp32" if c.get("dtype") == "fp32" else "bf16 inputs") + ", fp32 CPU math", "data": "synthetic",
        "config": config_dict(args, c, 1),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": smp.kind, "sample": smp.describe()},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_gpu_arm(args, c, rank, world):
    """--impl reference-gpu: the reference GPU path's own JSON line (rank 0 alone)."""
    if rank != 0:
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    r = run_reference_gpu(args, c, device)
    base = {"metric": metric_name(args, c), "impl": "reference-gpu"}
    if "unavailable" in r:
        print(json.dumps({**base, **r}))
        return
    print(json.dumps({**base, "value": r["value"], "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                      "dtype": "bf16", "data": "synthetic (same inputs as ours)",
                      "config": config_dict(args, c, 1), **{k: v for k, v in r.items() if k not in ("value",
                                                                                                   "ms_per_step")}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"],
                    help="reference: the reference library's CPU path on the host cores (the reference arm); "
                         "reference-gpu: the reference library's own GPU path (cuBLAS + Triton) from the "
                         "offline install under baseline/_ref")
    ap.add_argument("--chunk", type=int, default=None, help="chunk_size (default: the API default, 8192)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference GPU path that a 1-GPU run times before its own arm")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    c = CONFIGS[args.config]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, c, rank, world)
        return
    if args.impl == "reference-gpu":
        run_reference_gpu_arm(args, c, rank, world)
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        ref_gpu = run_reference_gpu(args, c, device)
    r = run_ours(args, c, rank, world, device)

    if rank == 0:
        burst, sustained, peak_src = load_peaks()
        F = f_algo(c)
        value = F / (r["ms"] * 1e-3) / 1e12
        launches = sum(v[0] for v in r["prof"].values())
        per_step = {k: v[0] / args.steps for k, v in r["prof"].items()}
        kernels = {}
        for name, (n, tot) in r["prof"].items():
            fl = kernel_flops(name, c, r["Vr"], per_step[name], args.chunk)
            avg = tot / n
            kernels[name] = {"launches": n, "avg_ms": round(avg, 4), "share": round(tot / max(1e-9, sum(
                v[1] for v in r["prof"].values())), 4)}
            if fl:
                kernels[name]["algo_tflops"] = round(fl / (avg * 1e-3) / 1e12, 1)
            if name == "bwd_scores_kernel":  # with the S recompute, which F_algo leaves out
                ex = 2.0 * c["N"] * r["Vr"] * c["K"] / per_step[name] + (fl or 0.0)
                kernels[name]["exec_tflops"] = round(ex / (avg * 1e-3) / 1e12, 1)
        dom = max(r["prof"].items(), key=lambda kv: kv[1][1])[0]
        dom_fl = kernel_flops(dom, c, r["Vr"], per_step[dom], args.chunk)
        dom_avg = r["prof"][dom][1] / r["prof"][dom][0]
        achieved = dom_fl / (dom_avg * 1e-3) / 1e12 if dom_fl else None
        line = {
            "metric": metric_name(args, c),
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(r["ms"], 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32" if c.get("dtype") == "fp32" else "bf16",
            "data": "synthetic (seeded; BASELINE config distributions; one problem at every N)",
            "config": config_dict(args, c, world),
            "tflops_exec": round(f_exec(c) / (r["ms"] * 1e-3) / 1e12, 2),
            "frac_of_peak": {"measured_burst": round(value / burst, 4), "measured_sustained": round(value / sustained, 4),
                             "spec_2250": round(value / 2250.0, 4), "peak_source": peak_src},
            "peak_mem_gib": round(r["peak_gib"], 3),
            "checksums": r["checksums"],
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1) if achieved else None,
                         "peak": sustained, "unit": "TFLOP/s",
                         "frac": round(achieved / sustained, 4) if achieved else None,
                         "traffic": (CAPTURED_TRAFFIC_GB.get((args.config, dom))
                                     if world == 1 and args.chunk is None else None),
                         "traffic_unit": "GB per launch (ncu dram read + write)",
                         "peak_kind": f"{peak_src} sustained cuBLAS bf16 (kernel timed inside a long step)"},
            "kernels": kernels,
            "gpu_launches": launches,
            "clocks": r["clocks"],
            "e2e": {"value": round(F / (r["ms_e2e"] * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(r["ms_e2e"], 3), "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": 4,
                    "h2d_scope": ("per rank: each rank copies 1/N of the replicated h, target and weight from pinned "
                                  "host memory and NVLink all-gathers the rest (vocab_parallel.replicate_from_host)"
                                  if world > 1 else "whole job: pinned host buffers, double-buffered on the device; step "
                                  "i+1's inputs are copied on a side stream while step i computes, every copy inside "
                                  "the timed region"),
                    "clocks": r["e2e_clocks"]},
        }
        if ref_gpu is not None:
            if "unavailable" not in ref_gpu:
                ref_gpu["speedup_ours"] = round(ref_gpu["ms_per_step"] / r["ms"], 3)
                ref_gpu["checksum_max_rel_diff"] = checksum_agreement(r["checksums"], ref_gpu["checksums"])
            line["reference_gpu"] = ref_gpu
        if world == 1 and not args.no_cpu_baseline:
            threads = cpu_threads()
            torch.set_num_threads(threads)
            smp = sized_cpu_sample(c, 10.0, threads)
            sec = smp.run()
            cv = f_algo(c, smp.rows) / sec / 1e12
            line["cpu_baseline"] = {"value": round(cv, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                                    "kind": smp.kind, "sample": smp.describe() + f"; {sec:.1f} s"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
