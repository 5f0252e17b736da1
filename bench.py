#!/usr/bin/env python
"""Benchmark of the CRESSO5 optimizer step (B200 build vs the reference CPU path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload c5]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload (default c5): the 7B-shaped fp32 parameter
set -- embed and lm_head (32000, 4096); 32 layers of q, k, v, o (4096, 4096),
gate, up (11008, 4096), down (4096, 11008) and two (4096,) norms --
rank 8, 64 hash bins, 2 tables, init N(0, 0.02), grads N(0, 1e-3), synthetic.
With N GPUs every tensor is row-sharded over the ranks (RowShardedCRESSO5: a
float64 NCCL all-reduce of the per-pass partial sums between passes), so the
total work is fixed ("scaling": "strong").  `--sharding zero` instead gives
every rank the full (replicated) set and partitions whole tensors
(ZeroCRESSO5; `--bucket-elements` > 0 overlaps each bucket's all-gather with
the next bucket's compute).

Metric: CRESSO5 ms/step and achieved HBM GB/s; `value` is the
whole-job algorithmic bandwidth 12 B x parameter elements / step time
(gradient read + parameter read + parameter write), device-resident inputs,
CUDA events, max over ranks.  `e2e` is the same metric through the public
optimizer API with the gradients copied host -> device from pinned memory
every step (double-buffered: the next step's copy overlaps the current step)
and a per-tensor drive-energy vector read back.

--impl reference times the reference's own PyTorch CPU path
(cresso_v5.CRESSO5(cuda_ops='off') of the unmodified reference installed into
baseline/_ref; the oracle restatement of the same torch operations if that is
absent) on all host cores, on a bounded sample of the workload (c5: one
(4096, 4096) weight of the set per step; c1-c4: the whole set), in the same
unit and with the same `config`.

The default run (c5, one GPU) adds `per_config`: c1, c2, c3, c4 and c4s (the
840 thin tensors on thin_matrix_route="spectral") timed the same way, and
`ref_cuda`: the same configs stepped by the reference's own CUDA extension
(`--impl reference-cuda` in a child process before this one allocates: the
unmodified package in baseline/_ref, JIT-built by its stock loader for
sm_100) with this build's speed-up over it per config.  With
N > 1 row-sharded GPUs the run first checks the sharded step against the
single-GPU step on this box (`parity` in the line; it exits non-zero above
1e-6 relative RMS or if the ranks' states differ) and reports the time of the
all-reduces between the passes (`exchange_ms`) and of the reduce / finalize
stages (`reduce_finalize_ms`) per step.
"""

from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "CRESSO5 ms/step and achieved HBM GB/s at 1/2/4/8 B200; vs host-CPU reference"
BYTES_PER_ELEM = 12  # grad read + param read + param write, fp32
# compulsory bytes per element of each pass kernel (the fp32 streams it must touch)
PASS_BYTES = {"P1": 4, "P2": 4, "P3": 8, "P4": 4, "P5": 12, "SCALAR": 12}
PASS_STAGE = {"P1": 1, "P2": 4, "P3": 7, "P4": 10, "P5": 13}


def workload_shapes(name: str):
    if name == "c5":
        shapes = [(32000, 4096), (32000, 4096)]
        for _ in range(32):
            shapes += [(4096, 4096)] * 4 + [(11008, 4096)] * 2 + [(4096, 11008)] + [(4096,)] * 2
        return shapes, dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 0.02
    if name == "c5layer":  # one layer of c5 (for the CPU baseline's extrapolation)
        return ([(4096, 4096)] * 4 + [(11008, 4096)] * 2 + [(4096, 11008)] + [(4096,)] * 2,
                dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 0.02)
    if name == "c5embed":  # the embedding / lm_head shape of c5
        return [(32000, 4096)], dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 0.02
    if name == "c2":
        return [(4096, 4096)], dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 0.02
    if name == "c1":
        return [(2048, 2048)], dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 0.02
    if name in ("c3", "c4", "c4s"):
        n = 64 if name == "c3" else 840
        shapes = [(4096, 16) if i % 2 == 0 else (16, 4096) for i in range(n)]
        kw = dict(lr=2e-3, rank=4, hash_bins=64, hash_tables=2)
        if name == "c4s":
            kw["thin_matrix_route"] = "spectral"
        return shapes, kw, 0.01
    raise SystemExit(f"unknown workload {name}")


def numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while a region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled: bool, uuids=None):
        self.proc = None
        self.enabled = enabled
        self.uuids = uuids or []

    def __enter__(self):
        if self.enabled:
            cmd = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100"]
            if self.uuids:
                cmd += ["-i", ",".join(self.uuids)]
            try:
                self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self, gpus=None):
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                idx = int(f[0])
            except ValueError:
                continue
            if gpus is not None and idx not in gpus:
                continue
            try:
                sm.append(float(f[1]))
                smax = max(smax, float(f[2]))
            except ValueError:
                pass
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if args.impl == "b200" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the reference's PyTorch CPU path
# ---------------------------------------------------------------------------
REF_DIR = ROOT / "baseline" / "_ref"


def reference_optimizer_class():
    """(CRESSO5 class, kind): the unmodified reference package installed under
    baseline/_ref (cresso_v5.CRESSO5 with cuda_ops='off', kind "reference"); if it
    is not installed, the oracle restatement of the same torch operations
    (kind "port")."""
    if (REF_DIR / "cresso_v5.py").exists():
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        import cresso_v5

        def make(params, **kw):
            return cresso_v5.CRESSO5(params, cuda_ops="off", **kw)
        return make, "reference"
    from oracle import cresso5_oracle as O

    return O.OracleCRESSO5, "port"


def cpu_model() -> str:
    try:
        for ln in subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def cpu_reference_steps(shapes, kw, istd, steps, warmup, budget_s=None, row_scale=False):
    """Times `steps` CPU steps of the reference path on a set of tensors (one
    optimizer over all of them, BASELINE inputs: init seed 0, fresh gradients
    each step); returns (seconds per step, elements per step, threads, steps
    timed, kind)."""
    make, kind = reference_optimizer_class()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(s, generator=g) * istd) for s in shapes]
    rs = None
    if row_scale:  # BASELINE c2: per-row log-normal(0, 0.5) gradient scale, drawn once (seed 7)
        rs = torch.exp(0.5 * torch.randn((shapes[0][0], 1), generator=torch.Generator().manual_seed(7)))
    opt = make(ps, **kw)

    def grads(step):
        gg = torch.Generator().manual_seed(1000 + step)
        for p in ps:
            x = torch.randn(p.shape, generator=gg) * 1e-3
            p.grad = x * rs if rs is not None else x

    for i in range(warmup):
        grads(i)
        opt.step()
    times = []
    for i in range(steps):
        grads(warmup + i)
        t0 = time.perf_counter()
        opt.step()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and sum(times) > budget_s:
            break
    return sum(times) / len(times), sum(numel(s) for s in shapes), threads, len(times), kind


def reference_sample(workload: str):
    """The bounded CPU sample of a workload: the whole set where a step takes
    seconds (c1-c4), one (4096, 4096) weight of the set per step for c5 (its
    per-element rate stands for the set: 226 of its 290 tensors are 4096-wide
    matrices)."""
    shapes, kw, istd = workload_shapes(workload)
    if workload == "c5":
        return [(4096, 4096)], kw, istd, "one (4096, 4096) weight of the 7B-shaped set per step"
    return shapes, kw, istd, f"the whole {workload} set per step"


def reference_arm(args, world, rank):
    if rank != 0:
        return
    shapes, kw, istd, what = reference_sample(args.workload)
    sec, n, threads, done, kind = cpu_reference_steps(shapes, kw, istd, args.steps, args.warmup, budget_s=240.0,
                                                      row_scale=args.workload == "c2")
    value = BYTES_PER_ELEM * n / sec / 1e9
    path = ("reference cresso_v5.CRESSO5(cuda_ops='off') from baseline/_ref, PyTorch CPU path" if kind == "reference"
            else "oracle restatement of the reference PyTorch CPU path")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": done, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, shapes_of(args.workload), kw, "f32"),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind, "cpu": cpu_model(),
                         "sample": f"{what}, {done} steps after {args.warmup} warm-up; {path}"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reference_cuda_arm(args, world, rank):
    """The reference's own CUDA extension on one GPU: the unmodified package in
    baseline/_ref, its stock JIT loader (cresso_cuda_ext.load_cuda_ops, built for
    sm_100 with TORCH_CUDA_ARCH_LIST=10.0, which its arch check accepts) and
    cresso_v5.CRESSO5(cuda_ops='required'), timed with CUDA events on the same
    BASELINE inputs, config by config.  Prints one JSON line with ms/step per
    config (c5: a few steps, its reference step takes seconds)."""
    if rank != 0:
        return
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    os.environ.setdefault("CRESSO_CUDA_BUILD_ROOT", str(ROOT / "baseline" / "_ref_build"))
    os.environ.setdefault("CRESSO_CUDA_MAX_JOBS", str(min(16, os.cpu_count() or 1)))
    if not (REF_DIR / "cresso_v5.py").exists():
        print(json.dumps({"impl": "reference-cuda", "unavailable": "reference not installed into baseline/_ref"}))
        return
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import cresso_v5

    device = torch.device("cuda", 0)
    t0 = time.perf_counter()
    cresso_v5._load_cuda_ops(required=True)
    build_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream(device)
    out = {}
    names = [w.strip() for w in args.ref_configs.split(",") if w.strip()]
    for name in names:
        shapes, kw, istd = workload_shapes(name)
        g = torch.Generator(device=device).manual_seed(1234)
        ps = []
        for shp in shapes:
            p = torch.nn.Parameter(torch.empty(shp, device=device).normal_(0.0, istd, generator=g))
            gr = torch.empty(shp, device=device).normal_(0.0, 1e-3, generator=g)
            if name == "c2":
                gr.mul_(torch.exp(0.5 * torch.empty((shp[0], 1), device=device).normal_(0.0, 1.0, generator=g)))
            p.grad = gr
            ps.append(p)
        opt = cresso_v5.CRESSO5(ps, cuda_ops="required", **kw)
        steps, warm = (2, 1) if name == "c5" else (args.steps, args.warmup)
        for _ in range(warm):
            opt.step()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            opt.step()
        e1.record(stream)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / steps
        n = sum(numel(x) for x in shapes)
        out[name] = {"ms_per_step": round(ms, 4), "value": round(BYTES_PER_ELEM * n / (ms * 1e-3) / 1e9, 3),
                     "unit": "GB/s", "steps": steps, "warmup": warm}
        print(json.dumps({"reference_cuda": name, **out[name]}), file=sys.stderr, flush=True)
        del opt, ps
        torch.cuda.empty_cache()
    line = {"impl": "reference-cuda", "metric": METRIC, "per_config": out, "n_gpus": 1,
            "path": "reference cresso_v5.CRESSO5(cuda_ops='required') from baseline/_ref, its JIT-built CUDA "
                    "extension (cresso_cuda_ext.load_cuda_ops) for sm_100",
            "build_or_load_s": round(build_s, 1), "torch_cuda_arch_list": os.environ["TORCH_CUDA_ARCH_LIST"]}
    print(json.dumps(line), flush=True)


def shapes_of(workload):
    return workload_shapes(workload)[0]


def workload_config(workload, shapes, kw, dtype):
    """The `config` object of a workload (identical for both arms)."""
    n_total = sum(numel(s) for s in shapes)
    desc = {"c5": f"7B-shaped {dtype} set, 290 tensors, 6,738,411,520 elements",
            "c3": "64 LoRA-thin (4096, 16) / (16, 4096), scalar route",
            "c4": "840 LoRA-thin (4096, 16) / (16, 4096), scalar route",
            "c4s": "840 LoRA-thin (4096, 16) / (16, 4096), thin_matrix_route='spectral'",
            "c5layer": "one layer of c5: 4 x (4096, 4096), 2 x (11008, 4096), (4096, 11008), 2 x (4096,)",
            "c5embed": "the (32000, 4096) embedding / lm_head shape of c5"}.get(workload, str(shapes[0]))
    return {"workload": f"{workload}: {desc}", "rank": kw["rank"], "hash_bins": kw["hash_bins"],
            "hash_tables": kw["hash_tables"], "elements": n_total,
            "l2": "flushed: inputs fit in the 126 MB L2, so every step is timed on its own with a "
                  "256 MB buffer written between steps, outside the timed intervals"
                  if fits_in_l2(n_total, 12 if dtype == "f32" else (6 if dtype in ("bf16", "f16") else 24))
                  else "no flush: inputs of every step (grads + params) exceed the 126 MB L2"}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def make_inputs(name, args, world, rank, device, zero):
    """Parameters (with gradients attached) of a workload on this rank: under row
    sharding row blocks of every 1-D / 2-D tensor on the spectral route and the
    other tensors whole (their owners step them), the whole set otherwise.
    Returns (shapes, kw, params, device gradients, local elements, total
    elements, bytes per element)."""
    import cresso_b200
    from cresso_b200._host import uses_spectral_route
    from cresso_b200.distributed import mark_row_shard, row_block

    shapes, kw, istd = workload_shapes(name)
    settings = cresso_b200.CRESSO5([torch.nn.Parameter(torch.zeros(1, device=device))], **kw).defaults
    pdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}[args.dtype]
    bpe = 3 * torch.empty((), dtype=pdt).element_size()  # grad read + param read + param write
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + (0 if zero else rank))
    params, grads_dev, n_local = [], [], 0
    for s in shapes:
        shard = world > 1 and not zero and len(s) <= 2 and uses_spectral_route(s, settings)
        if shard:
            start, stop = row_block(s[0], rank, world)
            local_shape = (stop - start,) + tuple(s[1:])
        else:
            start, local_shape = 0, tuple(s)
        p = torch.empty(local_shape, device=device)
        p.normal_(0.0, istd, generator=gen)
        p = torch.nn.Parameter(p.to(pdt))
        if shard:
            mark_row_shard(p, s, start)
        g = torch.empty(local_shape, device=device)
        g.normal_(0.0, 1e-3, generator=gen)
        if name == "c2":  # BASELINE c2: per-row log-normal(0, 0.5) gradient scale
            row_scale = torch.empty((local_shape[0], 1), device=device).normal_(0.0, 1.0, generator=gen)
            g.mul_(torch.exp(0.5 * row_scale))
        g = g.to(pdt)
        p.grad = g
        params.append(p)
        grads_dev.append(g)
        n_local += numel(local_shape)
    return shapes, kw, params, grads_dev, n_local, sum(numel(s) for s in shapes), bpe


L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def fits_in_l2(n_total, bpe):
    """Whether a step's inputs (gradients and parameters) could stay in L2 between steps."""
    return n_total * (2 * bpe // 3) <= 2 * 126e6


def time_steps(opt, steps, device, stream, world, flush=False):
    """Device time of exactly `steps` steps (CUDA events, barrier and synchronize on
    both sides, max over ranks), in ms per step.  With `flush` (inputs that fit in
    L2) every step is timed on its own and a 256 MB buffer is written between the
    steps, outside the timed intervals, so no step finds its inputs in L2."""
    gc.collect()  # no collection of an earlier workload's objects inside the timed steps
    buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device) if flush else None
    barrier(world)
    torch.cuda.synchronize(device)
    gc.disable()  # nor a collector pause (they reach milliseconds once a process holds many objects)
    try:
        if not flush:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                opt.step()
            e1.record(stream)
            torch.cuda.synchronize(device)
            ms = e0.elapsed_time(e1) / steps
        else:
            pairs = []
            for i in range(steps):
                buf.fill_(i & 255)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                opt.step()
                b.record(stream)
                pairs.append((a, b))
            torch.cuda.synchronize(device)
            ms = sum(a.elapsed_time(b) for a, b in pairs) / steps
    finally:
        gc.enable()
    barrier(world)
    return max_over_ranks(ms, world, device)


def sharded_parity_check(world, rank, device, steps=3):
    """Correctness of the row-sharded step on this box, before anything is timed:
    every rank steps its row block of one (4096, 4096) and one (4096,) tensor for
    `steps` steps (RowShardedCRESSO5), rank 0 steps the same whole tensors with
    the single-GPU CRESSO5, and the blocks are gathered (each rank adds its rows
    into a zero tensor, SUM-all-reduced: exact).  Returns the relative RMS of the
    parameters, the largest relative RMS of a state tensor against the
    single-GPU state, and whether every rank holds bitwise the same state."""
    import cresso_b200
    import torch.distributed as dist

    from cresso_b200.distributed import RowShardedCRESSO5, mark_row_shard, row_block

    shapes = [(4096, 4096), (4096,)]
    kw = dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2)
    g = torch.Generator(device=device).manual_seed(77)  # the same inputs on every rank
    inits = [torch.randn(s, generator=g, device=device) * 0.02 for s in shapes]
    grads = [[torch.randn(s, generator=g, device=device) * 1e-3 for s in shapes] for _ in range(steps)]
    local = []
    for s, x in zip(shapes, inits):
        a, b = row_block(s[0], rank, world)
        p = torch.nn.Parameter(x[a:b].clone())
        mark_row_shard(p, s, a)
        local.append((p, a, b))
    opt = RowShardedCRESSO5([p for p, _, _ in local], **kw)
    for gs in grads:
        for (p, a, b), gg in zip(local, gs):
            p.grad = gg[a:b].clone()
        opt.step()
    opt.check_device_status()
    full = []
    for (p, a, b), s in zip(local, shapes):
        t = torch.zeros(s, device=device)
        t[a:b] = p.detach()
        dist.all_reduce(t)
        full.append(t)
    identical = True
    states = [opt.state[p] for p, _, _ in local]
    for st in states:
        for k, v in sorted(st.items()):
            if torch.is_tensor(v) and v.is_floating_point():
                hi, lo = v.detach().clone(), v.detach().clone()
                dist.all_reduce(hi, op=dist.ReduceOp.MAX)
                dist.all_reduce(lo, op=dist.ReduceOp.MIN)
                identical = identical and bool(torch.equal(hi, lo))
    flag = torch.tensor([1.0 if identical else 0.0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    out = {"param_rel_rms": None, "state_max_rel": None, "state_identical_across_ranks": bool(flag.item() == 1.0),
           "shapes": [list(s) for s in shapes], "steps": steps}
    bad = torch.zeros(1, device=device)
    if rank == 0:
        ps = [torch.nn.Parameter(x.clone()) for x in inits]
        ref = cresso_b200.CRESSO5(ps, **kw)
        for gs in grads:
            for p, gg in zip(ps, gs):
                p.grad = gg.clone()
            ref.step()
        torch.cuda.synchronize(device)

        def rel(a, b):
            a, b = a.double(), b.double()
            return float(torch.sqrt(torch.mean((a - b) ** 2)) / (torch.sqrt(torch.mean(b * b)) + 1e-30))

        out["param_rel_rms"] = max(rel(f, p.detach()) for f, p in zip(full, ps))
        out["state_max_rel"] = max(rel(st[k], ref.state[p][k]) for st, p in zip(states, ps)
                                   for k, v in st.items() if torch.is_tensor(v) and v.is_floating_point())
        if out["param_rel_rms"] > 1e-6 or not out["state_identical_across_ranks"]:
            bad.fill_(1.0)
    dist.all_reduce(bad)  # every rank learns the verdict
    out["ok"] = bool(bad.item() == 0.0)
    del opt, local, full
    torch.cuda.empty_cache()
    return out


def quick_config(name, args, device, stream):
    """One more BASELINE config on this GPU (N = 1): device time of args.steps steps
    after args.warmup, and the end-to-end time through CRESSO5.step() with host
    gradients."""
    import cresso_b200

    shapes, kw, params, grads_dev, n_local, n_total, bpe = make_inputs(name, args, 1, 0, device, False)
    opt = cresso_b200.CRESSO5(params, **kw)
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize(device)
    ms = time_steps(opt, args.steps, device, stream, 1, flush=fits_in_l2(n_total, bpe))
    e2e = time_e2e(opt, params, grads_dev, args, 1, device, stream, n_total, bpe)
    opt.check_device_status()
    out = {"ms_per_step": round(ms, 5), "value": round(bpe * n_total / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
           "elements": n_total, "workload": workload_config(name, shapes, kw, args.dtype)["workload"],
           "l2": workload_config(name, shapes, kw, args.dtype)["l2"],
           "e2e": {"value": round(e2e["value"], 3), "ms_per_step": round(e2e["ms_per_step"], 5)}}
    del opt, params, grads_dev
    torch.cuda.empty_cache()
    return out


def reference_cuda_subprocess(timeout_s=600):
    """The reference CUDA extension timed in a child process (its own CUDA context,
    run before this process allocates the workload), per BASELINE config; None
    fields name why it is missing."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference-cuda", "--steps", "10", "--warmup", "3"]
    env = dict(os.environ)
    env.setdefault("CRESSO_CUDA_BUILD_ROOT", str(ROOT / "baseline" / "_ref_build"))
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s, env=env, cwd=str(ROOT))
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference CUDA build and timing exceeded {timeout_s} s"}
    for ln in reversed(r.stdout.splitlines()):
        try:
            d = json.loads(ln)
        except ValueError:
            continue
        if d.get("impl") == "reference-cuda":
            return d
    return {"unavailable": f"reference CUDA run failed (rc {r.returncode}): {r.stderr.strip()[-300:]}"}


def b200_arm(args, world, rank, local):
    from cresso_b200 import _lib
    import cresso_b200
    from cresso_b200.distributed import RowShardedCRESSO5, ZeroCRESSO5

    # ---- the reference's own CUDA extension on this GPU, before this process allocates (default run)
    ref_cuda = None
    if world == 1 and args.workload == "c5" and not args.skip_configs and not args.skip_ref_cuda:
        ref_cuda = reference_cuda_subprocess()

    device = torch.device("cuda", local)
    zero = world > 1 and args.sharding == "zero"  # ZeRO-1: whole tensors, replicated inputs
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)

    # ---- multi-GPU: correctness of the sharded step on this box before any timing
    parity = None
    if world > 1 and not zero:
        parity = sharded_parity_check(world, rank, device)
        if rank == 0:
            print(json.dumps({"sharded_parity": parity}), file=sys.stderr, flush=True)
        if not parity["ok"]:
            raise SystemExit(f"row-sharded step differs from the single-GPU step: {parity}")

    shapes, kw, params, grads_dev, n_local, n_total, bpe = make_inputs(args.workload, args, world, rank, device, zero)
    if zero:
        opt = ZeroCRESSO5(params, bucket_elements=args.bucket_elements, **kw)
        n_local = sum(p.numel() for p in params if opt.owner[p] == rank)
        args.skip_e2e = True  # non-owned tensors carry no state to read back
    else:
        opt = RowShardedCRESSO5(params, **kw) if world > 1 else cresso_b200.CRESSO5(params, **kw)

    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize(device)

    # ---- device-resident timing of exactly K steps
    uuids = []
    for i in range(torch.cuda.device_count()):
        try:
            u = str(torch.cuda.get_device_properties(i).uuid)
            uuids.append(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:
            pass
    launches0 = _lib.launch_count()
    with ClockSampler(rank == 0, uuids) as clk:
        ms = time_steps(opt, args.steps, device, stream, world, flush=fits_in_l2(n_total, bpe))
    launches = _lib.launch_count() - launches0
    opt.check_device_status()
    value = bpe * n_total / (ms * 1e-3) / 1e9

    # ---- per-pass kernel times (CUDA events on the launching stream, same steps)
    pass_ms, extra_ms = time_passes(opt, args, world, device, stream)
    if pass_ms:
        dom = max(pass_ms, key=pass_ms.get)
        dom_ms = max_over_ranks(pass_ms[dom], world, device)
        dom_bytes = PASS_BYTES[dom]
    else:  # float64: its own pipeline, timed as a whole step
        dom, dom_ms, dom_bytes = "step", ms, bpe
    peaks, peak_kind = measured_peaks()
    achieved = dom_bytes * n_local / (dom_ms * 1e-3) / 1e9
    traffic = None
    try:
        tr = json.loads((ROOT / "profiles" / "traffic_per_element.json").read_text())
        if dom in tr.get("bytes_per_element", {}):
            traffic = tr["bytes_per_element"][dom] * n_local
    except Exception:
        pass

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.skip_e2e:
        e2e = time_e2e(opt, params, grads_dev, args, world, device, stream, n_total, bpe)

    # ---- the other BASELINE configs on one GPU (default run only)
    per_config = None
    if world == 1 and args.workload == "c5" and not args.skip_configs:
        del opt, params, grads_dev
        torch.cuda.empty_cache()
        per_config = {name: quick_config(name, args, device, stream) for name in ("c1", "c2", "c3", "c4", "c4s")}

    # ---- CPU baseline (rank 0, N = 1): the reference PyTorch CPU path on a bounded sample
    cpu = None
    if world == 1 and not args.skip_cpu:
        cshapes, ckw, cistd, what = reference_sample(args.workload)
        sec, n, threads, done, kind = cpu_reference_steps(cshapes, ckw, cistd, 2, 1, budget_s=30.0,
                                                          row_scale=args.workload == "c2")
        cpu = {"value": BYTES_PER_ELEM * n / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
               "cpu": cpu_model(),
               "sample": f"{what}, {done} steps after 1 warm-up, "
                         + ("reference cresso_v5.CRESSO5(cuda_ops='off') from baseline/_ref" if kind == "reference"
                            else "oracle restatement of the reference PyTorch CPU path")}

    if rank == 0:
        config = workload_config(args.workload, shapes, kw, args.dtype)
        config.update({
            "sharding": ((f"ZeRO-1 over {world} GPU(s), {len(opt.buckets)} buckets of >= "
                          f"{args.bucket_elements} elements, all-gather of bucket k under the compute of "
                          f"bucket k + 1" if args.bucket_elements > 0 else
                          f"ZeRO-1 over {world} GPU(s), one all-gather after the step") if zero else
                         f"row-sharded over {world} GPU(s)" if world > 1 else "single GPU"),
            "per_pass_ms": {k: round(v, 4) for k, v in pass_ms.items()},
            "param_dtype": args.dtype, "bytes_per_element": bpe})
        if extra_ms:
            config.update({k: round(v, 4) for k, v in extra_ms.items()})
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64" if args.dtype == "f64" else "f32", "data": "synthetic",
            "config": config,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "algorithmic_bytes_per_element": dom_bytes,
                         "step_frac": value / world / peaks["hbm_gbs"]},
            "clocks": clk.summary(),
            "gpu_launches": launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if per_config is not None:
            line["per_config"] = per_config
        if ref_cuda is not None:
            ours = dict(per_config or {})
            ours["c5"] = {"ms_per_step": ms}
            rc = {"path": ref_cuda.get("path"), "unavailable": ref_cuda.get("unavailable")}
            for name, v in (ref_cuda.get("per_config") or {}).items():
                mine = ours.get(name, {}).get("ms_per_step")
                rc[name] = {"ms_per_step": v["ms_per_step"], "steps": v["steps"],
                            "speedup": round(v["ms_per_step"] / mine, 2) if mine else None}
            line["ref_cuda"] = rc
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line), flush=True)


def time_passes(opt, args, world, device, stream):
    """Runs min(K, 3) more steps stage by stage with events around the five pass
    kernels, the reduce / finalize stages between them, and (row sharding) the
    all-reduces of the reduction vectors.  Returns (per-pass ms, other ms)."""
    from cresso_b200 import _lib
    import torch.distributed as dist

    from cresso_b200.distributed import RowShardedCRESSO5

    exchange = isinstance(opt, RowShardedCRESSO5) and world > 1  # row sharding all-reduces between passes
    acc = {k: 0.0 for k in PASS_STAGE}
    acc["SCALAR"] = 0.0
    other = {"reduce_finalize_ms": 0.0}
    last = {}
    reps = max(1, min(args.steps, 3))
    orig = opt._spectral_stages
    orig_scalar = opt._run_scalar

    def scalar_timed(*a, **k):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        orig_scalar(*a, **k)
        ev1.record(stream)
        events.append(("SCALAR", ev0, ev1))

    def timed(name, fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        events.append((name, a, b))

    def instrumented(run, scratch, layout):
        bounds = set(_lib.REDUCTION_BOUNDARIES)
        k = 0
        for st in range(_lib.SPECTRAL_STAGES):
            name = next((n for n, s in PASS_STAGE.items() if s == st), None)
            timed(name if name is not None else "reduce_finalize_ms", lambda st=st: run(st, st + 1))
            if st + 1 in bounds and exchange:
                k += 1
                dist.all_reduce(opt._reduction_view(scratch, layout, k), group=opt.process_group)
        last["scratch"], last["layout"] = scratch, layout

    opt._spectral_stages = instrumented
    opt._run_scalar = scalar_timed
    pipelined = getattr(opt, "pipeline_exchange", False)
    if pipelined:  # per-pass times of the unsplit group: the exchange is timed on its own
        opt.pipeline_exchange = False
    try:
        for _ in range(reps):
            events = []
            opt.step()
            torch.cuda.synchronize(device)
            for name, a, b in events:
                if name in other:
                    other[name] += a.elapsed_time(b)
                else:
                    acc[name] += a.elapsed_time(b)
    finally:
        opt._spectral_stages = orig
        opt._run_scalar = orig_scalar
        if pipelined:
            opt.pipeline_exchange = True
    extra = {k: max_over_ranks(v / reps, world, device) for k, v in other.items() if v > 0.0}
    if exchange and last:
        # the four float64 all-reduces of a step on their own, after a barrier (the
        # in-step time would include one rank waiting for the other's pass)
        views = [opt._reduction_view(last["scratch"], last["layout"], k) for k in range(1, 5)]
        ex = 0.0
        for _ in range(reps):
            torch.cuda.synchronize(device)
            barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for v in views:
                dist.all_reduce(v, group=opt.process_group)
            b.record(stream)
            torch.cuda.synchronize(device)
            ex += a.elapsed_time(b)
        extra["exchange_ms"] = max_over_ranks(ex / reps, world, device)
        extra["exchange_bytes"] = int(sum(v.numel() * 8 for v in views))
    return {k: v / reps for k, v in acc.items() if v > 0.0}, extra


def time_e2e(opt, params, grads_dev, args, world, device, stream, n_total, bpe=BYTES_PER_ELEM):
    """Gradients from pinned host memory each step, drive energies read back each step.

    The gradients are double-buffered on the device: step k+1's host -> device
    copy runs on a copy stream while step k computes (input prefetch, as a
    training loop's loader does), so a step costs max(copy, compute).  Every
    step's full gradient copy and result read lies inside the timed region."""
    # all gradients of a step in one flat pinned host buffer (as a training loop's
    # gradient buckets hold them) and two flat device buffers; the gradients are views
    dtype = grads_dev[0].dtype
    sizes = [g.numel() for g in grads_dev]
    offs, total = [], 0
    for n in sizes:  # each gradient starts on a 256-byte boundary
        offs.append(total)
        total += (n + 63) // 64 * 64
    host_flat = torch.zeros(total, dtype=dtype, pin_memory=True)
    for g, n, off in zip(grads_dev, sizes, offs):
        host_flat[off:off + n].copy_(g.reshape(-1))
    h2d = total * host_flat.element_size()
    out_host = torch.empty(len(params), dtype=torch.float32, pin_memory=True)
    dev_flat = [torch.empty(total, dtype=dtype, device=device) for _ in range(2)]
    bufs = []
    for flat in dev_flat:
        bufs.append([flat[off:off + n].view(g.shape) for g, n, off in zip(grads_dev, sizes, offs)])
    copy_stream = torch.cuda.Stream(device)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    stepped = [torch.cuda.Event(), torch.cuda.Event()]

    def copy_in(k):  # step k's gradients into buffer k % 2, after step k - 2 released it
        b = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(stepped[b])
            dev_flat[b].copy_(host_flat, non_blocking=True)
            copied[b].record(copy_stream)

    def run(n):
        for k in range(n):
            b = k % 2
            if k + 1 < n:
                copy_in(k + 1)
            stream.wait_event(copied[b])
            for p, g in zip(params, bufs[b]):
                p.grad = g
            opt.step()
            stepped[b].record(stream)
            de = torch.stack([opt.state[p]["drive_energy"] for p in params])
            out_host.copy_(de, non_blocking=True)

    for b in range(2):
        stepped[b].record(stream)
    copy_in(0)
    run(max(1, args.warmup))
    torch.cuda.synchronize(device)
    gc.collect()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for b in range(2):
        stepped[b].record(stream)
    copy_in(0)  # step 0's copy starts after e0: inside the timed region
    run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, device)
    # the copy bound: the same pinned host -> device gradient copy alone, on every rank at once
    barrier(world)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(copy_stream)
    reps = 2
    with torch.cuda.stream(copy_stream):
        for _ in range(reps):
            dev_flat[0].copy_(host_flat, non_blocking=True)
    c1.record(copy_stream)
    torch.cuda.synchronize(device)
    copy_ms = max_over_ranks(c0.elapsed_time(c1) / reps, world, device)
    for p, g in zip(params, grads_dev):
        p.grad = g
    return {"value": bpe * n_total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_host.numel() * 4,
            "overlap": "step k+1's host->device gradient copy runs on a copy stream under step k",
            "copy_bound": {"ms": copy_ms, "gbs_per_rank": h2d / (copy_ms * 1e-3) / 1e9,
                           "note": "the step's pinned host->device gradient copy timed alone, all ranks at "
                                   "once (max over ranks): e2e ms_per_step cannot go below max(this, the "
                                   "device step)"}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference", "reference-cuda"], default="b200")
    ap.add_argument("--ref-configs", default="c1,c2,c3,c4,c4s,c5",
                    help="--impl reference-cuda: the BASELINE configs to time")
    ap.add_argument("--workload", default="c5")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--dtype", choices=["f32", "bf16", "f16", "f64"], default="f32",
                    help="parameter / gradient type (work and state: float64 for f64, else float32)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-configs", action="store_true", help="default c5 run: leave out the c1-c4 lines")
    ap.add_argument("--skip-ref-cuda", action="store_true",
                    help="default c5 run: leave out the reference CUDA extension timings (ref_cuda)")
    ap.add_argument("--sharding", choices=["row", "zero"], default="row",
                    help="N > 1: row sharding (default) or ZeRO-1 whole-tensor partition")
    ap.add_argument("--bucket-elements", type=int, default=0,
                    help="ZeRO-1: elements per all-gather bucket (0: one bucket after the step)")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            reference_arm(args, world, rank)
        elif args.impl == "reference-cuda":
            reference_cuda_arm(args, world, rank)
        else:
            b200_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
