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

--impl reference times the reference algorithm's PyTorch CPU path (the
oracle restatement in oracle/, the same torch operations as
cresso_v5.CRESSO5(cuda_ops='off')) on the host cores, on a bounded sample of
the workload (one tensor of the set per step), in the same unit.
"""

from __future__ import annotations

import argparse
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
# reference arm / CPU baseline: the reference algorithm's PyTorch CPU path
# ---------------------------------------------------------------------------
def cpu_reference_steps(shape, kw, istd, steps, warmup, budget_s=None):
    """Times `steps` CPU steps of the oracle restatement on one tensor; returns
    (seconds per step, elements per step, threads, sample description)."""
    from oracle import cresso5_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    p = torch.nn.Parameter(torch.randn(shape, generator=g) * istd)
    grads = [torch.randn(shape, generator=g) * 1e-3 for _ in range(2)]
    opt = O.OracleCRESSO5([p], **kw)
    for i in range(warmup):
        p.grad = grads[i % 2]
        opt.step()
    times = []
    for i in range(steps):
        p.grad = grads[i % 2]
        t0 = time.perf_counter()
        opt.step()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and sum(times) > budget_s:
            break
    return sum(times) / len(times), numel(shape), threads, len(times)


def reference_arm(args, world, rank):
    if rank != 0:
        return
    shapes, kw, istd = workload_shapes(args.workload)
    # bounded sample: one tensor of the set per step, shrunk until a step is a few seconds
    sample = max(shapes, key=lambda s: (numel(s) if numel(s) <= 4096 * 4096 else 0))
    t_probe, _, _, _ = cpu_reference_steps((min(sample[0], 1024),) + tuple(sample[1:]), kw, istd, 1, 0)
    per_elem = t_probe / numel((min(sample[0], 1024),) + tuple(sample[1:]))
    rows = sample[0]
    while rows > 256 and per_elem * rows * numel(sample[1:]) > 6.0:
        rows //= 2
    shape = (rows,) + tuple(sample[1:])
    sec, n, threads, done = cpu_reference_steps(shape, kw, istd, args.steps, args.warmup)
    value = BYTES_PER_ELEM * n / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": done, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload} sample {shape}", "rank": kw["rank"], "hash_bins": kw["hash_bins"],
                   "hash_tables": kw["hash_tables"], "path": "reference PyTorch CPU path (oracle restatement)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"one {shape} tensor of {args.workload} per step, {done} steps after "
                                   f"{args.warmup} warm-up"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def b200_arm(args, world, rank, local):
    import cresso_b200
    from cresso_b200 import _lib
    from cresso_b200.distributed import RowShardedCRESSO5, ZeroCRESSO5, mark_row_shard, row_block

    device = torch.device("cuda", local)
    zero = world > 1 and args.sharding == "zero"  # ZeRO-1: whole tensors, replicated inputs
    torch.cuda.set_device(device)
    shapes, kw, istd = workload_shapes(args.workload)
    params, grads_dev = [], []
    pdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}[args.dtype]
    bpe = 3 * torch.empty((), dtype=pdt).element_size()  # grad read + param read + param write
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + (0 if zero else rank))
    n_local = 0
    for i, s in enumerate(shapes):
        if world > 1 and not zero:
            start, stop = row_block(s[0], rank, world)
            local_shape = (stop - start,) + tuple(s[1:])
        else:
            start, local_shape = 0, tuple(s)
        p = torch.empty(local_shape, device=device)
        p.normal_(0.0, istd, generator=gen)
        p = torch.nn.Parameter(p.to(pdt))
        if world > 1 and not zero:
            mark_row_shard(p, s, start)
        g = torch.empty(local_shape, device=device)
        g.normal_(0.0, 1e-3, generator=gen)
        if args.workload == "c2":  # BASELINE c2: per-row log-normal(0, 0.5) gradient scale
            row_scale = torch.empty((local_shape[0], 1), device=device).normal_(0.0, 1.0, generator=gen)
            g.mul_(torch.exp(0.5 * row_scale))
        g = g.to(pdt)
        p.grad = g
        params.append(p)
        grads_dev.append(g)
        n_local += numel(local_shape)
    n_total = sum(numel(s) for s in shapes)
    if zero:
        opt = ZeroCRESSO5(params, bucket_elements=args.bucket_elements, **kw)
        n_local = sum(p.numel() for p in params if opt.owner[p] == rank)
        args.skip_e2e = True  # non-owned tensors carry no state to read back
    else:
        opt = RowShardedCRESSO5(params, **kw) if world > 1 else cresso_b200.CRESSO5(params, **kw)
    stream = torch.cuda.current_stream(device)

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
        barrier(world)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            opt.step()
        e1.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
    launches = _lib.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world, device)
    value = bpe * n_total / (ms * 1e-3) / 1e9

    # ---- per-pass kernel times (CUDA events on the launching stream, same steps)
    pass_ms = time_passes(opt, args, world, device, stream)
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

    # ---- CPU baseline (rank 0, N = 1)
    cpu = None
    if world == 1 and not args.skip_cpu:
        sample = (1024, 4096)
        sec, n, threads, done = cpu_reference_steps(sample, kw, istd, 2, 1, budget_s=30.0)
        cpu = {"value": BYTES_PER_ELEM * n / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"one {sample} tensor of {args.workload}, {done} steps after 1 warm-up, "
                         f"reference PyTorch CPU path (oracle restatement)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64" if args.dtype == "f64" else "f32", "data": "synthetic",
            "config": {"workload": f"{args.workload}: " + (f"7B-shaped {args.dtype} set, 290 tensors, 6,738,411,520 elements"
                                                            if args.workload == "c5" else str(shapes[0])),
                       "rank": kw["rank"], "hash_bins": kw["hash_bins"], "hash_tables": kw["hash_tables"],
                       "sharding": ((f"ZeRO-1 over {world} GPU(s), {len(opt.buckets)} buckets of >= "
                                     f"{args.bucket_elements} elements, all-gather of bucket k under the compute of "
                                     f"bucket k + 1" if args.bucket_elements > 0 else
                                     f"ZeRO-1 over {world} GPU(s), one all-gather after the step") if zero else
                                    f"row-sharded over {world} GPU(s)" if world > 1 else "single GPU"),
                       "l2": "no flush: inputs of every step (grads + params) exceed the 126 MB L2"
                             if n_total * 8 > 2 * 126e6 else "inputs fit in L2",
                       "elements": n_total, "per_pass_ms": {k: round(v, 4) for k, v in pass_ms.items()},
                       "param_dtype": args.dtype, "bytes_per_element": bpe},
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
        print(json.dumps(line), flush=True)


def time_passes(opt, args, world, device, stream):
    """Runs min(K, 3) more steps stage by stage with events around the five pass kernels."""
    from cresso_b200 import _lib
    import torch.distributed as dist

    from cresso_b200.distributed import RowShardedCRESSO5

    exchange = isinstance(opt, RowShardedCRESSO5)  # row sharding all-reduces between passes
    acc = {k: 0.0 for k in PASS_STAGE}
    acc["SCALAR"] = 0.0
    reps = max(1, min(args.steps, 3))
    orig = opt._spectral_stages
    orig_scalar = opt._run_scalar

    def scalar_timed(*a, **k):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        orig_scalar(*a, **k)
        ev1.record(stream)
        events.append(("SCALAR", ev0, ev1))

    def instrumented(run, scratch, layout):
        bounds = set(_lib.REDUCTION_BOUNDARIES)
        k = 0
        for st in range(_lib.SPECTRAL_STAGES):
            name = next((n for n, s in PASS_STAGE.items() if s == st), None)
            if name is not None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                run(st, st + 1)
                b.record(stream)
                events.append((name, a, b))
            else:
                run(st, st + 1)
            if st + 1 in bounds and world > 1 and exchange:
                k += 1
                dist.all_reduce(opt._reduction_view(scratch, layout, k))

    opt._spectral_stages = instrumented
    opt._run_scalar = scalar_timed
    try:
        for _ in range(reps):
            events = []
            opt.step()
            torch.cuda.synchronize(device)
            for name, a, b in events:
                acc[name] += a.elapsed_time(b)
    finally:
        opt._spectral_stages = orig
        opt._run_scalar = orig_scalar
    return {k: v / reps for k, v in acc.items() if v > 0.0}


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
    for p, g in zip(params, grads_dev):
        p.grad = g
    return {"value": bpe * n_total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_host.numel() * 4,
            "overlap": "step k+1's host->device gradient copy runs on a copy stream under step k"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="c5")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--dtype", choices=["f32", "bf16", "f16", "f64"], default="f32",
                    help="parameter / gradient type (work and state: float64 for f64, else float32)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--sharding", choices=["row", "zero"], default="row",
                    help="N > 1: row sharding (default) or ZeRO-1 whole-tensor partition")
    ap.add_argument("--bucket-elements", type=int, default=0,
                    help="ZeRO-1: elements per all-gather bucket (0: one bucket after the step)")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            reference_arm(args, world, rank)
        else:
            b200_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
