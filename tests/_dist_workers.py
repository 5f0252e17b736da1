"""Process entry points for the multi-process tests (importable by spawn)."""

from __future__ import annotations

import datetime
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _init(rank, world, port, backend, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def stages_worker(rank, world, port, outdir):
    """RowShardedCRESSO5 stage orchestration with a fake kernel runner (gloo)."""
    from cresso_b200 import _lib
    from cresso_b200.distributed import RowShardedCRESSO5

    _init(rank, world, port, "gloo")
    opt = RowShardedCRESSO5([torch.nn.Parameter(torch.zeros(4))], process_group=None)
    layout = np.zeros(9, dtype=np.int64)
    # four reduction vectors at 256-byte offsets with lengths 1, 5, 3, 29
    lens = [1, 5, 3, 29]
    off = 0
    for k, n in enumerate(lens, start=1):
        layout[2 * k - 1] = off
        layout[2 * k] = n
        off += (8 * n + 255) // 256 * 256
    scratch = torch.zeros(off, dtype=torch.uint8)
    calls = []

    def run(b, e):
        calls.append((b, e))
        # the stage that completes vector k writes rank+1 into it
        for k, bound in enumerate(_lib.REDUCTION_BOUNDARIES, start=1):
            if e == bound:
                opt._reduction_view(scratch, layout, k).fill_(float(rank + 1) * k)

    opt._spectral_stages(run, scratch, layout)
    out = [opt._reduction_view(scratch, layout, k).clone() for k in range(1, 5)]
    torch.save({"calls": calls, "out": out}, os.path.join(outdir, f"stages_{rank}.pt"))
    dist.destroy_process_group()


def zero_gather_worker(rank, world, port, outdir, bucket_elements=0):
    from cresso_b200.distributed import ZeroCRESSO5

    _init(rank, world, port, "gloo")
    shapes = [(7, 5), (13,), (4, 4), (30,), (2, 3), (3, 3, 3), (11,), (5, 8)]
    ps = [torch.nn.Parameter(torch.full(s, -1.0)) for s in shapes]
    ps[6].data = ps[6].data.double()  # a second dtype: one all-gather per (bucket, dtype)
    opt = ZeroCRESSO5(ps, bucket_elements=bucket_elements)
    for i, p in enumerate(ps):
        if opt.owner[p] == rank:
            p.data.fill_(float(100 * i + 7))
    opt.gather_params()
    index = {id(p): j for j, p in enumerate(ps)}
    plan = [[[index[id(p)] for p in run] for run in bucket] for bucket in opt.buckets]
    torch.save({"vals": [p.detach().clone() for p in ps], "owner": [opt.owner[p] for p in ps], "plan": plan},
               os.path.join(outdir, f"zero_{rank}_{bucket_elements}.pt"))
    dist.destroy_process_group()


def zero_gather_bucketed_worker(rank, world, port, outdir):
    zero_gather_worker(rank, world, port, outdir, bucket_elements=20)


def gpu_zero_worker(rank, world, port, outdir):
    """Bucketed ZeRO-1 CUDA step on `world` GPUs against the single-GPU step."""
    import cresso_b200
    from cresso_b200.distributed import ZeroCRESSO5

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl", timeout_s=120)
    dev = torch.device("cuda", rank)
    g = torch.Generator().manual_seed(4)
    shapes = [(256, 192), (1536,), (96, 64), (512, 16), (7, 9), (128, 128), (4, 8, 3, 3)]
    inits = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s in shapes] for _ in range(3)]
    kw = dict(rank=8, hash_bins=64, hash_tables=2)
    ps = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
    opt = ZeroCRESSO5(ps, bucket_elements=20000, **kw)
    for gs in grads:
        for p, gg in zip(ps, gs):
            p.grad = gg.clone().to(dev)
        opt.step()
    torch.cuda.synchronize()
    out = [p.detach().cpu() for p in ps]
    ref_out = None
    if rank == 0:
        full = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
        ref = cresso_b200.CRESSO5(full, **kw)
        for gs in grads:
            for p, gg in zip(full, gs):
                p.grad = gg.to(dev)
            ref.step()
        torch.cuda.synchronize()
        ref_out = [p.detach().cpu() for p in full]
    torch.save({"params": out, "ref": ref_out, "n_buckets": len(opt.buckets),
                "owned": [opt.owner[p] == rank for p in ps]}, os.path.join(outdir, f"gpu_zero_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def failing_rank_worker(rank, world, port, outdir):
    """Rank 1 fails before the first exchange; rank 0 must see an error, not hang."""
    from cresso_b200.distributed import RowShardedCRESSO5

    _init(rank, world, port, "gloo", timeout_s=5)
    opt = RowShardedCRESSO5([torch.nn.Parameter(torch.zeros(4))])
    layout = np.zeros(9, dtype=np.int64)
    for k in range(1, 5):
        layout[2 * k - 1] = 256 * (k - 1)
        layout[2 * k] = 4
    scratch = torch.zeros(1024, dtype=torch.uint8)

    def run(b, e):
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")

    t0 = time.time()
    status = "ok"
    try:
        opt._spectral_stages(run, scratch, layout)
    except Exception as exc:  # the survivor's collective ends with an error
        status = type(exc).__name__ + ": " + str(exc)[:200]
    with open(os.path.join(outdir, f"fail_{rank}.txt"), "w") as f:
        f.write(f"{status}\n{time.time() - t0:.2f}\n")
    # no destroy_process_group: the peer is gone


def gpu_row_shard_worker(rank, world, port, outdir):
    """Row-sharded CUDA step on `world` GPUs against the single-GPU step."""
    import cresso_b200
    from cresso_b200.distributed import RowShardedCRESSO5, mark_row_shard, row_block

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl", timeout_s=120)
    dev = torch.device("cuda", rank)
    g = torch.Generator().manual_seed(3)
    shapes = [(256, 192), (1536,), (96, 64)]
    # passed whole in the same group: LoRA-thin and small (scalar route), a 4-D and an
    # unmarked 2-D spectral tensor; each is stepped by its owner and all-gathered
    whole_shapes = [(512, 16), (7, 9), (8, 16, 3, 3), (80, 48), (16, 300)]
    inits = [torch.randn(s, generator=g) * 0.02 for s in shapes + whole_shapes]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s in shapes + whole_shapes] for _ in range(3)]
    kw = dict(rank=8, hash_bins=64, hash_tables=2, min_spectral_size=1024)
    ps = []
    for s, x in zip(shapes, inits):
        a, b = row_block(s[0], rank, world)
        p = torch.nn.Parameter(x[a:b].clone().to(dev))
        mark_row_shard(p, s, a)
        ps.append(p)
    ws = [torch.nn.Parameter(x.clone().to(dev)) for x in inits[len(shapes):]]
    opt = RowShardedCRESSO5(ps + ws, **kw)
    for gs in grads:
        for p, s, gg in zip(ps, shapes, gs):
            a, b = row_block(s[0], rank, world)
            p.grad = gg[a:b].clone().to(dev)
        for p, gg in zip(ws, gs[len(shapes):]):
            p.grad = gg.clone().to(dev)
        opt.step()
    torch.cuda.synchronize()
    shard = [p.detach().cpu() for p in ps]
    states = [{k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in ps]
    whole = [p.detach().cpu() for p in ws]
    whole_states = [{k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in ws]
    owners = next(iter(opt._whole_plans.values()))[1][3]
    if rank == 0:
        full = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
        ref = cresso_b200.CRESSO5(full, **kw)
        for gs in grads:
            for p, gg in zip(full, gs):
                p.grad = gg.to(dev)
            ref.step()
        torch.cuda.synchronize()
        ref_out = ([p.detach().cpu() for p in full],
                   [{k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in ref.state[p].items()} for p in full])
    else:
        ref_out = None
    torch.save({"shard": shard, "states": states, "whole": whole, "whole_states": whole_states, "owners": owners,
                "n_sharded": len(shapes), "ref": ref_out}, os.path.join(outdir, f"gpu_rs_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def zero_consolidate_worker(rank, world, port, outdir):
    """consolidate_state_dict on CPU ranks: each rank fakes the state of the
    tensors it owns (as a step would leave it); rank 0 collects all of them."""
    from cresso_b200.distributed import ZeroCRESSO5

    _init(rank, world, port, "gloo")
    shapes = [(7, 5), (13,), (4, 4), (30,), (2, 3)]
    ps = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    opt = ZeroCRESSO5(ps)
    for i, p in enumerate(ps):
        if opt.owner[p] == rank:
            opt.state[p] = {"step": 3, "force_rms": torch.tensor(float(i)), "q": torch.full((2,), float(10 * i))}
    sd = opt.consolidate_state_dict(to=0)
    torch.save({"sd": sd, "owner": [opt.owner[p] for p in ps]}, os.path.join(outdir, f"consolidate_{rank}.pt"))
    dist.destroy_process_group()


def status_exchange_worker(rank, world, port, outdir):
    """A device-side failure reported on rank 1 only reaches every rank after the
    per-step status exchange, and every rank's next check raises (gloo; the
    failure word is a host tensor here, set as a kernel would set it)."""
    from cresso_b200.distributed import RowShardedCRESSO5, exchange_status

    _init(rank, world, port, "gloo")
    opt = RowShardedCRESSO5([torch.nn.Parameter(torch.zeros(4))])
    word = opt._status_word(torch.device("cpu"))
    if rank == 1:
        word.fill_(1)  # as the kernels OR bit 1 in after a bounded wait gave up
    before = int(word.item())
    exchange_status(opt)
    after = int(word.item())
    raised = ""
    try:
        opt.check_device_status()
    except RuntimeError as exc:
        raised = str(exc)[:300]
    with open(os.path.join(outdir, f"status_{rank}.txt"), "w") as f:
        f.write(f"{before}\n{after}\n{raised}\n")
    dist.destroy_process_group()


def zero_deferred_gather_worker(rank, world, port, outdir):
    """Deferred ZeRO-1 all-gathers finished by forward pre-hooks (gloo, CPU): the
    parameters another rank owns stay stale until a module using them runs."""
    from cresso_b200.distributed import ZeroCRESSO5

    _init(rank, world, port, "gloo")
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(4, 5), torch.nn.Linear(5, 3))
    for p in model.parameters():
        p.data.fill_(-1.0)
    # one tensor per bucket: bucket 0 holds both tensors of the first layer (the LPT
    # partition gives rank 0 the weight and rank 1 the bias), bucket 1 the second layer's
    opt = ZeroCRESSO5(list(model.parameters()), defer_gather=True, bucket_elements=1)
    opt.prefetch_forward(model)
    ps = list(model.parameters())
    for i, p in enumerate(ps):
        if opt.owner[p] == rank:
            p.data.fill_(float(10 * i + 1))
    for bucket in opt.buckets:  # what a deferred step does after its compute
        opt._defer(opt._gather_bucket_async(bucket))
    stale_before = [bool(torch.all(p == -1.0)) for p in ps]
    model[0](torch.zeros(2, 4))  # the first layer only: its parameters are finished
    after_first = [bool(torch.all(p == float(10 * i + 1))) for i, p in enumerate(ps)]
    opt.wait_params()
    after_all = [bool(torch.all(p == float(10 * i + 1))) for i, p in enumerate(ps)]
    torch.save({"owner": [opt.owner[p] for p in ps], "stale_before": stale_before, "after_first": after_first,
                "after_all": after_all}, os.path.join(outdir, f"zdefer_{rank}.pt"))
    dist.destroy_process_group()


def gpu_zero_deferred_worker(rank, world, port, outdir):
    """A small model trained three steps with deferred, forward-finished ZeRO-1
    all-gathers against the same training with gathers finished in the step."""
    from cresso_b200.distributed import ZeroCRESSO5

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl", timeout_s=120)
    dev = torch.device("cuda", rank)
    outs = []
    for defer in (False, True):
        torch.manual_seed(3)
        model = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 256),
                                    torch.nn.GELU(), torch.nn.Linear(256, 64)).to(dev)
        opt = ZeroCRESSO5(list(model.parameters()), defer_gather=defer, bucket_elements=50000, rank=8,
                          hash_bins=64, hash_tables=2)
        if defer:
            opt.prefetch_forward(model)
        g = torch.Generator(device=dev).manual_seed(7)
        for _ in range(3):
            x = torch.randn(32, 256, device=dev, generator=g)
            loss = model(x).square().mean()
            model.zero_grad()
            loss.backward()
            opt.step()
        opt.wait_params()
        torch.cuda.synchronize()
        outs.append([p.detach().cpu().clone() for p in model.parameters()])
    torch.save({"plain": outs[0], "deferred": outs[1]}, os.path.join(outdir, f"gpu_zdefer_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def whole_broadcast_worker(rank, world, port, outdir):
    """The whole-tensor exchange on CPU ranks: each rank writes distinctive values
    into the tensors it owns and garbage elsewhere; afterwards every rank holds the
    owners' parameters and floating state (float32 and float64), and integer
    state is left alone."""
    from cresso_b200.distributed import broadcast_whole, lpt_partition

    _init(rank, world, port, "gloo")
    shapes = [(7, 5), (13,), (4, 4, 2), (30,), ()]
    items = []
    for s in shapes:
        st = {"step": 3, "q": torch.full((), -1.0), "metric": torch.full(s, -1.0, dtype=torch.float64),
              "freqs": torch.full((2,), -1, dtype=torch.int64)}
        items.append((torch.full(s, -1.0), None, st))
    owners = lpt_partition([max(1, p.numel()) for p, _, _ in items], world)
    for i, ((p, _, st), o) in enumerate(zip(items, owners)):
        if o == rank:
            p.fill_(100 * i + 7)
            st["q"].fill_(i)
            st["metric"].fill_(0.5 * i)
            st["freqs"].fill_(rank)
    broadcast_whole(items, owners, world)
    torch.save({"owners": owners, "params": [p for p, _, _ in items], "q": [st["q"] for _, _, st in items],
                "metric": [st["metric"] for _, _, st in items], "freqs": [st["freqs"] for _, _, st in items]},
               os.path.join(outdir, f"wbcast_{rank}.pt"))
    dist.destroy_process_group()


def whole_plan_worker(rank, world, port, outdir):
    """RowShardedCRESSO5's split of a routed group on CPU ranks, with the kernel
    launches replaced by a recorder that 'steps' a tensor by writing a value into
    it: the row shards go to the exchanged step on every rank, each whole tensor
    is stepped on its owner only and reaches every rank through the exchange; a
    second call reuses the cached plan."""
    import cresso_b200.optim as optim
    from cresso_b200.distributed import RowShardedCRESSO5, mark_row_shard

    _init(rank, world, port, "gloo")
    calls = []

    def fake_run_routed(self, group, routed, spectral_devices, select=None, tag=None):
        kinds = []
        for kind, per in enumerate(routed):
            for d, its in per.items():
                for p, g, st in its:
                    kinds.append((kind, int(p.numel()), bool(getattr(p, "_cresso_shard", None))))
                    if not getattr(p, "_cresso_shard", None):
                        p.data.fill_(1000 + 10 * int(p.numel()) + kind)
                        st["q"].fill_(float(p.numel()))
        calls.append((tag, sorted(kinds)))

    optim.CRESSO5._run_routed = fake_run_routed
    cpu = torch.device("cpu")
    shard = mark_row_shard(torch.nn.Parameter(torch.zeros(4, 8)), (8, 8), 4 * rank)
    whole = [torch.nn.Parameter(torch.zeros(s)) for s in [(64, 16), (7, 9), (3, 4, 5), (30,), (16, 64)]]
    opt = RowShardedCRESSO5([shard] + whole, rank=8)
    states = {id(p): {"step": 1, "q": torch.zeros(())} for p in [shard] + whole}
    routed = ({cpu: [(shard, None, states[id(shard)]), (whole[2], None, states[id(whole[2])])]},
              {cpu: [(p, None, states[id(p)]) for p in (whole[0], whole[1], whole[4])]},
              {cpu: [(whole[3], None, states[id(whole[3])])]}, {})
    group = opt.param_groups[0]
    opt._run_routed(group, routed, set())
    n_plans = len(opt._whole_plans)
    opt._run_routed(group, routed, set())  # the cached plan
    owners = next(iter(opt._whole_plans.values()))[1][3]
    torch.save({"calls": calls, "owners": owners, "n_plans": n_plans, "n_plans2": len(opt._whole_plans),
                "whole": [p.detach().clone() for p in whole],
                "q": [states[id(p)]["q"].clone() for p in whole]},
               os.path.join(outdir, f"wplan_{rank}.pt"))
    dist.destroy_process_group()
