"""Multi-GPU CRESSO5: one process per GPU, ``torch.distributed`` over NCCL.

The reference is single-GPU (it has no collective anywhere).  Two ways of
spreading one optimizer step over the GPUs of a box are provided:

``RowShardedCRESSO5`` (row sharding)
    Every rank holds a contiguous row block of each large 2-D tensor and a
    contiguous element range of each large 1-D tensor (mark the local blocks
    with ``mark_row_shard`` / ``shard_rows``), i.e. the FSDP layout.  The fused
    step runs locally; between its passes the per-tensor partial sums (force
    energy; density / hash-bin / projection / column sums; error, projection
    and port-bin sums; the drive Gram) are SUM-all-reduced as one float64
    vector per pass, four small all-reduces per step for all tensors together.
    Every rank then holds identical rank / hash / scalar state, and updates its
    own rows.  Hash indices and carrier coordinates use global indices, so the
    result equals the single-GPU step up to the float64 summation order.
    Tensors passed whole (small and LoRA-thin scalar-route tensors, micro-field
    tensors, spectral tensors of rank >= 3, float64 or rank > 16 spectral
    tensors, and any tensor not marked as a shard) take no part in the
    exchange: each is stepped by one owner rank (a greedy partition on element
    counts) and its updated values and state reach the other ranks in one
    all-gather, so a LoRA-heavy set is split over the GPUs too.

``ZeroCRESSO5`` (ZeRO-1 partition)
    Whole tensors are assigned to ranks by a longest-processing-time greedy
    partition on element counts.  A rank steps only the tensors it owns (no
    collective during the step) and the updated tensors are then
    all-gathered, so every rank ends with the full updated parameters.  With
    ``bucket_elements`` the owned tensors go in buckets whose all-gather runs
    while the next bucket computes.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .optim import CRESSO5


def mark_row_shard(param: Tensor, global_shape: Sequence[int], offset: int) -> Tensor:
    """Declares `param` to be the block of a larger tensor of `global_shape`
    that starts at global row `offset` (2-D) or element `offset` (1-D)."""
    param._cresso_shard = (tuple(int(d) for d in global_shape), int(offset))
    return param


def row_block(length: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of rank's contiguous block of `length` rows, sizes differing by at most one."""
    base, extra = divmod(int(length), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(full: Tensor, rank: int, world: int) -> Tuple[Tensor, int]:
    """This rank's block of `full` (rows of a 2-D, elements of a 1-D tensor) and its offset."""
    start, stop = row_block(full.shape[0], rank, world)
    return full[start:stop].contiguous(), start


def lpt_partition(sizes: Sequence[int], world: int) -> List[int]:
    """Owner rank of each item: largest first onto the least-loaded rank
    (ties to the lowest rank), a deterministic greedy LPT schedule."""
    order = sorted(range(len(sizes)), key=lambda i: (-int(sizes[i]), i))
    load = [0] * int(world)
    owner = [0] * len(sizes)
    for i in order:
        r = min(range(int(world)), key=lambda j: (load[j], j))
        owner[i] = r
        load[r] += int(sizes[i])
    return owner


def exchange_status(opt: CRESSO5, group=None) -> None:
    """Spreads a device-side failure report of any rank to every rank: the failure
    words are MAX-all-reduced once per step (every rank takes this collective in
    every step, so it cannot unbalance the collective order) and the host copies
    re-queued, so all ranks raise together at a later step().  The words only
    take the values 0, 1 and 3 (bit 2 is only ever set with bit 1), so MAX is
    their union."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    if dist.get_backend(group) == "nccl":
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device("cpu")
    word = opt._status_word(device)
    dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group)
    opt._publish_status([device])


def _whole_segments(items: Sequence[tuple]) -> List[List[Tensor]]:
    """Per item the tensors an owner sends: the parameter, then its floating-point
    state tensors by key (integer state, the frequency pack, never changes)."""
    out = []
    for p, _, st in items:
        ts = [p.data]
        for k in sorted(st):
            v = st[k]
            if torch.is_tensor(v) and v.is_floating_point():
                ts.append(v)
        out.append(ts)
    return out


class WholeExchange:
    """The exchange of the tensors stepped whole under row sharding: after each
    owner stepped its tensors, every rank receives the owners' parameters and
    floating-point state.

    One byte layout per plan: rank r's tensors (parameter, then state by key)
    at 16-byte aligned offsets of an S-byte block, S the largest rank's total.
    Each step packs this rank's block, all-gathers the blocks (one collective)
    and unpacks the other ranks' blocks into the tensors.  On CUDA devices the
    packing and the unpacking are one launch each (``cresso_copy_segments``
    over device tables of (source, destination, bytes) rows built once); the
    tables hold device addresses, so the plan is rebuilt when the parameters or
    state tensors are replaced (``invalidate_caches``).  CPU tensors (gloo test
    ranks) take the same layout through tensor copies."""

    def __init__(self, items: Sequence[tuple], owners: Sequence[int], world: int, rank: int):
        self.world, self.rank = int(world), int(rank)
        segs = _whole_segments(items)
        per_rank: List[List[Tuple[Tensor, int, int]]] = [[] for _ in range(self.world)]  # (tensor, offset, bytes)
        used = [0] * self.world
        for ts, o in zip(segs, owners):
            for t in ts:
                nb = t.numel() * t.element_size()
                per_rank[o].append((t, used[o], nb))
                used[o] += (nb + 15) // 16 * 16
        self.block = max(max(used), 16)
        device = items[0][0].device
        if any(it[0].device != device for it in items):
            raise RuntimeError("RowShardedCRESSO5: the tensors stepped whole must all be on this rank's device")
        self.device = device
        self.send = torch.zeros(self.block, dtype=torch.uint8, device=device)
        self.recv = torch.zeros(self.world * self.block, dtype=torch.uint8, device=device)
        self.per_rank = per_rank
        if device.type == "cuda":
            sb, rb = self.send.data_ptr(), self.recv.data_ptr()
            pack = [(t.data_ptr(), sb + off, nb) for t, off, nb in per_rank[self.rank]]
            unpack = [(rb + r * self.block + off, t.data_ptr(), nb)
                      for r in range(self.world) if r != self.rank for t, off, nb in per_rank[r]]
            self.pack_table = self._table(pack, device)
            self.unpack_table = self._table(unpack, device)
            self.n_pack, self.n_unpack = len(pack), len(unpack)

    @staticmethod
    def _table(rows, device) -> Tensor:
        if not rows:
            return torch.zeros(3, dtype=torch.int64, device=device)
        return torch.tensor(rows, dtype=torch.int64).reshape(-1).to(device)

    def run(self, group=None) -> None:
        if self.device.type == "cuda":
            L = _lib.lib()
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _lib.check(L.cresso_copy_segments(_lib.ptr(self.pack_table), self.n_pack, stream), "copy_segments")
            dist.all_gather_into_tensor(self.recv, self.send, group=group)
            _lib.check(L.cresso_copy_segments(_lib.ptr(self.unpack_table), self.n_unpack, stream), "copy_segments")
            return
        for t, off, nb in self.per_rank[self.rank]:
            self.send[off:off + nb].copy_(t.reshape(-1).view(torch.uint8))
        dist.all_gather(list(self.recv.split(self.block)), self.send, group=group)
        for r in range(self.world):
            if r == self.rank:
                continue
            for t, off, nb in self.per_rank[r]:
                base = r * self.block + off
                t.reshape(-1).view(torch.uint8).copy_(self.recv[base:base + nb])


def broadcast_whole(items: Sequence[tuple], owners: Sequence[int], world: int, group=None) -> None:
    """One exchange of whole tensors (a WholeExchange built for this call)."""
    WholeExchange(items, owners, world, dist.get_rank(group)).run(group)


def _is_shard(param: Tensor) -> bool:
    return getattr(param, "_cresso_shard", None) is not None


class RowShardedCRESSO5(CRESSO5):
    """CRESSO5 over row-sharded tensors with one float64 all-reduce per pass.

    With ``pipeline_exchange`` (the default) a spectral group of two or more
    tensors is stepped as two halves of about equal size: each half's
    all-reduce runs (on NCCL's stream) while the other half computes its next
    pass, so the exchange between passes leaves the compute stream's critical
    path.  Every rank takes the same halves and collectives in the same order.

    Tensors passed whole are stepped without any exchange between passes.  With
    ``partition_whole`` (the default) each is stepped by one owner rank (LPT on
    element counts over the group's whole tensors, the same plan on every rank)
    and its values reach the other ranks in one all-gather (``WholeExchange``);
    without it every rank steps every whole tensor itself.  The plan is cached
    per group and keyed on the parameter objects; it holds the device addresses
    of the parameters and state tensors, so a caller that replaces a
    parameter's storage (``p.data = t``) or a state tensor calls
    ``invalidate_caches()`` afterwards (``load_state_dict`` does so itself)."""

    def __init__(self, params: Iterable[Tensor], process_group=None, pipeline_exchange: bool = True,
                 partition_whole: bool = True, **kwargs):
        super().__init__(params, **kwargs)
        self.process_group = process_group
        self.pipeline_exchange = bool(pipeline_exchange)
        self.partition_whole = bool(partition_whole)
        self._local = False  # set while whole tensors are stepped: their sums are complete per rank
        self._whole_plans: Dict[int, tuple] = {}  # id(group) -> (parameter ids, plan)

    def _run_routed(self, group: dict, routed, spectral_devices: set, select=None, tag=None) -> None:
        world = self._world()
        if world == 1 or select is not None:
            super()._run_routed(group, routed, spectral_devices, select, tag)
            return
        # the group's routed items in a fixed order; the plan (which items are row shards,
        # which whole ones this rank steps, the exchange) is keyed on the parameters
        flat = [(kind, d, it) for kind, per in enumerate(routed) for d, its in per.items() for it in its]
        ident = tuple(id(it[0]) for _, _, it in flat)
        cached = self._whole_plans.get(id(group))  # the group's last plan only
        if cached is None or cached[0] != ident:
            cached = self._whole_plans[id(group)] = (ident, self._plan_whole(flat, world))
        sharded_idx, whole_idx, mine_idx, owners, exchange = cached[1]

        def subset(idx):
            out: Tuple[Dict, ...] = ({}, {}, {}, {})
            for i in idx:
                kind, d, it = flat[i]
                out[kind].setdefault(d, []).append(it)
            return out

        if sharded_idx:  # the exchanged step of the row shards
            super()._run_routed(group, subset(sharded_idx), spectral_devices, None, tag)
        if not whole_idx:
            return
        self._local = True
        try:
            super()._run_routed(group, subset(mine_idx), spectral_devices, None, ("whole", tag))
        finally:
            self._local = False
        if exchange is not None:
            exchange.run(self.process_group)

    def _plan_whole(self, flat: list, world: int) -> tuple:
        """(row-shard positions, whole positions, positions this rank steps, owners,
        exchange) of a group's routed items."""
        sharded_idx = [i for i, (kind, _, it) in enumerate(flat) if kind == 0 and _is_shard(it[0])]
        whole_idx = [i for i, (kind, _, it) in enumerate(flat) if not (kind == 0 and _is_shard(it[0]))]
        if not whole_idx:
            return sharded_idx, whole_idx, [], [], None
        if not self.partition_whole:
            return sharded_idx, whole_idx, whole_idx, [], None
        me = dist.get_rank(self.process_group)
        items = [flat[i][2] for i in whole_idx]
        owners = lpt_partition([it[0].numel() for it in items], world)
        mine_idx = [i for i, o in zip(whole_idx, owners) if o == me]
        return sharded_idx, whole_idx, mine_idx, owners, WholeExchange(items, owners, world, me)

    def invalidate_caches(self) -> None:
        super().invalidate_caches()
        self._whole_plans.clear()

    def _run_spectral(self, group: dict, hp, device, items: list, tag=None) -> None:
        if self._local or not self.pipeline_exchange or self._world() == 1 or len(items) < 2:
            super()._run_spectral(group, hp, device, items, tag)
            return
        sizes = [p.numel() for p, _, _ in items]
        total, acc, cut = sum(sizes), 0, 1
        for i, n in enumerate(sizes[:-1]):
            acc += n
            cut = i + 1
            if 2 * acc >= total:
                break
        halves = [items[:cut], items[cut:]]
        setups = [self._spectral_setup(group, hp, device, h, (tag, i), "spectral" if i == 0 else "spectral_b")
                  for i, h in enumerate(halves)]
        bounds = (0,) + tuple(_lib.REDUCTION_BOUNDARIES) + (_lib.SPECTRAL_STAGES,)
        works = [None, None]
        for k in range(len(bounds) - 1):
            for i, (run, scratch, layout) in enumerate(setups):
                if works[i] is not None:
                    works[i].wait()  # the compute stream waits for this half's exchange
                run(bounds[k], bounds[k + 1])
                works[i] = None
                if k + 1 < len(bounds) - 1:
                    works[i] = dist.all_reduce(self._reduction_view(scratch, layout, k + 1), op=dist.ReduceOp.SUM,
                                               group=self.process_group, async_op=True)

    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        loss = super().step(closure)
        # a rank whose kernel gave up fed partial sums into the exchange, which spoils
        # every rank's state: every rank learns of it
        exchange_status(self, self.process_group)
        return loss

    def _world(self) -> int:
        if not dist.is_available() or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.process_group)

    def _spectral_stages(self, run, scratch: Tensor, layout) -> None:
        if self._local or self._world() == 1:
            run(0, _lib.SPECTRAL_STAGES)
            return
        begin = 0
        for k, end in enumerate(_lib.REDUCTION_BOUNDARIES, start=1):
            run(begin, end)
            dist.all_reduce(self._reduction_view(scratch, layout, k), op=dist.ReduceOp.SUM, group=self.process_group)
            begin = end
        run(begin, _lib.SPECTRAL_STAGES)


class ZeroCRESSO5(CRESSO5):
    """ZeRO-1 style CRESSO5: each rank steps the whole tensors it owns, then
    the updated parameters are all-gathered.

    With ``bucket_elements > 0`` the owned tensors of every rank are cut, in
    parameter order, into runs of at least that many elements; bucket k is the
    k-th run of every rank.  The step computes bucket k, starts its all-gather
    asynchronously (NCCL runs it on its own stream) and goes on with bucket
    k + 1, so the exchange of one bucket overlaps the compute of the next;
    the gathered values are copied into the parameters at the end of the step.
    Every rank derives the same plan from the shapes alone.

    With ``defer_gather=True`` the step only starts the all-gathers: each one is
    finished when a parameter it carries is first needed.  ``prefetch_forward
    (model)`` registers forward pre-hooks that finish, before a module runs, the
    all-gathers of the buckets holding its parameters, so the exchange of the
    later buckets runs under the first layers of the next forward.  Anything
    else that reads the parameters first calls ``wait_params()``; the next
    step() and gather_params() do so themselves."""

    def __init__(self, params: Iterable[Tensor], process_group=None, bucket_elements: int = 0,
                 defer_gather: bool = False, **kwargs):
        super().__init__(params, **kwargs)
        self.process_group = process_group
        self.defer_gather = bool(defer_gather)
        self._deferred: List[tuple] = []             # all-gathers started, not yet finished
        self._deferred_of: Dict[int, List[int]] = {}  # id(param) -> indices into _deferred
        self._hooks: list = []
        world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.world = world
        all_params = [p for g in self.param_groups for p in g["params"]]
        self.owner: Dict[Tensor, int] = {}
        for p, r in zip(all_params, lpt_partition([p.numel() for p in all_params], world)):
            self.owner[p] = r
        self.bucket_elements = int(bucket_elements)
        self.buckets = self._plan_buckets(all_params)

    def _plan_buckets(self, all_params: List[Tensor]) -> List[List[List[Tensor]]]:
        """buckets[k][r]: rank r's tensors of bucket k (possibly none)."""
        chunks = []
        for r in range(self.world):
            runs: List[List[Tensor]] = []
            cur: List[Tensor] = []
            n = 0
            for p in all_params:
                if self.owner[p] != r:
                    continue
                cur.append(p)
                n += p.numel()
                if self.bucket_elements > 0 and n >= self.bucket_elements:
                    runs.append(cur)
                    cur, n = [], 0
            if cur or not runs:
                runs.append(cur)
            chunks.append(runs)
        k_max = max(len(c) for c in chunks)
        return [[chunks[r][k] if k < len(chunks[r]) else [] for r in range(self.world)] for k in range(k_max)]

    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.check_device_status(block=False)
        # route once per step, with the gradients of the tensors other ranks own hidden (so
        # the routing cache of an unchanged step matches), then run each bucket's slice
        mine_all = {id(p) for bucket in self.buckets for p in bucket[self.rank]}
        hidden = [(p, p.grad) for g in self.param_groups for p in g["params"]
                  if id(p) not in mine_all and p.grad is not None]
        for p, _ in hidden:
            p.grad = None
        try:
            routed = [self._route_group(gi, group) for gi, group in enumerate(self.param_groups)]
        finally:
            for p, gr in hidden:
                p.grad = gr
        spectral_devices: set = set()
        self.wait_params()  # a deferred exchange of the previous step, if no forward finished it
        pending: list = []  # all-gathers of the previous bucket, still in flight
        for k, bucket in enumerate(self.buckets):
            mine = {id(p) for p in bucket[self.rank]}
            if mine:
                for group, r in zip(self.param_groups, routed):
                    self._run_routed(group, r, spectral_devices, select=mine, tag=("bucket", k))
            if self.world > 1:
                started = self._gather_bucket_async(bucket)
                if self.defer_gather:  # finished by the next forward (or wait_params)
                    self._defer(started)
                    continue
                # the previous bucket's exchange ran while this bucket computed; its
                # values go into the parameters now (at most two buckets in flight)
                for item in pending:
                    self._finish_gather(item)
                pending = started
        for item in pending:
            self._finish_gather(item)
        self._publish_status(spectral_devices)
        exchange_status(self, self.process_group)
        return loss

    def _gather_bucket_async(self, bucket: List[List[Tensor]]) -> list:
        """Starts the all-gathers of one bucket (one per dtype); returns their handles."""
        dtypes = []
        for ps in bucket:
            for p in ps:
                if p.dtype not in dtypes:
                    dtypes.append(p.dtype)
        out_items = []
        for dtype in dtypes:
            per_rank = [[p for p in ps if p.dtype == dtype] for ps in bucket]
            width = max(max(sum(p.numel() for p in ps) for ps in per_rank), 1)
            dev = next(p for ps in per_rank for p in ps).device
            local = torch.empty(width, dtype=dtype, device=dev)
            mine = per_rank[self.rank]
            n_mine = sum(p.numel() for p in mine)
            if mine:
                torch.cat([p.detach().reshape(-1) for p in mine], out=local[:n_mine])
            if n_mine < width:
                local[n_mine:].zero_()
            out = torch.empty(width * self.world, dtype=dtype, device=dev)
            if dist.get_backend(self.process_group) == "nccl":
                work = dist.all_gather_into_tensor(out, local, group=self.process_group, async_op=True)
            else:
                work = dist.all_gather(list(out.chunk(self.world)), local, group=self.process_group, async_op=True)
            out_items.append((per_rank, width, out, local, work))
        return out_items

    def _finish_gather(self, item) -> None:
        per_rank, width, out, _local, work = item
        work.wait()
        dsts, srcs = [], []
        for r, ps in enumerate(per_rank):
            if r == self.rank:
                continue
            off = r * width
            for p in ps:
                dsts.append(p.detach())
                srcs.append(out[off:off + p.numel()].view_as(p))
                off += p.numel()
        if dsts:
            torch._foreach_copy_(dsts, srcs)  # a few multi-tensor launches instead of one per tensor

    def _defer(self, items: list) -> None:
        for item in items:
            idx = len(self._deferred)
            self._deferred.append(item)
            for r, ps in enumerate(item[0]):
                if r == self.rank:
                    continue
                for p in ps:
                    self._deferred_of.setdefault(id(p), []).append(idx)

    def wait_params(self, params: Optional[Iterable[Tensor]] = None) -> None:
        """Finishes the deferred all-gathers carrying `params` (all of them by
        default), in the order they were started, and copies the gathered values
        into the parameters (stream-ordered: the current stream waits for NCCL,
        the host does not)."""
        if not self._deferred_of:
            return
        if params is None:
            wanted = range(len(self._deferred))
        else:
            wanted = sorted({i for p in params for i in self._deferred_of.get(id(p), ())})
        for i in wanted:
            item = self._deferred[i]
            if item is None:
                continue
            self._finish_gather(item)
            self._deferred[i] = None
        if all(item is None for item in self._deferred):
            self._deferred.clear()
            self._deferred_of.clear()

    def prefetch_forward(self, model: torch.nn.Module) -> None:
        """Registers on every submodule that directly owns parameters of this
        optimizer a forward pre-hook finishing the deferred all-gathers of those
        parameters (a no-op once they are finished)."""
        mine = {id(p) for g in self.param_groups for p in g["params"]}
        for module in model.modules():
            own = [p for p in module.parameters(recurse=False) if id(p) in mine]
            if own:
                self._hooks.append(module.register_forward_pre_hook(
                    lambda mod, args, own=own: self.wait_params(own)))

    def consolidate_state_dict(self, to: int = 0) -> Optional[dict]:
        """The optimizer state of all ranks (each holds the state of the tensors it
        owns) as one ``state_dict`` in the reference layout, on rank ``to``; the
        other ranks get None.  It loads into CRESSO5 (or the reference's
        optimizer) like a single-process state_dict."""
        sd = self.state_dict()
        if self.world == 1:
            return sd
        local = {k: {n: (v.detach().cpu() if torch.is_tensor(v) else v) for n, v in st.items()}
                 for k, st in sd["state"].items()}
        parts = [None] * self.world if self.rank == to else None
        dist.gather_object(local, parts, dst=to, group=self.process_group)
        if self.rank != to:
            return None
        merged: Dict[int, dict] = {}
        for part in parts:
            merged.update(part)
        return {"state": {k: merged[k] for k in sorted(merged)}, "param_groups": sd["param_groups"]}

    @torch.no_grad()
    def gather_params(self) -> None:
        """All-gathers every rank's owned parameters into all ranks, bucket by bucket."""
        self.wait_params()
        pending = []
        for bucket in self.buckets:
            pending.extend(self._gather_bucket_async(bucket))
        for item in pending:
            self._finish_gather(item)
