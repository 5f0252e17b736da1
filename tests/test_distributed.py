"""Multi-process host logic of the distributed optimizers on CPU ranks (gloo),
and the row-sharded CUDA step on 2 GPUs (NCCL) when the box has them."""

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from cresso_b200 import _lib
from cresso_b200.distributed import lpt_partition, row_block
from tests import _dist_workers as W


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn(fn, world, tmp_path):
    mp.spawn(fn, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)


@pytest.mark.parametrize("length,world", [(4096, 8), (11008, 8), (7, 3), (32000, 6), (1, 2)])
def test_row_blocks_tile_the_rows(length, world):
    blocks = [row_block(length, r, world) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == length
    for (a, b), (c, d) in zip(blocks, blocks[1:]):
        assert b == c
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1


def test_lpt_partition_is_balanced_and_deterministic():
    sizes = [32000 * 4096] * 2 + [4096 * 4096] * 128 + [11008 * 4096] * 96 + [4096] * 64
    owner = lpt_partition(sizes, 8)
    assert owner == lpt_partition(sizes, 8)
    load = np.zeros(8)
    for s, o in zip(sizes, owner):
        load[o] += s
    assert load.max() / load.mean() < 1.02


def test_device_failure_report_reaches_every_rank_gloo(tmp_path):
    spawn(W.status_exchange_worker, 2, tmp_path)
    rows = [(tmp_path / f"status_{r}.txt").read_text().splitlines() for r in range(2)]
    assert [int(r[0]) for r in rows] == [0, 1]  # only rank 1 saw the failure itself
    for r in rows:
        assert int(r[1]) == 1  # after the exchange every rank holds it
        assert "bounded wait" in r[2]  # and every rank's check raises


def test_zero_deferred_gather_finished_by_forward_hooks_gloo(tmp_path):
    spawn(W.zero_deferred_gather_worker, 2, tmp_path)
    for r in range(2):
        d = torch.load(tmp_path / f"zdefer_{r}.pt")
        for i, own in enumerate(d["owner"]):
            mine = own == r
            assert d["stale_before"][i] == (not mine)  # another rank's tensor waits for its gather
            first_layer = i < 2  # the weight and bias of model[0]
            assert d["after_first"][i] == (mine or first_layer)
            assert d["after_all"][i]


def test_row_sharded_stage_orchestration_gloo(tmp_path):
    spawn(W.stages_worker, 2, tmp_path)
    r0 = torch.load(tmp_path / "stages_0.pt")
    r1 = torch.load(tmp_path / "stages_1.pt")
    assert r0["calls"] == [(0, 3), (3, 6), (6, 9), (9, 12), (12, _lib.SPECTRAL_STAGES)]
    for k, (a, b) in enumerate(zip(r0["out"], r1["out"]), start=1):
        # each rank wrote (rank + 1) * k; the exchange sums them
        assert torch.equal(a, b)
        assert torch.all(a == 3.0 * k)


@pytest.mark.parametrize("bucketed", [False, True])
def test_zero_partition_gathers_owned_params_gloo(tmp_path, bucketed):
    spawn(W.zero_gather_bucketed_worker if bucketed else W.zero_gather_worker, 2, tmp_path)
    be = 20 if bucketed else 0
    r0 = torch.load(tmp_path / f"zero_0_{be}.pt")
    r1 = torch.load(tmp_path / f"zero_1_{be}.pt")
    assert set(r0["owner"]) == {0, 1}
    assert r0["plan"] == r1["plan"]  # every rank derives the same bucket plan
    assert (len(r0["plan"]) > 1) == bucketed
    for i, (a, b) in enumerate(zip(r0["vals"], r1["vals"])):
        assert torch.all(a == 100 * i + 7) and torch.equal(a, b)
    # each tensor is in exactly one bucket, under its owner
    seen = sorted(i for bucket in r0["plan"] for r, run in enumerate(bucket) for i in run
                  if r0["owner"][i] == r)
    assert seen == list(range(len(r0["vals"])))


def test_zero_consolidate_state_dict_gloo(tmp_path):
    spawn(W.zero_consolidate_worker, 2, tmp_path)
    r0 = torch.load(tmp_path / "consolidate_0.pt")
    r1 = torch.load(tmp_path / "consolidate_1.pt")
    assert r1["sd"] is None
    sd = r0["sd"]
    assert sorted(sd["state"].keys()) == list(range(5))  # every tensor, whichever rank owned it
    for i, st in sd["state"].items():
        assert st["step"] == 3 and float(st["force_rms"]) == float(i) and torch.all(st["q"] == 10 * i)
    assert set(r0["owner"]) == {0, 1}
    assert len(sd["param_groups"]) == 1 and sd["param_groups"][0]["params"] == list(range(5))


def test_failed_rank_surfaces_as_an_error_not_a_hang_gloo(tmp_path):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=W.failing_rank_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung instead of failing")
    s0 = (tmp_path / "fail_0.txt").read_text().splitlines()
    s1 = (tmp_path / "fail_1.txt").read_text().splitlines()
    assert "injected failure" in s1[0]
    assert s0[0] != "ok" and float(s0[1]) < 30.0


def test_whole_tensors_reach_every_rank_from_their_owners_gloo(tmp_path):
    spawn(W.whole_broadcast_worker, 2, tmp_path)
    r = [torch.load(tmp_path / f"wbcast_{k}.pt") for k in range(2)]
    assert r[0]["owners"] == r[1]["owners"] and set(r[0]["owners"]) == {0, 1}
    for k in range(2):
        for i, o in enumerate(r[k]["owners"]):
            assert torch.all(r[k]["params"][i] == 100 * i + 7)
            assert float(r[k]["q"][i]) == i
            assert r[k]["metric"][i].dtype == torch.float64 and torch.all(r[k]["metric"][i] == 0.5 * i)
            assert torch.all(r[k]["freqs"][i] == (k if o == k else -1))  # integer state is not sent


def test_row_sharded_split_and_whole_exchange_gloo(tmp_path):
    spawn(W.whole_plan_worker, 2, tmp_path)
    r = [torch.load(tmp_path / f"wplan_{k}.pt") for k in range(2)]
    assert r[0]["owners"] == r[1]["owners"] and set(r[0]["owners"]) == {0, 1}
    assert r[0]["n_plans"] == r[0]["n_plans2"] == 1  # the second call reused the plan
    for k in range(2):
        sharded = [c for c in r[k]["calls"] if c[0] is None]
        owned = [c for c in r[k]["calls"] if c[0] is not None]
        assert len(sharded) == 2 and all(c[1] == [(0, 32, True)] for c in sharded)  # the shard alone
        # this rank stepped exactly the whole tensors it owns (plan order: kinds 0, 1, 2)
        order = [(0, 60), (1, 1024), (1, 63), (1, 1024), (2, 30)]
        mine = sorted((kind, n, False) for (kind, n), o in zip(order, r[k]["owners"]) if o == k)
        assert all(c[1] == mine for c in owned), (owned, mine)
        # every rank ends with each owner's values
        kinds = {60: 0, 1024: 1, 63: 1, 30: 2}
        for p, q in zip(r[k]["whole"], r[k]["q"]):
            n = p.numel()
            assert torch.all(p == 1000 + 10 * n + kinds[n]) and float(q) == n


@pytest.mark.gpu
def test_row_sharded_step_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    spawn(W.gpu_row_shard_worker, 2, tmp_path)
    r = [torch.load(tmp_path / f"gpu_rs_{k}.pt") for k in range(2)]
    ref_params, ref_states = r[0]["ref"]
    for i, full in enumerate(ref_params[:r[0]["n_sharded"]]):
        got = torch.cat([r[0]["shard"][i], r[1]["shard"][i]])
        rel = float((got.double() - full.double()).pow(2).mean().sqrt() / full.double().pow(2).mean().sqrt())
        assert rel <= 1e-6, (i, rel)
        for k, v in ref_states[i].items():
            a, b = r[0]["states"][i][k], r[1]["states"][i][k]
            if torch.is_tensor(v):
                assert torch.equal(a, b), (i, k)  # every rank holds the same rank / hash state
                if v.dtype.is_floating_point:
                    d = float((a.double() - v.double()).abs().max())
                    assert d <= 1e-4 * max(float(v.double().abs().max()), 1e-6), (i, k, d)
            else:
                assert a == v == b
    # tensors passed whole: stepped by their owners (both ranks own some) and all-gathered
    assert set(r[0]["owners"]) == {0, 1}
    n = r[0]["n_sharded"]
    for i, (a, b) in enumerate(zip(r[0]["whole"], r[1]["whole"])):
        full = ref_params[n + i]
        assert torch.equal(a, b), i
        rel = float((a.double() - full.double()).pow(2).mean().sqrt() / full.double().pow(2).mean().sqrt())
        assert rel <= 1e-6, (i, rel)
        for k, v in ref_states[n + i].items():
            x, y = r[0]["whole_states"][i][k], r[1]["whole_states"][i][k]
            if torch.is_tensor(v):
                assert torch.equal(x, y), (i, k)
                if v.dtype.is_floating_point:
                    d = float((x.double() - v.double()).abs().max())
                    assert d <= 1e-4 * max(float(v.double().abs().max()), 1e-6), (i, k, d)
            else:
                assert x == v == y


@pytest.mark.gpu
def test_zero_bucketed_step_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    spawn(W.gpu_zero_worker, 2, tmp_path)
    r = [torch.load(tmp_path / f"gpu_zero_{k}.pt") for k in range(2)]
    assert r[0]["n_buckets"] > 1
    for i, full in enumerate(r[0]["ref"]):
        a, b = r[0]["params"][i], r[1]["params"][i]
        assert torch.equal(a, b), i  # every rank ends with the owner's values
        rel = float((a.double() - full.double()).pow(2).mean().sqrt() / full.double().pow(2).mean().sqrt())
        assert rel <= 1e-6, (i, rel)


@pytest.mark.gpu
def test_zero_deferred_gather_matches_in_step_gather(tmp_path):
    """ZeRO-1 all-gathers left in flight by the step and finished by forward
    pre-hooks of the next forward: three training steps of a small model give the
    same parameters, bit for bit, as gathers finished inside the step."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    spawn(W.gpu_zero_deferred_worker, 2, tmp_path)
    for k in range(2):
        r = torch.load(tmp_path / f"gpu_zdefer_{k}.pt")
        for a, b in zip(r["plain"], r["deferred"]):
            assert torch.equal(a, b)
