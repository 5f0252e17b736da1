"""Full-step parity of the CUDA path (reference test_cresso_v5_cuda_ops.py:64-211
widened): every golden case of tests/golden (outputs of the reference itself),
multi-step runs at the benchmark shapes against the oracle, determinism and
state_dict round trips.

Tolerances (stated per check):
* parameters: relative RMS of (p_cuda - p_ref) over RMS(p_ref) <= 1e-5, and of
  the accumulated update (p - p0) <= 2e-4 of its own RMS;
* every state tensor: relative RMS distance to a float64 run of the reference
  arithmetic <= 2x the float32 reference's own distance to it, plus 1e-5, and
  distance to the float32 reference <= 3x that plus 1e-5 (the reference is
  float32; some states, e.g. metric_cos, sit on cancelling projections and
  carry ~1e-5..1e-4 float32 noise);
* hash bins are integer work and bit-exact (tested in test_gpu_ops.py).
"""

import copy
import os

import numpy as np
import pytest
import torch

import cresso_b200
from oracle import cresso5_oracle as O
from tests._cases import ROOT, case_inputs, extra_case_inputs, extra_cases, golden_cases, rel_rms, ulp_distance

pytestmark = pytest.mark.gpu

CASES = golden_cases()


def run_cuda(shape, kw, init, grads):
    p = torch.nn.Parameter(init.clone().cuda())
    opt = cresso_b200.CRESSO5([p], cuda_ops="required", **kw)
    for g in grads:
        p.grad = g.clone().cuda()
        opt.step()
    torch.cuda.synchronize()
    return p.detach().cpu(), {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}, opt


def run_oracle(kw, init, grads, dtype=torch.float32, device="cpu"):
    p = torch.nn.Parameter(init.clone().to(device=device, dtype=dtype))
    opt = O.OracleCRESSO5([p], **kw)
    for g in grads:
        p.grad = g.clone().to(device=device, dtype=dtype)
        opt.step()
    return p.detach().cpu(), {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}


def check_against(name, init, p, st, p_ref, st_ref, p64, st64, upd_tol=2e-4):
    errs = {}
    errs["param"] = rel_rms(p, p_ref)
    errs["update"] = rel_rms(p - init, p_ref - init)
    assert errs["param"] <= 1e-5, (name, errs)
    assert errs["update"] <= upd_tol, (name, errs)
    for k, v in st_ref.items():
        if not torch.is_tensor(v):
            assert st[k] == v, (name, k)
            continue
        if v.dtype == torch.int64:
            assert torch.equal(st[k], v), (name, k)
            continue
        noise = rel_rms(st_ref[k].double(), st64[k].double())
        e32 = rel_rms(st[k].double(), v.double())
        e64 = rel_rms(st[k].double(), st64[k].double())
        errs[k] = (e32, e64, noise)
        # at least as close to the float64 truth as twice the float32 reference's own error,
        # and therefore within 3x that error of the float32 reference
        assert e64 <= 2.0 * noise + 1e-5, (name, k, e64, noise)
        assert e32 <= 3.0 * noise + 1e-5, (name, k, e32, noise)
    print(name, {k: (tuple(round(x, 9) for x in v) if isinstance(v, tuple) else round(v, 9)) for k, v in errs.items()})
    return errs


@pytest.mark.parametrize("name", list(CASES.keys()))
def test_golden_case_parity(golden, name):
    shape, kw, steps, seed, istd, gstd = CASES[name]
    init, grads = case_inputs(golden, name, shape, steps, seed, istd, gstd)
    p, st, opt = run_cuda(shape, kw, init, grads)
    p_ref = torch.from_numpy(golden[f"step_{name}_final"])
    st_ref = {k[len(f"step_{name}_state_"):]: golden[k] for k in golden if k.startswith(f"step_{name}_state_")
              and k != f"step_{name}_state_elements"}
    st_ref = {k: (torch.from_numpy(v) if v.ndim > 0 or v.dtype.kind == "f" else int(v)) for k, v in st_ref.items()}
    p64, st64 = run_oracle(kw, init, grads, torch.float64)
    check_against(name, init, p, st, p_ref, st_ref, p64, st64)
    assert set(st.keys()) == set(st_ref.keys())
    assert cresso_b200.count_optimizer_state_elements(opt) == int(golden[f"step_{name}_state_elements"])


EXTRA_CASES = extra_cases()


@pytest.mark.parametrize("name", list(EXTRA_CASES.keys()))
def test_extra_golden_parity(golden_extra, name):
    """The second golden table against the reference's own output: float16 /
    bfloat16 parameters (spectral and scalar routes), spectral tensors of
    rank 3 to 5 (leading axes flattened into rows, carriers and the instant
    metric composed over every axis), the micro-field route, float64
    parameters (every route, float64 work and state) and mode ranks 17 to 200
    (the float64-arithmetic pipeline; above 64 with its modes in memory).

    float32 parameters: the criterion of the float32 golden cases.  16-bit
    parameters: every element within one unit in the last place of the
    parameter type per step (at the tensor's scale; a difference feeds the
    next step's force through weight decay) and a mean distance of at most
    0.15 of that unit: the update is rounded to the parameter type before the
    add and the sum rounded again, so a float32-level difference in an update
    (the drive mixes terms that partly cancel) can move a rounding by one
    unit; the reference's own 16-bit tests allow 3e-3 (float16) and 3e-2
    (bfloat16) absolute on parameters of scale 0.05.  States (float32): the
    criterion of the float32 tests, against a float64 run from the same
    inputs."""
    shape, kw, steps, seed, istd, gstd, dt = EXTRA_CASES[name]
    init, grads = extra_case_inputs(golden_extra, name, shape, steps, seed, istd, gstd, dt)
    p = torch.nn.Parameter(init.clone().cuda())
    opt = cresso_b200.CRESSO5([p], cuda_ops="required", **kw)
    for g in grads:
        p.grad = g.clone().cuda()
        opt.step()
    torch.cuda.synchronize()
    assert p.dtype == getattr(torch, dt)
    assert opt._device_status() == 0
    ref = golden_extra[f"step_{name}_final"]
    p64, st64 = run_oracle(kw, init.float(), [g.float() for g in grads], torch.float64)
    st_ref = {k[len(f"step_{name}_state_"):]: golden_extra[k] for k in golden_extra
              if k.startswith(f"step_{name}_state_") and k != f"step_{name}_state_elements"}
    assert set(opt.state[p].keys()) == set(st_ref.keys())
    assert cresso_b200.count_optimizer_state_elements(opt) == int(golden_extra[f"step_{name}_state_elements"])
    if dt == "float64":
        # float64 work and state: every value within 1e-9 relative RMS of the reference's
        # (float32 arithmetic would be ~1e-7 off); the update within 1e-8 of its own size
        got = p.detach().cpu().numpy()
        init64 = init.double().numpy()
        assert rel_rms(got, ref) <= 1e-12, name
        assert rel_rms(got - init64, ref - init64) <= 1e-8, (name, rel_rms(got - init64, ref - init64))
        for k, v in opt.state[p].items():
            if not torch.is_tensor(v):
                assert v == int(st_ref[k]), (name, k)
                continue
            if v.dtype == torch.int64:
                assert np.array_equal(v.cpu().numpy(), st_ref[k]), (name, k)
                continue
            assert v.dtype == torch.float64, (name, k)
            assert rel_rms(v.cpu().numpy(), st_ref[k]) <= 1e-9, (name, k, rel_rms(v.cpu().numpy(), st_ref[k]))
        return
    if dt == "float32":
        st_ref = {k: (torch.from_numpy(v) if v.ndim > 0 or v.dtype.kind == "f" else int(v)) for k, v in st_ref.items()}
        st = {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
        check_against(name, init, p.detach().cpu(), st, torch.from_numpy(ref), st_ref, p64, st64)
        return
    got = p.detach().float().cpu().numpy()
    ulps = ulp_distance(got, ref, dt)
    assert ulps.max() <= steps, (name, float(ulps.max()))  # at most one unit per step
    assert float(np.mean(ulps)) <= 0.15, (name, float(np.mean(ulps)), float(np.mean(ulps > 0)))
    for k, v in opt.state[p].items():
        ref_v = st_ref[k]
        if not torch.is_tensor(v):
            assert v == int(ref_v), (name, k)
            continue
        if v.dtype == torch.int64:
            assert np.array_equal(v.cpu().numpy(), ref_v), (name, k)
            continue
        assert v.dtype == torch.float32, (name, k)
        noise = rel_rms(ref_v, st64[k].double().numpy())
        e32 = rel_rms(v.double().cpu().numpy(), ref_v)
        e64 = rel_rms(v.double().cpu().numpy(), st64[k].double().numpy())
        assert e64 <= 2.0 * noise + 1e-5, (name, k, e64, noise)
        assert e32 <= 3.0 * noise + 1e-5, (name, k, e32, noise)


def _bench_inputs(cfg, steps):
    g = torch.Generator().manual_seed(0)
    if cfg == "c1":
        shapes = [(2048, 2048)]
        kw = dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2)
        istd = 0.02
    elif cfg == "c2":
        shapes = [(4096, 4096)]
        kw = dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2)
        istd = 0.02
    else:  # c3: 64 LoRA-like thin params; c4: 840 of them, c4s: the same on the spectral route
        n = 64 if cfg == "c3" else 840
        shapes = [(4096, 16) if i % 2 == 0 else (16, 4096) for i in range(n)]
        kw = dict(lr=2e-3, rank=4, hash_bins=64, hash_tables=2)
        if cfg == "c4s":
            kw["thin_matrix_route"] = "spectral"
        istd = 0.01
    inits = [torch.randn(s, generator=g) * istd for s in shapes]
    row_scale = None
    if cfg == "c2":
        row_scale = torch.exp(0.5 * torch.randn((4096, 1), generator=torch.Generator().manual_seed(7)))
    grads = []
    for step in range(steps):
        gg = torch.Generator().manual_seed(1000 + step)
        gs = []
        for s in shapes:
            x = torch.randn(s, generator=gg) * 1e-3
            if row_scale is not None:
                x = x * row_scale
            gs.append(x)
        grads.append(gs)
    return shapes, kw, inits, grads


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c4", "c4s"])
def test_benchmark_config_ten_steps(cfg):
    """BASELINE configs c1-c4 at full size for ten steps against the float32 and
    float64 oracle run by torch on the same GPU; every tensor of the group is
    checked (c3: 64 LoRA-thin tensors in one grouped launch; c4: 840 of them on
    the scalar route, c4s: the same 840 on thin_matrix_route="spectral")."""
    steps = 10
    shapes, kw, inits, grads = _bench_inputs(cfg, steps)
    dev = torch.device("cuda")
    ps = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
    opt = cresso_b200.CRESSO5(ps, cuda_ops="required", **kw)
    refs32 = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
    ref32 = O.OracleCRESSO5(refs32, **kw)
    refs64 = [torch.nn.Parameter(x.clone().to(dev, torch.float64)) for x in inits]
    ref64 = O.OracleCRESSO5(refs64, **kw)
    for gs in grads:
        for p, r, r64, g in zip(ps, refs32, refs64, gs):
            g = g.to(dev)
            p.grad = g.clone()
            r.grad = g.clone()
            r64.grad = g.double()
        opt.step()
        ref32.step()
        ref64.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0  # no bounded in-kernel wait gave up
    if len(ps) == 1:
        st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[ps[0]].items()}
        st32 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref32.state[refs32[0]].items()}
        st64 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref64.state[refs64[0]].items()}
        check_against(cfg, inits[0], ps[0].detach().cpu(), st, refs32[0].detach().cpu(), st32,
                      refs64[0].detach().cpu(), st64, upd_tol=5e-4)
        return
    check_group(cfg, inits, [p.detach().cpu() for p in ps], [opt.state[p] for p in ps],
                [r.detach().cpu() for r in refs32], [ref32.state[r] for r in refs32],
                [ref64.state[r] for r in refs64])


def check_group(name, inits, ps, states, rs, states32, states64, upd_tol=5e-4):
    """The criterion of check_against for a group of many small tensors.
    Parameters and updates per tensor.  A state of a small tensor is a handful of
    float32 scalars, whose distance to the float64 run is one noisy sample each,
    so each state key is checked over the whole group (its values of every tensor
    as one vector, the way a large tensor's state vector is checked): at least as
    close to the float64 truth as twice the float32 reference, plus 1e-5; and
    every single tensor's state within 2x + 1e-3 (a component whose true value
    is zero, such as a zero-frequency mode of a momentum, carries an absolute
    float32 error of ~1e-8 that is large relative to a small state vector; a
    mis-routed or mis-computed tensor is far outside either bound)."""
    for i, (x0, p, r) in enumerate(zip(inits, ps, rs)):
        assert rel_rms(p, r) <= 1e-5, (name, i, rel_rms(p, r))
        assert rel_rms(p - x0, r - x0) <= upd_tol, (name, i, rel_rms(p - x0, r - x0))
    cat = lambda sts, k: torch.cat([st[k].detach().reshape(-1).cpu().double() for st in sts])  # noqa: E731
    for k, v in states32[0].items():
        if not torch.is_tensor(v):
            assert all(st[k] == st32[k] for st, st32 in zip(states, states32)), (name, k)
            continue
        if v.dtype == torch.int64:
            assert all(torch.equal(st[k].cpu(), st32[k].cpu()) for st, st32 in zip(states, states32)), (name, k)
            continue
        got, ref, truth = cat(states, k), cat(states32, k), cat(states64, k)
        noise, e32, e64 = rel_rms(ref, truth), rel_rms(got, ref), rel_rms(got, truth)
        assert e64 <= 2.0 * noise + 1e-5, (name, k, e64, noise)
        assert e32 <= 3.0 * noise + 1e-5, (name, k, e32, noise)
        for i, (st, st32, st64) in enumerate(zip(states, states32, states64)):
            a, b, c = (x[k].detach().cpu().double() for x in (st, st32, st64))
            assert rel_rms(a, c) <= 2.0 * rel_rms(b, c) + 1e-3, (name, i, k, rel_rms(a, c), rel_rms(b, c))
        print(name, k, {"e32": e32, "e64": e64, "noise": noise})


def test_c5_shapes_full_size_parity():
    """The four distinct tensor shapes of the 7B-shaped benchmark set (c5) at
    full size in one group -- (32000, 4096), (11008, 4096), (4096, 11008),
    (4096,) -- ten steps (the step count of every BASELINE config) against the
    float32 and float64 oracle run by torch on the same GPU, with the criterion
    of the golden cases."""
    shapes = [(32000, 4096), (11008, 4096), (4096, 11008), (4096,)]
    kw = dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(5)
    inits = [torch.randn(s, generator=g, device=dev) * 0.02 for s in shapes]
    grads = [[torch.randn(s, generator=g, device=dev) * 1e-3 for s in shapes] for _ in range(10)]
    ps = [torch.nn.Parameter(x.clone()) for x in inits]
    opt = cresso_b200.CRESSO5(ps, **kw)
    for gs in grads:
        for p, gg in zip(ps, gs):
            p.grad = gg.clone()
        opt.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0
    for i, (p, x0) in enumerate(zip(ps, inits)):
        r = torch.nn.Parameter(x0.clone())
        r64 = torch.nn.Parameter(x0.double())
        ref32, ref64 = O.OracleCRESSO5([r], **kw), O.OracleCRESSO5([r64], **kw)
        for gs in grads:
            r.grad = gs[i].clone()
            r64.grad = gs[i].double()
            ref32.step()
            ref64.step()
        st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
        st32 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref32.state[r].items()}
        st64 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref64.state[r64].items()}
        check_against(f"c5{shapes[i]}", x0.cpu(), p.detach().cpu(), st, r.detach().cpu(), st32, r64.detach().cpu(),
                      st64, upd_tol=5e-4)
        del r, r64, ref32, ref64
        torch.cuda.empty_cache()


# Hyper-parameter variants on a shape that takes the tensor-core (tcgen05) form
# of P3-P5: 2-D, full 256-column tiles, 16-row items (the planner picks them for
# >= ~38k row-tiles of work), rank padded to 8, <= 256 bins.
TCR_VARIANTS = {
    "wd_maximize": dict(weight_decay=0.01, maximize=True),
    "no_echo_no_hash": dict(echo_mix=0.0, hash_bins=0),
    "local_ipow_ep": dict(local_sharpness=0.5, instant_metric_power=0.7, energy_power=1.5),
    "rank5_bins256": dict(rank=5, hash_bins=256, hash_tables=1),
}


@pytest.mark.parametrize("variant", list(TCR_VARIANTS.keys()))
def test_tensor_core_path_variants(variant):
    steps = 3
    shape = (8192, 2048)
    kw = dict(lr=2e-3, rank=8, max_frequency=5, hash_bins=64, hash_tables=2)
    kw.update(TCR_VARIANTS[variant])
    g = torch.Generator().manual_seed(11)
    init = torch.randn(shape, generator=g) * 0.02
    grads = [torch.randn(shape, generator=g) * 1e-3 for _ in range(steps)]
    dev = torch.device("cuda")
    p = torch.nn.Parameter(init.clone().to(dev))
    opt = cresso_b200.CRESSO5([p], cuda_ops="required", **kw)
    r32 = torch.nn.Parameter(init.clone().to(dev))
    ref32 = O.OracleCRESSO5([r32], **kw)
    r64 = torch.nn.Parameter(init.clone().to(dev, torch.float64))
    ref64 = O.OracleCRESSO5([r64], **kw)
    for gr in grads:
        p.grad = gr.to(dev)
        r32.grad = gr.to(dev)
        r64.grad = gr.to(dev, torch.float64)
        opt.step()
        ref32.step()
        ref64.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0
    st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
    st32 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref32.state[r32].items()}
    st64 = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in ref64.state[r64].items()}
    check_against(f"tcr[{variant}]", init, p.detach().cpu(), st, r32.detach().cpu(), st32, r64.detach().cpu(), st64,
                  upd_tol=5e-4)


SCALAR_VARIANTS = {
    "defaults": dict(),
    "wd_maximize_local": dict(weight_decay=0.01, maximize=True, local_sharpness=0.5),
    "power_no_instant": dict(instant_metric_power=0.7, energy_power=1.5, instant_metric_coupling=0.0),
}


@pytest.mark.parametrize("variant", list(SCALAR_VARIANTS.keys()))
def test_scalar_route_cluster_shapes(variant):
    """Scalar-route group mixing the cluster form (ragged row slices, an odd-width
    wide tensor, 1-D, 0-d) with tensors it does not hold (a thin tensor too long
    for one cluster, a 3-D tensor), which take the one-block-per-tensor kernel."""
    steps = 3
    shapes = [(4099, 16), (16, 4097), (32000, 16), (300,), (), (4, 5, 6), (24, 40)]
    kw = dict(lr=2e-3, rank=4, hash_bins=64, hash_tables=2)
    kw.update(SCALAR_VARIANTS[variant])
    g = torch.Generator().manual_seed(21)
    inits = [torch.randn(s, generator=g) * 0.01 for s in shapes]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s in shapes] for _ in range(steps)]
    dev = torch.device("cuda")
    ps = [torch.nn.Parameter(x.clone().to(dev)) for x in inits]
    opt = cresso_b200.CRESSO5(ps, cuda_ops="required", **kw)
    r32 = [torch.nn.Parameter(x.clone()) for x in inits]
    ref32 = O.OracleCRESSO5(r32, **kw)
    r64 = [torch.nn.Parameter(x.clone().double()) for x in inits]
    ref64 = O.OracleCRESSO5(r64, **kw)
    for gs in grads:
        for p, a, b, gr in zip(ps, r32, r64, gs):
            p.grad = gr.to(dev)
            a.grad = gr.clone()
            b.grad = gr.double()
        opt.step()
        ref32.step()
        ref64.step()
    torch.cuda.synchronize()
    for i, (p, a, b, x0) in enumerate(zip(ps, r32, r64, inits)):
        assert "q" in opt.state[p] and "freqs" not in opt.state[p]  # scalar route
        st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
        st32 = {k: (v if torch.is_tensor(v) else v) for k, v in ref32.state[a].items()}
        st64 = {k: (v if torch.is_tensor(v) else v) for k, v in ref64.state[b].items()}
        check_against(f"scalar[{variant}][{shapes[i]}]", x0, p.detach().cpu(), st, a.detach(), st32, b.detach(), st64,
                      upd_tol=5e-4)


@pytest.mark.parametrize("case", ["c1", "f64", "r96"])
def test_run_to_run_deterministic(case):
    """The same inputs give bit-identical parameters and state in two runs: the
    fused float32 path (c1), the float64 pipeline and its wide-rank form, whose
    hash-bin sums are exact integer sums inside a block and fixed-order float64
    sums across blocks."""
    if case == "c1":
        shapes, kw, inits, grads = _bench_inputs("c1", 3)
        init, gl, dt = inits[0], [gs[0] for gs in grads], torch.float32
    else:
        g = torch.Generator().manual_seed(11)
        shape = (192, 160) if case == "f64" else (96, 80)
        kw = dict(rank=8 if case == "f64" else 96, hash_bins=64, hash_tables=2, min_spectral_size=1024)
        dt = torch.float64 if case == "f64" else torch.float32
        init = torch.randn(shape, generator=g) * 0.02
        gl = [torch.randn(shape, generator=g) * 1e-3 for _ in range(3)]
    outs = []
    for _ in range(2):
        p = torch.nn.Parameter(init.clone().to("cuda", dt))
        opt = cresso_b200.CRESSO5([p], **kw)
        for gg in gl:
            p.grad = gg.to("cuda", dt)
            opt.step()
        outs.append((p.detach().cpu(), {k: v.cpu() for k, v in opt.state[p].items() if torch.is_tensor(v)}))
    assert "hash_energy" in outs[0][1]
    assert torch.equal(outs[0][0], outs[1][0])
    for k in outs[0][1]:
        assert torch.equal(outs[0][1][k], outs[1][1][k]), k


def test_state_dict_round_trip_with_oracle_layout():
    """A CUDA state_dict loads into the oracle (reference layout) and the two
    continue in step; and back."""
    shapes, kw, inits, grads = _bench_inputs("c1", 4)
    x0 = inits[0][:256, :256].contiguous()
    gs = [g[0][:256, :256].contiguous() for g in grads]
    p = torch.nn.Parameter(x0.clone().cuda())
    opt = cresso_b200.CRESSO5([p], **kw)
    for g in gs[:2]:
        p.grad = g.cuda()
        opt.step()
    sd = opt.state_dict()
    assert set(sd["state"][0].keys()) >= {"step", "freqs", "omega", "q_cos", "hash_energy", "force_rms"}
    # a fresh CUDA optimizer continues identically after load_state_dict
    p2 = torch.nn.Parameter(p.detach().clone())
    opt2 = cresso_b200.CRESSO5([p2], **kw)
    opt2.load_state_dict(copy.deepcopy(sd))  # torch's load_state_dict keeps the tensors it is given
    for g in gs[2:]:
        p.grad = g.cuda()
        p2.grad = g.cuda()
        opt.step()
        opt2.step()
    assert torch.equal(p.detach(), p2.detach())
    # the oracle accepts the same state (reference keys / shapes / dtypes) and continues close by
    pr = torch.nn.Parameter(p.detach().clone().cpu())
    ref = O.OracleCRESSO5([pr], **kw)
    ref.state[pr] = {k: (v.detach().cpu().clone() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
    g = torch.randn((256, 256), generator=torch.Generator().manual_seed(5)) * 1e-3
    p.grad = g.cuda()
    pr.grad = g.clone()
    opt.step()
    ref.step()
    assert rel_rms(p.detach().cpu(), pr.detach()) <= 1e-5


@pytest.mark.parametrize("micro", [0, 4096])
def test_mixed_routes_in_one_group(micro):
    """Spectral 2-D / 1-D / 3-D, LoRA-thin and small tensors in one param group;
    with micro_field_max_size = 4096 the tensors of 1 to 4096 elements and
    rank >= 1 take the micro-field route instead."""
    g = torch.Generator().manual_seed(1)
    shapes = [(300, 200), (4096,), (512, 16), (16, 512), (7, 9), (100,), (), (3, 4, 5), (24, 10, 12)]
    inits = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s in shapes] for _ in range(3)]
    kw = dict(rank=8, hash_bins=64, hash_tables=2, micro_field_max_size=micro)
    ps = [torch.nn.Parameter(x.clone().cuda()) for x in inits]
    rs = [torch.nn.Parameter(x.clone()) for x in inits]
    r64s = [torch.nn.Parameter(x.clone().double()) for x in inits]
    opt = cresso_b200.CRESSO5(ps, **kw)
    ref = O.OracleCRESSO5(rs, **kw)
    ref64 = O.OracleCRESSO5(r64s, **kw)
    for gs in grads:
        for p, r, r64, gg in zip(ps, rs, r64s, gs):
            p.grad = gg.cuda()
            r.grad = gg.clone()
            r64.grad = gg.double()
        opt.step()
        ref.step()
        ref64.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0
    for p, r, r64, s, x0 in zip(ps, rs, r64s, shapes, inits):
        assert set(opt.state[p].keys()) == set(ref.state[r].keys()), s
        st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
        # the criterion of every other case: parameters and update, and each state tensor
        # against the float64 run within twice the float32 reference's own distance to it
        check_against(f"mixed{s}", x0, p.detach().cpu(), st, r.detach(), ref.state[r], r64.detach(),
                      ref64.state[r64], upd_tol=5e-4)


def test_float64_spectral_route_in_a_mixed_group():
    """float64 tensors of every route in one group next to float32 ones: the
    float64 spectral tensors run the float64 pipeline (float64 state), and the
    whole group matches the oracle run in float64 / float32."""
    g = torch.Generator().manual_seed(8)
    specs = [((96, 64), torch.float64), ((3000,), torch.float64), ((9, 7), torch.float64), ((96, 64), torch.float32),
             ((4, 6, 50), torch.float64)]
    inits = [torch.randn(s, generator=g) * 0.02 for s, _ in specs]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s, _ in specs] for _ in range(3)]
    kw = dict(rank=8, hash_bins=64, hash_tables=2)
    ps = [torch.nn.Parameter(x.clone().to("cuda", dt)) for x, (_, dt) in zip(inits, specs)]
    rs = [torch.nn.Parameter(x.clone().to(dt)) for x, (_, dt) in zip(inits, specs)]
    r64s = [torch.nn.Parameter(x.clone().double()) for x in inits]  # float64 truth of the float32 tensors
    opt = cresso_b200.CRESSO5(ps, **kw)
    ref = O.OracleCRESSO5(rs, **kw)
    ref64 = O.OracleCRESSO5(r64s, **kw)
    for gs in grads:
        for p, r, r64, gg in zip(ps, rs, r64s, gs):
            p.grad = gg.to("cuda", p.dtype)
            r.grad = gg.to(r.dtype)
            r64.grad = gg.double()
        opt.step()
        ref.step()
        ref64.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0
    for (shape, dt), p, r, r64, x0 in zip(specs, ps, rs, r64s, inits):
        for k, v in ref.state[r].items():
            if torch.is_tensor(v) and v.dtype.is_floating_point:
                assert opt.state[p][k].dtype == v.dtype, (shape, k)
        if dt == torch.float64:
            assert rel_rms(p.detach().cpu().double(), r.detach().double()) <= 1e-12, shape
            for k, v in ref.state[r].items():
                if torch.is_tensor(v) and v.dtype.is_floating_point:
                    assert rel_rms(opt.state[p][k].cpu().double(), v.double()) <= 1e-9, (shape, k)
        else:  # float32 tensors: the criterion of every float32 case
            st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
            check_against(f"f64group{shape}", x0, p.detach().cpu(), st, r.detach(), ref.state[r], r64.detach(),
                          ref64.state[r64], upd_tol=5e-4)


def test_bin_values_beyond_the_fixed_point_range():
    """Hash-bin sums take fixed-point shared-memory atomics for values below a
    bound and float atomics for the rest (outlier gradients): a class-0 tensor
    (full 256-column tiles, the lean kernels) with planted outliers 1000x the
    gradient scale, whose P2 densities and P3 ports exceed the fixed-point range,
    against the oracle."""
    g = torch.Generator().manual_seed(77)
    shape = (512, 1024)
    init = torch.randn(shape, generator=g) * 0.02
    grads = []
    for _ in range(3):
        x = torch.randn(shape, generator=g) * 1e-3
        idx = torch.randint(0, x.numel(), (64,), generator=g)
        x.view(-1)[idx] = torch.sign(torch.randn(64, generator=g)) * 1.0
        grads.append(x)
    kw = dict(rank=8, hash_bins=64, hash_tables=2)
    p, st, opt = run_cuda(shape, kw, init, grads)
    assert opt._device_status() == 0
    p_ref, st_ref = run_oracle(kw, init, grads)
    p64, st64 = run_oracle(kw, init, grads, torch.float64)
    check_against("outliers", init, p, st, p_ref, st_ref, p64, st64)


def test_float64_pipeline_groups_of_many_tensors():
    """Rank 24 in one group: 30 float64 tensors and float32 / float16 / bfloat16
    ones interleaved (the float64-arithmetic pipeline launches consecutive
    tensors of one state type as one group, so this runs many groups of one to
    several tensors), with shapes from 1-D to 3-D and hashed and hash-less
    (non-hard) tensors, against the oracle."""
    g = torch.Generator().manual_seed(24)
    specs = []
    for i in range(30):
        shape = [(40, 33), (700,), (5, 6, 21), (3, 200), (64, 64)][i % 5]
        specs.append((shape, torch.float64))
        if i % 6 == 2:
            specs.append(((48, 40), torch.float32))
        if i % 6 == 4:
            specs.append(((30, 50), [torch.bfloat16, torch.float16][i % 4 // 2]))
    inits = [torch.randn(s, generator=g) * 0.02 for s, _ in specs]
    grads = [[torch.randn(s, generator=g) * 1e-3 for s, _ in specs] for _ in range(3)]
    kw = dict(rank=24, hash_bins=64, hash_tables=2, hard_channel_min_size=1500, min_spectral_size=1,
              thin_matrix_route="spectral")
    ps = [torch.nn.Parameter(x.clone().to("cuda", dt)) for x, (_, dt) in zip(inits, specs)]
    rs = [torch.nn.Parameter(x.clone().to(dt)) for x, (_, dt) in zip(inits, specs)]
    r64s = [torch.nn.Parameter(x.clone().to(dt).double()) for x, (_, dt) in zip(inits, specs)]
    opt = cresso_b200.CRESSO5(ps, **kw)
    ref = O.OracleCRESSO5(rs, **kw)
    ref64 = O.OracleCRESSO5(r64s, **kw)
    for gs in grads:
        for p, r, r64, gg, (_, dt) in zip(ps, rs, r64s, gs, specs):
            p.grad = gg.to("cuda", dt)
            r.grad = gg.to(dt)
            r64.grad = gg.to(dt).double()
        opt.step()
        ref.step()
        ref64.step()
    torch.cuda.synchronize()
    assert opt._device_status() == 0
    for (shape, dt), p, r, r64, x0 in zip(specs, ps, rs, r64s, inits):
        assert p.dtype == dt
        if dt == torch.float64:
            assert rel_rms(p.detach().cpu().double(), r.detach().double()) <= 1e-12, shape
            for k, v in ref.state[r].items():
                if torch.is_tensor(v) and v.dtype.is_floating_point:
                    assert opt.state[p][k].dtype == torch.float64, (shape, k)
                    assert rel_rms(opt.state[p][k].cpu().double(), v.double()) <= 1e-9, (shape, k)
        elif dt == torch.float32:
            st = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
            check_against(f"r24group{shape}", x0, p.detach().cpu(), st, r.detach(), ref.state[r], r64.detach(),
                          ref64.state[r64], upd_tol=5e-4)
        else:  # 16-bit: within one unit of the parameter type per step, mostly exact
            ulps = ulp_distance(p.detach().float().cpu().numpy(), r.detach().float().numpy(),
                                str(dt).split(".")[-1])
            assert ulps.max() <= 3 and float(np.mean(ulps)) <= 0.15, (shape, dt, float(ulps.max()))
            for k, v in ref64.state[r64].items():
                if torch.is_tensor(v) and v.dtype.is_floating_point:
                    assert opt.state[p][k].dtype == torch.float32, (shape, k)


def test_bounded_wait_runs_out_and_reports_status():
    """The bounded in-kernel wait that guards the tensor-core passes, on a GPU:
    an mbarrier nothing arrives on makes the wait give up after its limit and
    report status 1; with the arrival it reports 0; the context stays usable."""
    from cresso_b200 import _lib, ops
    L = _lib.lib()
    st = torch.full((2,), 7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _lib.check(L.cresso_selftest_bounded_wait(2_000_000, 0, st[0:1].data_ptr(), stream), "selftest")
    e1.record()
    _lib.check(L.cresso_selftest_bounded_wait(2_000_000, 1, st[1:2].data_ptr(), stream), "selftest")
    torch.cuda.synchronize()
    assert st.tolist() == [1, 0]
    assert 2.0 <= e0.elapsed_time(e1) < 1000.0  # gave up after its 2 ms limit, not before
    idx = ops.hash_index((1024,), 64, 0, "cuda")  # the context still runs work
    assert int(idx.max()) < 64


def test_device_failure_word_raises_at_the_next_step():
    """A failure bit in the device status word (set here as a pass kernel sets it
    when a bounded wait gives up) makes check_device_status() raise, and the next
    step() raise before it launches anything; a clean step leaves the word at 0."""
    p = torch.nn.Parameter((torch.randn((512, 512), generator=torch.Generator().manual_seed(3)) * 0.02).cuda())
    opt = cresso_b200.CRESSO5([p], rank=8, hash_bins=64, hash_tables=2)
    p.grad = torch.full_like(p, 1e-3)
    opt.step()
    opt.check_device_status()  # clean: no raise
    assert opt._device_status() == 0
    opt._status_word(p.device).fill_(1)
    opt.step()  # its start still sees the previous step's clean copy
    with pytest.raises(RuntimeError, match="bounded wait"):
        opt.check_device_status()
    with pytest.raises(RuntimeError, match="bounded wait"):
        opt.step()


def test_nvtx_ranges_switch_on_without_changing_results():
    """CRESSO_B200_NVTX=1 wraps the entry calls and stages in NVTX ranges; the
    step is unchanged (a child process, so the switch is read at load)."""
    import subprocess
    import sys
    code = (
        "import torch, cresso_b200\n"
        "g = torch.Generator().manual_seed(0)\n"
        "ps = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).cuda()) for s in [(256, 256), (512, 16), (9,)]]\n"
        "opt = cresso_b200.CRESSO5(ps, rank=8, hash_bins=64, micro_field_max_size=16)\n"
        "for _ in range(2):\n"
        "    for p in ps: p.grad = torch.full_like(p, 1e-3)\n"
        "    opt.step()\n"
        "torch.cuda.synchronize()\n"
        "print(repr([float(p.double().sum()) for p in ps]))\n"
    )
    env = dict(os.environ)
    outs = []
    for flag in ("0", "1"):
        env["CRESSO_B200_NVTX"] = flag
        r = subprocess.run([sys.executable, "-c", code], env=env, cwd=str(ROOT), capture_output=True, text=True,
                           timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(r.stdout.strip().splitlines()[-1])
    assert outs[0] == outs[1]


def test_fast_routing_path_follows_the_full_one():
    """Steps reuse the previous routing only while nothing it depends on changed:
    a parameter without a gradient, a state_dict reload and a new gradient type
    each send the step back through the full checks.  The sequence is compared
    with the oracle doing the same steps."""
    g = torch.Generator().manual_seed(11)
    shapes = [(256, 256), (512, 16), (9,)]
    inits = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    kw = dict(rank=8, hash_bins=64, hash_tables=2, micro_field_max_size=16)
    ps = [torch.nn.Parameter(x.clone().cuda()) for x in inits]
    rs = [torch.nn.Parameter(x.clone()) for x in inits]
    opt = cresso_b200.CRESSO5(ps, **kw)
    ref = O.OracleCRESSO5(rs, **kw)
    for step in range(6):
        gs = [torch.randn(s, generator=g) * 1e-3 for s in shapes]
        for i, (p, r, gg) in enumerate(zip(ps, rs, gs)):
            skip = step == 3 and i == 0
            p.grad = None if skip else gg.cuda()
            r.grad = None if skip else gg.clone()
        if step == 4:  # reload the state: new state dicts, the cached routing must not be used
            opt.load_state_dict(copy.deepcopy(opt.state_dict()))
        opt.step()
        ref.step()
        assert (0 in opt._fast) == (step != 3)  # recorded after every pass in which all took part
    torch.cuda.synchronize()
    for p, r, s in zip(ps, rs, shapes):
        assert opt.state[p]["step"] == ref.state[r]["step"], s
        assert rel_rms(p.detach().cpu(), r.detach()) <= 1e-5, s
