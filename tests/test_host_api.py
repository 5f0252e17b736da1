"""Host-side API of cresso_b200 (no GPU): frequency pack and routing against
the reference goldens, constructor validation, state sizes, required-mode
errors.  Mirrors the reference's routing and safety tests
(tests/test_cresso_v5_routing.py, tests/test_cresso_v5_safety.py)."""

import numpy as np
import pytest
import torch

import cresso_b200
from cresso_b200 import _host
from oracle import cresso5_oracle as O


def test_frequency_pack_matches_reference(golden):
    for key, val in golden.items():
        if key.startswith("freqs_"):
            _, nd, mf, rk = key.split("_")
            got = np.asarray(_host.multiscale_frequencies(int(rk[1:]), int(nd[1:]), int(mf[1:])), dtype=np.int64)
            np.testing.assert_array_equal(got.reshape(val.shape), val.astype(np.int64), err_msg=key)


def test_omega_matches_oracle():
    f = _host.frequencies_tensor(8, 2, 5, "cpu")
    torch.testing.assert_close(_host.omega_from_freqs(f), O.omega_from_freqs(f), rtol=0, atol=0)


@pytest.mark.parametrize("shape", [(128, 16), (16, 128), (4096, 16), (64, 64), (4096,), (8, 8), (300, 8), (1, 5000)])
@pytest.mark.parametrize("route", ["scalar", "spectral"])
def test_routing_and_state_size_match_oracle(shape, route):
    group = O.hparams(rank=4, min_spectral_size=1024, thin_matrix_route=route)
    assert _host.uses_spectral_route(shape, group) == O.uses_spectral(shape, group)
    kw = dict(rank=4, thin_matrix_route=route)
    assert _host.theoretical_state_elements(shape, **kw) == O.theoretical_state_elements(shape, **kw)


def test_lora_thin_matrix_uses_scalar_route_by_default():
    """tests/test_cresso_v5_routing.py:18-29: (128,16) -> scalar route, 8 state elements."""
    assert not _host.uses_spectral_route((128, 16), O.hparams(rank=4))
    assert cresso_b200.theoretical_state_elements((128, 16), rank=4) == 8
    assert cresso_b200.theoretical_state_elements((128, 16), rank=4, thin_matrix_route="spectral") == 4 * 2 + 48 + 3 * 128 * 2 + 4


def test_constructor_defaults_match_reference_keys():
    p = torch.nn.Parameter(torch.zeros(4))
    opt = cresso_b200.CRESSO5([p])
    g = opt.param_groups[0]
    for k, v in O.DEFAULTS.items():
        assert g[k] == v, k
    assert g["cuda_ops"] == "auto"
    assert cresso_b200.CRESSO is cresso_b200.CRESSO5


@pytest.mark.parametrize("kw,msg", [
    (dict(lr=-1.0), "lr must be >="), (dict(dt=2.0), "dt must be <="), (dict(rank=-1), "rank must be non-negative"),
    (dict(hash_tables=0), "hash_tables must be >= 1"), (dict(min_gain=7.0), "min_gain must be <= max_gain"),
    (dict(thin_matrix_route="x"), "thin_matrix_route"), (dict(cuda_ops="sometimes"), "cuda_ops must be one of"),
    (dict(energy_power=float("nan")), "finite"), (dict(thin_matrix_min_aspect=0.5), "thin_matrix_min_aspect"),
])
def test_constructor_validation(kw, msg):
    p = torch.nn.Parameter(torch.zeros(4))
    with pytest.raises(ValueError, match=msg):
        cresso_b200.CRESSO5([p], **kw)


@pytest.mark.parametrize("mode", ["off", False])
def test_cuda_ops_off_is_rejected(mode):
    with pytest.raises(ValueError, match="fused CUDA path"):
        cresso_b200.CRESSO5([torch.nn.Parameter(torch.zeros(4))], cuda_ops=mode)


def test_required_rejects_cpu_params():
    """tests/test_cresso_v5_safety.py:39-45."""
    p = torch.nn.Parameter(torch.ones(4, 4))
    p.grad = torch.ones_like(p)
    opt = cresso_b200.CRESSO5([p], cuda_ops="required", min_spectral_size=1)
    with pytest.raises(RuntimeError, match="cuda_ops='required'.*CUDA parameter"):
        opt.step()


def test_params_without_grad_are_skipped_and_closure_is_returned():
    p = torch.nn.Parameter(torch.ones(3))
    opt = cresso_b200.CRESSO5([p])
    assert opt.step(lambda: 7.0) == 7.0
    assert len(opt.state) == 0


def test_count_state_elements_helper():
    class Fake:
        state = {0: {"a": torch.zeros(3, 2), "step": 4}, 1: {"b": torch.zeros(())}}
    assert cresso_b200.count_optimizer_state_elements(Fake()) == 7


@pytest.mark.parametrize("workload,sharded", [("c2", True), ("c3", False)])
def test_bench_row_sharding_marks_only_spectral_route_tensors(workload, sharded):
    """bench.py at N > 1 (row sharding): 1-D / 2-D tensors on the spectral route
    are cut into row blocks, the rest (LoRA-thin scalar-route tensors) stay whole
    for their owner ranks."""
    import bench
    from cresso_b200.distributed import row_block

    class Args:
        dtype = "f32"

    shapes, kw, params, grads, n_local, n_total, bpe = bench.make_inputs(workload, Args, 2, 1, torch.device("cpu"),
                                                                        False)
    for s, p in zip(shapes, params):
        spec = getattr(p, "_cresso_shard", None)
        assert (spec is not None) == sharded
        if sharded:
            start, stop = row_block(s[0], 1, 2)
            assert tuple(p.shape) == (stop - start,) + tuple(s[1:]) and spec == (tuple(s), start)
        else:
            assert tuple(p.shape) == tuple(s)
