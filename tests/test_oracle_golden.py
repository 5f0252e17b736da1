"""The oracle restatement against golden vectors produced by the reference
itself (tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest
import torch

from oracle import cresso5_oracle as O
from tests._cases import case_inputs, extra_case_inputs, extra_cases, golden_cases


def test_frequency_pack_matches_reference(golden):
    n = 0
    for key, val in golden.items():
        if not key.startswith("freqs_"):
            continue
        _, nd, mf, rk = key.split("_")
        got = np.asarray(O.multiscale_frequencies(int(rk[1:]), int(nd[1:]), int(mf[1:])), dtype=np.int64)
        np.testing.assert_array_equal(got.reshape(val.shape), val.astype(np.int64), err_msg=key)
        n += 1
    assert n == 3 * 4 * 19


@pytest.mark.parametrize("bins", [1, 7, 37, 64, 128, 4096])
def test_hash_index_bit_exact(golden, bins):
    for salt in range(4):
        ref = golden[f"hash_b{bins}_s{salt}"].astype(np.int64)
        np.testing.assert_array_equal(O.hash_index_np(1024, bins, salt), ref)
        t = O.hash_index_tensor((1024,), bins, "cpu", salt=salt).numpy()
        np.testing.assert_array_equal(t, ref)


@pytest.mark.parametrize("n", [2048 * 2048, 4096 * 4096])
def test_hash_bin_counts_at_benchmark_sizes(golden, n):
    for salt in range(2):
        idx = O.hash_index_np(n, 64, salt)
        np.testing.assert_array_equal(np.bincount(idx, minlength=64), golden[f"hashcount_n{n}_b64_s{salt}"])
        np.testing.assert_array_equal(idx[-257:], golden[f"hashtail_n{n}_b64_s{salt}"])


def test_hash_tail_of_largest_tensor(golden):
    n = 32000 * 4096
    for salt in range(2):
        np.testing.assert_array_equal(O.hash_index_np(257, 64, salt, offset=n - 257), golden[f"hashtail_n{n}_b64_s{salt}"])


def test_basis_projection_and_reconstruction(golden):
    keys = [k[: -len("_x")] for k in golden if k.startswith("basis_") and k.endswith("_x")]
    assert len(keys) == 8
    for key in keys:
        x = torch.from_numpy(golden[key + "_x"])
        rank = golden[key + "_cos"].shape[0]
        freqs = O.freqs_tensor(rank, x.ndim, int(golden[key + "_maxf"]))
        c, s = O.project(x, freqs)
        np.testing.assert_array_equal(c.numpy(), golden[key + "_cos"])
        np.testing.assert_array_equal(s.numpy(), golden[key + "_sin"])
        gates = torch.sigmoid(torch.linspace(-2.0, 2.0, rank))
        rec = O.reconstruct(c, s, freqs, tuple(x.shape), torch.float32, gates=gates)
        np.testing.assert_array_equal(rec.numpy(), golden[key + "_rec"])


def test_hash_mean_and_instant_metric(golden):
    x = torch.from_numpy(golden["hashmean_23x29_b37_s2_x"])
    idx = O.hash_index_tensor((23, 29), 37, "cpu", salt=2)
    np.testing.assert_array_equal(O.hash_reduce_mean(x, idx, 37).numpy(), golden["hashmean_23x29_b37_s2"])
    for shape in ("33x47", "500", "3x4x5"):
        rel = torch.from_numpy(golden[f"instant_{shape}_rel"])
        np.testing.assert_array_equal(O.instant_axis_metric(rel, 1.0, 0.55, 1e-8).numpy(), golden[f"instant_{shape}"])


@pytest.mark.parametrize("name", list(golden_cases().keys()))
def test_full_steps_bit_exact(golden, name):
    torch.set_num_threads(1)
    shape, kw, steps, seed, istd, gstd = golden_cases()[name]
    init, grads = case_inputs(golden, name, shape, steps, seed, istd, gstd)
    p = torch.nn.Parameter(init.clone())
    opt = O.OracleCRESSO5([p], **kw)
    for g in grads:
        p.grad = g.clone()
        opt.step()
    np.testing.assert_array_equal(p.detach().numpy(), golden[f"step_{name}_final"])
    st = opt.state[p]
    for k, v in st.items():
        ref = golden[f"step_{name}_state_{k}"]
        got = v.numpy() if torch.is_tensor(v) else np.asarray(v)
        np.testing.assert_array_equal(got.astype(ref.dtype), ref, err_msg=k)
    assert O.count_state_elements(opt.state) == int(golden[f"step_{name}_state_elements"])


@pytest.mark.parametrize("name", list(extra_cases().keys()))
def test_extra_steps_bit_exact(golden_extra, name):
    """float16 / bfloat16 parameters (fp32 work and state, update rounded to the
    parameter type before the add), float64 parameters (float64 work and state),
    spectral tensors of rank 3 to 5 and the micro-field route: the oracle
    reproduces the reference bit for bit."""
    torch.set_num_threads(1)
    shape, kw, steps, seed, istd, gstd, dt = extra_cases()[name]
    init, grads = extra_case_inputs(golden_extra, name, shape, steps, seed, istd, gstd, dt)
    p = torch.nn.Parameter(init.clone())
    opt = O.OracleCRESSO5([p], **kw)
    for g in grads:
        p.grad = g.clone()
        opt.step()
    assert p.dtype == getattr(torch, dt)
    np.testing.assert_array_equal(p.detach().double().numpy(), golden_extra[f"step_{name}_final"].astype(np.float64))
    for k, v in opt.state[p].items():
        ref = golden_extra[f"step_{name}_state_{k}"]
        got = v.numpy() if torch.is_tensor(v) else np.asarray(v)
        if torch.is_tensor(v) and torch.is_floating_point(v):
            assert v.dtype == (torch.float64 if dt == "float64" else torch.float32), k
        np.testing.assert_array_equal(got.astype(ref.dtype), ref, err_msg=k)
