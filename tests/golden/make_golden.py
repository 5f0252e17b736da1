"""Generate golden vectors for the CRESSO5 step by running the reference itself.

Usage:  python tests/golden/make_golden.py [path-to-reference-checkout] [--extra-only]

The reference (win10ogod/cresso, ``cresso_v5.py``) is imported from the given
checkout and run on CPU with ``cuda_ops='off'`` and one thread, which is its
PyTorch path.  Outputs are written next to this script:

* ``golden_small.npz`` - frequency packs, hash indices, hash bin counts at the
  benchmark sizes, basis projections / reconstructions, instant metrics and
  full optimizer steps (inputs, final params, every state tensor).
* ``golden_extra.npz`` - full optimizer steps of ``EXTRA_CASES``: float16 /
  bfloat16 parameters (values stored as float32, which holds every 16-bit
  value exactly) and spectral-route tensors of rank 3 to 5.  ``--extra-only``
  regenerates just this file.

The reference is not available where the tests run, so the vectors are
committed; the tests only read the ``.npz``.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    spec = importlib.util.spec_from_file_location("cresso_v5_reference", root / "cresso_v5.py")
    mod = importlib.util.module_from_spec(spec)
    assert spec is not None and spec.loader is not None
    spec.loader.exec_module(mod)
    return mod


# Full-step cases: name -> (shape, kwargs, steps, seed, init_std, grad_std)
STEP_CASES = {
    "spec_31x37_ref_test": ((31, 37), dict(lr=2e-3, rank=8, max_frequency=5, min_spectral_size=1,
                                           hard_channel_min_size=1, thin_matrix_hard_cutoff=0,
                                           hash_bins=37, hash_tables=2, basis_cache_limit_elements=0),
                            3, 9012, 1.0, 1.0),
    "spec_64x64_b64": ((64, 64), dict(rank=8, max_frequency=5, hash_bins=64, hash_tables=2), 5, 11, 0.02, 1e-3),
    "spec_48x80_wd_local": ((48, 80), dict(rank=8, hash_bins=64, hash_tables=2, weight_decay=0.01,
                                           local_sharpness=0.3, min_spectral_size=1, maximize=True), 3, 12, 0.02, 1e-3),
    "spec_1d_1500": ((1500,), dict(rank=8, hash_bins=64, hash_tables=2), 4, 13, 0.02, 1e-3),
    "spec_r5_40x50": ((40, 50), dict(rank=5, max_frequency=3, hash_bins=16, hash_tables=3,
                                     min_spectral_size=1, warmup_steps=0), 3, 14, 0.02, 1e-3),
    "spec_maxf0_40x40": ((40, 40), dict(rank=4, max_frequency=0, hash_bins=64, hash_tables=1,
                                        min_spectral_size=1), 3, 15, 0.02, 1e-3),
    "spec_nohash_96x40": ((96, 40), dict(rank=8, hash_bins=0, min_spectral_size=1, echo_mix=0.0), 3, 16, 0.02, 1e-3),
    "spec_thincut_300x8": ((300, 8), dict(rank=4, hash_bins=64, thin_matrix_route="spectral",
                                          min_spectral_size=1), 3, 17, 0.02, 1e-3),
    "spec_thin_128x16": ((128, 16), dict(rank=4, hash_bins=64, hash_tables=2, thin_matrix_route="spectral",
                                         min_spectral_size=1), 3, 18, 0.01, 1e-3),
    "spec_r16_72x90": ((72, 90), dict(rank=16, max_frequency=5, hash_bins=128, hash_tables=2,
                                      min_spectral_size=1), 3, 19, 0.02, 1e-3),
    "spec_256x256_b64": ((256, 256), dict(rank=8, hash_bins=64, hash_tables=2), 3, 20, 0.02, 1e-3),
    "scal_128x16": ((128, 16), dict(lr=2e-3, rank=4, thin_matrix_route="scalar", min_spectral_size=1), 3, 2468, 1.0, 1.0),
    "scal_16x128": ((16, 128), dict(rank=4, min_spectral_size=1), 3, 21, 0.01, 1e-3),
    "scal_small_10x12": ((10, 12), dict(rank=8), 3, 22, 0.02, 1e-3),
    "scal_1d_300": ((300,), dict(rank=8, weight_decay=0.02), 3, 23, 0.02, 1e-3),
    "scal_0d": ((), dict(rank=8), 3, 24, 0.02, 1e-3),
    "scal_3d_4x5x6": ((4, 5, 6), dict(rank=8, local_sharpness=0.2), 3, 25, 0.02, 1e-3),
    "scal_4096x16": ((4096, 16), dict(rank=4, hash_bins=64, hash_tables=2), 3, 26, 0.01, 1e-3),
}


# More cases: name -> (shape, kwargs, steps, seed, init_std, grad_std, dtype).  The 16-bit ones
# start with the shapes and settings of the reference's own 16-bit tests
# (tests/test_cresso_v5_cuda_ops.py:109-146, 213-250); the N-d ones are spectral-route
# tensors of rank 3 to 5 (conv-like weights) with the four carrier kinds and the instant metric.
_REF_SPEC16 = dict(lr=1.0e-3, rank=8, max_frequency=5, min_spectral_size=1, hard_channel_min_size=1,
                   thin_matrix_hard_cutoff=0, hash_bins=37, hash_tables=2, basis_cache_limit_elements=0)
_REF_SCAL16 = dict(lr=1.0e-3, rank=4, thin_matrix_route="scalar", thin_matrix_max_width=64, min_spectral_size=1)
EXTRA_CASES = {
    "spec16_31x37_f16": ((31, 37), _REF_SPEC16, 2, 8642, 0.05, 0.05, "float16"),
    "spec16_31x37_bf16": ((31, 37), _REF_SPEC16, 2, 8643, 0.05, 0.05, "bfloat16"),
    "scal16_64x16_f16": ((64, 16), _REF_SCAL16, 2, 3579, 0.05, 0.05, "float16"),
    "scal16_64x16_bf16": ((64, 16), _REF_SCAL16, 2, 3580, 0.05, 0.05, "bfloat16"),
    "spec16_256x256_bf16_wd": ((256, 256), dict(rank=8, hash_bins=64, hash_tables=2, weight_decay=0.01),
                               3, 31, 0.02, 1e-3, "bfloat16"),
    "scal16_16x4096_f16": ((16, 4096), dict(rank=4, hash_bins=64, hash_tables=2), 3, 32, 0.01, 1e-3, "float16"),
    "nd_16x8x3x3": ((16, 8, 3, 3), dict(rank=8, hash_bins=64, hash_tables=2), 3, 41, 0.02, 1e-3, "float32"),
    "nd_8x6x40_wd_local": ((8, 6, 40), dict(rank=8, hash_bins=37, hash_tables=2, weight_decay=0.01,
                                            local_sharpness=0.3, maximize=True), 3, 42, 0.02, 1e-3, "float32"),
    "nd_3x4x5x6x7_r16": ((3, 4, 5, 6, 7), dict(rank=16, max_frequency=3, hash_bins=16, hash_tables=3,
                                               warmup_steps=0), 3, 43, 0.02, 1e-3, "float32"),
    "nd_4x64x256": ((4, 64, 256), dict(rank=8, hash_bins=64, hash_tables=2, instant_metric_power=0.7), 3, 44,
                    0.02, 1e-3, "float32"),
    "nd_32x16x5x5_bf16": ((32, 16, 5, 5), dict(rank=4, hash_bins=64, hash_tables=1), 3, 45, 0.02, 1e-3,
                          "bfloat16"),
    # micro-field route (micro_field_max_size > 0): per-element energy / impulse / refractory state
    "micro_64x32": ((64, 32), dict(micro_field_max_size=4096), 4, 51, 0.02, 1e-3, "float32"),
    "micro_4096_wd_max": ((4096,), dict(micro_field_max_size=4096, weight_decay=0.01, maximize=True), 3, 52, 0.02,
                          1e-3, "float32"),
    "micro_8x6x5_ip": ((8, 6, 5), dict(micro_field_max_size=1000, instant_metric_power=0.7,
                                       instant_metric_coupling=0.2, micro_drive_mix=0.5), 3, 53, 0.02, 1e-3,
                       "float32"),
    "micro_1x1000": ((1, 1000), dict(micro_field_max_size=1000, energy_power=1.0), 3, 54, 0.02, 1e-3, "float32"),
    "micro_3": ((3,), dict(micro_field_max_size=16), 3, 55, 0.02, 1e-3, "float32"),
    "micro_1": ((1,), dict(micro_field_max_size=16), 3, 56, 0.02, 1e-3, "float32"),
    "micro_64x256": ((64, 256), dict(micro_field_max_size=16384, micro_decay=0.8), 3, 57, 0.02, 1e-3, "float32"),
    "micro_300x7_bf16": ((300, 7), dict(micro_field_max_size=4096), 3, 58, 0.02, 1e-3, "bfloat16"),
    "micro_2x3x4x5_f16": ((2, 3, 4, 5), dict(micro_field_max_size=4096, weight_decay=0.05), 3, 59, 0.02, 1e-3,
                          "float16"),
    # float64 parameters: float64 work and state on the scalar and micro-field routes
    "scal64_256x16": ((256, 16), dict(rank=4, hash_bins=64, hash_tables=2), 3, 61, 0.02, 1e-3, "float64"),
    "scal64_7x9_wd": ((7, 9), dict(weight_decay=0.01, maximize=True), 3, 62, 0.02, 1e-3, "float64"),
    "scal64_3x4x5": ((3, 4, 5), dict(instant_metric_power=0.7), 3, 63, 0.02, 1e-3, "float64"),
    "scal64_1024x16": ((1024, 16), dict(rank=4), 3, 64, 0.01, 1e-3, "float64"),
    "micro64_30x20": ((30, 20), dict(micro_field_max_size=1000), 3, 65, 0.02, 1e-3, "float64"),
    "micro64_2x3x4": ((2, 3, 4), dict(micro_field_max_size=100, maximize=True, weight_decay=0.02), 3, 66, 0.02, 1e-3,
                      "float64"),
    # float64 parameters on the spectral route
    "spec64_96x80": ((96, 80), dict(), 3, 71, 0.02, 1e-3, "float64"),
    "spec64_64x64_wd_local_max": ((64, 64), dict(rank=8, hash_bins=64, hash_tables=2, weight_decay=0.01,
                                                 local_sharpness=0.3, maximize=True), 3, 72, 0.02, 1e-3, "float64"),
    "spec64_2048": ((2048,), dict(rank=8, hash_bins=64, hash_tables=2), 3, 73, 0.02, 1e-3, "float64"),
    "spec64_8x6x40": ((8, 6, 40), dict(rank=4, hash_bins=32, hash_tables=1), 3, 74, 0.02, 1e-3, "float64"),
    "spec64_128x40_r16": ((128, 40), dict(rank=16, hash_bins=37, hash_tables=3, instant_metric_power=0.7,
                                          warmup_steps=0), 3, 75, 0.02, 1e-3, "float64"),
    "spec64_thin_8x512": ((8, 512), dict(rank=8, thin_matrix_route="spectral"), 3, 76, 0.02, 1e-3, "float64"),
    # rank above 16 (the float64-arithmetic spectral path for float32 tensors)
    "r32_96x80": ((96, 80), dict(rank=32, hash_bins=64, hash_tables=2), 3, 81, 0.02, 1e-3, "float32"),
    "r24_3000_wd": ((3000,), dict(rank=24, weight_decay=0.01, max_frequency=7), 3, 82, 0.02, 1e-3, "float32"),
    "r20_6x8x30": ((6, 8, 30), dict(rank=20, hash_bins=37, hash_tables=1, local_sharpness=0.2), 3, 83, 0.02, 1e-3,
                   "float32"),
    "r32_f64_64x48": ((64, 48), dict(rank=32), 3, 84, 0.02, 1e-3, "float64"),
    # 16-bit parameters above rank 16, and ranks 33 to 64 (the same float64-arithmetic path)
    "r24_bf16_80x96": ((80, 96), dict(rank=24, hash_bins=64, hash_tables=2), 3, 85, 0.02, 1e-3, "bfloat16"),
    "r20_f16_2000_wd": ((2000,), dict(rank=20, weight_decay=0.01, max_frequency=7), 3, 86, 0.02, 1e-3, "float16"),
    "r48_64x80": ((64, 80), dict(rank=48, hash_bins=64, hash_tables=2), 3, 87, 0.02, 1e-3, "float32"),
    "r40_5x6x20_local": ((5, 6, 20), dict(rank=40, hash_bins=37, hash_tables=1, local_sharpness=0.2), 3, 88, 0.02,
                         1e-3, "float32"),
    "r64_f64_40x50": ((40, 50), dict(rank=64, hash_bins=64, hash_tables=2), 3, 89, 0.02, 1e-3, "float64"),
    "r64_bf16_48x64": ((48, 64), dict(rank=64, max_frequency=7), 3, 90, 0.02, 1e-3, "bfloat16"),
    # ranks above 64 (modes in memory, projections in chunks of modes)
    "r96_64x80": ((64, 80), dict(rank=96, hash_bins=64, hash_tables=2), 3, 91, 0.02, 1e-3, "float32"),
    "r65_40x50": ((40, 50), dict(rank=65, hash_bins=37, hash_tables=3, instant_metric_power=0.7), 3, 92, 0.02,
                  1e-3, "float32"),
    "r128_3000_wd": ((3000,), dict(rank=128, weight_decay=0.01, max_frequency=7), 3, 93, 0.02, 1e-3, "float32"),
    "r80_f64_6x8x30": ((6, 8, 30), dict(rank=80, hash_bins=37, hash_tables=1, local_sharpness=0.2), 3, 94, 0.02,
                       1e-3, "float64"),
    "r200_bf16_48x64": ((48, 64), dict(rank=200, max_frequency=7), 3, 95, 0.02, 1e-3, "bfloat16"),
}


def run_steps(ref, shape, kwargs, steps, seed, init_std, grad_std, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    init = (torch.randn(shape, generator=gen) * init_std).float().to(dtype)
    grads = [(torch.randn(shape, generator=gen) * grad_std).float().to(dtype) for _ in range(steps)]
    p = torch.nn.Parameter(init.clone())
    opt = ref.CRESSO5([p], cuda_ops="off", **kwargs)
    for g in grads:
        p.grad = g.clone()
        opt.step()
    st = opt.state[p]
    # float64 results stay float64; the other types are stored as float32, which holds them exactly
    final = p.detach().numpy() if dtype == torch.float64 else p.detach().float().numpy()
    out = {"final": final.copy(),
           "init_sum": np.asarray(init.double().sum().item()),
           "grad_sum": np.asarray(sum(g.double().abs().sum().item() for g in grads))}
    if init.numel() <= 4096:
        # Small inputs are stored; larger ones are regenerated from the seed and
        # checked against the stored sums.
        out["init"] = init.float().numpy()
        out["grads"] = np.stack([g.float().numpy() for g in grads])
    for k, v in st.items():
        if torch.is_tensor(v):
            out["state_" + k] = v.detach().cpu().numpy().copy()
        else:
            out["state_" + k] = np.asarray(v)
    out["state_elements"] = np.asarray(ref.count_optimizer_state_elements(opt))
    return out


def main() -> None:
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = Path(args[0] if args else os.environ.get("CRESSO_REFERENCE", "/root/reference"))
    ref = load_reference(root)
    torch.set_num_threads(1)

    extra: dict[str, np.ndarray] = {}
    for name, (shape, kwargs, steps, seed, istd, gstd, dt) in EXTRA_CASES.items():
        out = run_steps(ref, shape, kwargs, steps, seed, istd, gstd, getattr(torch, dt))
        for k, v in out.items():
            extra[f"step_{name}_{k}"] = v
    np.savez_compressed(HERE / "golden_extra.npz", **extra)
    print("wrote", HERE / "golden_extra.npz", len(extra), "arrays")
    if "--extra-only" in sys.argv:
        return

    data: dict[str, np.ndarray] = {}

    # Frequency packs (cresso_v5.py:145-227).
    for ndim in (1, 2, 3):
        for maxf in (0, 1, 2, 5):
            for rank in list(range(1, 17)) + [24, 32, 64]:
                f = ref._make_multiscale_frequencies(rank, ndim, maxf, torch.device("cpu"))
                data[f"freqs_n{ndim}_m{maxf}_r{rank}"] = f.numpy().astype(np.int16)

    # Hash indices (cresso_v5.py:495-516): full vectors at small n, counts at benchmark sizes.
    for bins in (1, 7, 37, 64, 128, 4096):
        for salt in range(4):
            idx = ref._hash_index_tensor((1024,), bins, torch.device("cpu"), salt=salt)
            data[f"hash_b{bins}_s{salt}"] = idx.numpy().astype(np.int32)
    for n in (2048 * 2048, 4096 * 4096, 32000 * 4096):
        for salt in range(2):
            idx = ref._hash_index_tensor((n,), 64, torch.device("cpu"), salt=salt)
            data[f"hashcount_n{n}_b64_s{salt}"] = torch.bincount(idx, minlength=64).numpy().astype(np.int64)
            # Spot values at the top of the range, where the first product is largest.
            data[f"hashtail_n{n}_b64_s{salt}"] = idx[-257:].numpy().astype(np.int32)
            del idx

    # Basis projection / reconstruction (cresso_v5.py:295-376), incl. the reference test shape.
    for shape, rank, maxf, seed in (((17, 19), 8, 5, 1234), ((31, 37), 8, 5, 5), ((1500,), 8, 5, 6),
                                    ((8, 200), 4, 3, 7), ((200, 8), 16, 5, 8), ((64, 64), 32, 5, 9),
                                    ((1, 50), 8, 5, 10), ((50, 1), 8, 5, 11)):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(shape, generator=gen)
        freqs = ref._make_multiscale_frequencies(rank, len(shape), maxf, torch.device("cpu"))
        c, s = ref._project(x, freqs, rank)
        gates = torch.sigmoid(torch.linspace(-2.0, 2.0, rank))
        rec = ref._reconstruct(c, s, freqs, shape, torch.float32, gates=gates)
        key = "basis_" + "x".join(str(d) for d in shape) + f"_r{rank}"
        data[key + "_x"] = x.numpy()
        data[key + "_cos"] = c.numpy()
        data[key + "_sin"] = s.numpy()
        data[key + "_rec"] = rec.numpy()
        data[key + "_maxf"] = np.asarray(maxf)

    # Hash bin mean (reference test shape) and instant metric.
    gen = torch.Generator().manual_seed(5678)
    x = torch.randn((23, 29), generator=gen)
    idx = ref._hash_index_tensor((23, 29), 37, torch.device("cpu"), salt=2)
    data["hashmean_23x29_b37_s2_x"] = x.numpy()
    data["hashmean_23x29_b37_s2"] = ref._hash_reduce_mean(x, idx, 37).numpy()
    for shape in ((33, 47), (500,), (3, 4, 5)):
        gen = torch.Generator().manual_seed(77)
        rel = torch.rand(shape, generator=gen) * 3.0 + 1e-3
        key = "instant_" + "x".join(str(d) for d in shape)
        data[key + "_rel"] = rel.numpy()
        data[key] = ref._instant_axis_metric(rel, 1.0, 0.55, 1e-8).numpy()

    # Full optimizer steps through the reference's own CRESSO5 (PyTorch path).
    for name, (shape, kwargs, steps, seed, istd, gstd) in STEP_CASES.items():
        out = run_steps(ref, shape, kwargs, steps, seed, istd, gstd)
        for k, v in out.items():
            data[f"step_{name}_{k}"] = v

    np.savez_compressed(HERE / "golden_small.npz", **data)
    print("wrote", HERE / "golden_small.npz", len(data), "arrays")


if __name__ == "__main__":
    main()
