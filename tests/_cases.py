"""Shared case definitions and input generators for the parity tests.

The full-step cases and their seeds are the ones tests/golden/make_golden.py
ran through the reference; inputs are regenerated here with the same torch CPU
generator calls (and checked against the stored input sums).
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]


def golden_cases():
    spec = importlib.util.spec_from_file_location("make_golden", ROOT / "tests" / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.STEP_CASES


def case_inputs(golden, name, shape, steps, seed, istd, gstd):
    gen = torch.Generator().manual_seed(seed)
    init = (torch.randn(shape, generator=gen) * istd).float()
    grads = [(torch.randn(shape, generator=gen) * gstd).float() for _ in range(steps)]
    np.testing.assert_allclose(float(init.double().sum()), float(golden[f"step_{name}_init_sum"]), rtol=0, atol=0)
    np.testing.assert_allclose(sum(float(g.double().abs().sum()) for g in grads),
                               float(golden[f"step_{name}_grad_sum"]), rtol=1e-12)
    return init, grads


def extra_cases():
    spec = importlib.util.spec_from_file_location("make_golden", ROOT / "tests" / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.EXTRA_CASES


def extra_case_inputs(golden, name, shape, steps, seed, istd, gstd, dtype):
    """Inputs of a case of the second golden table (16-bit parameters, tensors of
    rank >= 3), regenerated from its seed exactly as the generator made them
    (float32 draws rounded to the parameter type)."""
    dt = getattr(torch, dtype)
    gen = torch.Generator().manual_seed(seed)
    init = (torch.randn(shape, generator=gen) * istd).float().to(dt)
    grads = [(torch.randn(shape, generator=gen) * gstd).float().to(dt) for _ in range(steps)]
    np.testing.assert_allclose(float(init.double().sum()), float(golden[f"step_{name}_init_sum"]), rtol=0, atol=0)
    np.testing.assert_allclose(sum(float(g.double().abs().sum()) for g in grads),
                               float(golden[f"step_{name}_grad_sum"]), rtol=1e-12)
    return init, grads


def ulp_distance(a, b, dtype) -> "np.ndarray":
    """|a - b| in units in the last place of `dtype` (float16 / bfloat16) at the
    larger of |b| and the RMS of b: near zero a parameter's own ulp is far below
    the rounding step of the update it receives, so the tensor's scale is used."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    mant = 10 if dtype == "float16" else 7
    scale = max(float(np.sqrt(np.mean(b * b))), 2.0 ** -14 if dtype == "float16" else 2.0 ** -126)
    e = np.floor(np.log2(np.maximum(np.abs(b), scale)))
    return np.abs(a - b) / 2.0 ** (e - mant)


def rel_rms(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.sqrt(np.mean(b * b))
    return float(np.sqrt(np.mean((a - b) ** 2)) / max(den, 1e-30))
