"""Host-side helpers of the CRESSO5 API: constructor validation, routing
predicates, the deterministic frequency pack and state-size utilities.

These are small pieces of Python logic of the reference API
(``cresso_v5.py``) that the B200 build keeps on the host; every function
cites the reference lines whose behaviour it reproduces.
"""

from __future__ import annotations

import math
from typing import Iterable, List, Sequence, Tuple

import torch


def validate_scalar(name: str, value, lower=None, upper=None) -> None:
    """cresso_v5.py:110-116."""
    if not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise ValueError(f"{name} must be a finite scalar, got {value!r}")
    if lower is not None and value < lower:
        raise ValueError(f"{name} must be >= {lower}, got {value}")
    if upper is not None and value > upper:
        raise ValueError(f"{name} must be <= {upper}, got {value}")


def normalize_thin_matrix_route(route: str) -> str:
    """cresso_v5.py:538-542."""
    r = str(route).lower()
    if r not in {"scalar", "spectral"}:
        raise ValueError("thin_matrix_route must be one of 'scalar' or 'spectral'")
    return r


def is_lora_thin_matrix_shape(shape: Sequence[int], thin_matrix_max_width: int = 64,
                              thin_matrix_min_aspect: float = 4.0) -> bool:
    """2-D, short side <= max width, aspect >= min aspect.  cresso_v5.py:545-557."""
    dims = tuple(int(d) for d in shape)
    if len(dims) != 2 or int(thin_matrix_max_width) <= 0:
        return False
    short, long_ = min(dims), max(dims)
    if short <= 0:
        return False
    return short <= int(thin_matrix_max_width) and (long_ / short) >= float(thin_matrix_min_aspect)


def thin_matrix_uses_scalar_route(shape: Sequence[int], thin_matrix_route: str = "scalar",
                                  thin_matrix_max_width: int = 64, thin_matrix_min_aspect: float = 4.0) -> bool:
    """cresso_v5.py:560-570."""
    return normalize_thin_matrix_route(thin_matrix_route) == "scalar" and is_lora_thin_matrix_shape(
        shape, thin_matrix_max_width, thin_matrix_min_aspect)


def uses_spectral_route(shape: Sequence[int], group: dict) -> bool:
    """CRESSO5._use_spectral_route, cresso_v5.py:847-855."""
    n = 1
    for d in shape:
        n *= int(d)
    if not (n >= int(group["min_spectral_size"]) and int(group["rank"]) > 0 and len(shape) > 0):
        return False
    return not thin_matrix_uses_scalar_route(
        tuple(shape), str(group.get("thin_matrix_route", "scalar")),
        int(group.get("thin_matrix_max_width", 64)), float(group.get("thin_matrix_min_aspect", 4.0)))


def hard_enabled(shape: Sequence[int], group: dict) -> bool:
    """Hash / instant channels switch (cresso_v5.py:981-983)."""
    dims = tuple(int(d) for d in shape)
    n = 1
    for d in dims:
        n *= d
    cutoff = int(group["thin_matrix_hard_cutoff"])
    thin = len(dims) == 2 and cutoff > 0 and min(dims) <= cutoff
    return n >= int(group["hard_channel_min_size"]) and not thin


def multiscale_frequencies(rank: int, ndim: int, max_frequency: int) -> List[Tuple[int, ...]]:
    """Deterministic frequency pack (cresso_v5.py:145-227): zero mode, axis-local
    modes, (anti-)diagonals, pairwise mixed modes, then hashed modes."""
    rank, ndim, maxf = int(rank), int(ndim), max(0, int(max_frequency))
    if rank <= 0:
        return []
    modes: List[Tuple[int, ...]] = [tuple([0] * ndim)]
    seen = {modes[0]}

    def add(t) -> bool:
        t = tuple(t)
        if t not in seen:
            modes.append(t)
            seen.add(t)
        return len(modes) >= rank

    if maxf <= 0:
        return [modes[0]] * rank
    for f in range(1, maxf + 1):
        for axis in range(ndim):
            v = [0] * ndim
            v[axis] = f
            if add(v):
                return modes[:rank]
    for f in range(1, maxf + 1):
        if add([f] * ndim):
            return modes[:rank]
        if ndim > 1 and add([f if i % 2 == 0 else max(1, maxf + 1 - f) for i in range(ndim)]):
            return modes[:rank]
    if ndim > 1:
        for f1 in range(1, maxf + 1):
            for f2 in range(1, maxf + 1):
                for a in range(ndim):
                    v = [0] * ndim
                    v[a] = f1
                    v[(a + 1) % ndim] = f2
                    if add(v):
                        return modes[:rank]
    primes = (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37)
    n = 1
    attempts = 0
    guard = max(64, 10 * rank * max(1, ndim))
    while len(modes) < rank:
        v = []
        active = 0
        for axis in range(ndim):
            f = (n * primes[axis % len(primes)] + axis * axis + 3 * axis + 1) % (maxf + 1)
            active += f != 0
            v.append(int(f))
        if active == 0:
            v[n % ndim] = 1 + (n % maxf)
        elif active == 1 and ndim > 1:
            v[(n + 1) % ndim] = 1 + ((n // 2) % maxf)
        t = tuple(v)
        if t not in seen or attempts >= guard:
            modes.append(t)
            seen.add(t)
        n += 1
        attempts += 1
    return modes[:rank]


def frequencies_tensor(rank: int, ndim: int, max_frequency: int, device) -> torch.Tensor:
    modes = multiscale_frequencies(rank, ndim, max_frequency)
    if not modes:
        return torch.empty((0, ndim), dtype=torch.long, device=device)
    return torch.tensor(modes, dtype=torch.long, device=device)


def omega_from_freqs(freqs: torch.Tensor, base: float = 1.0) -> torch.Tensor:
    """base * sqrt(1 + |f|^2) per mode (cresso_v5.py:230-234)."""
    if freqs.numel() == 0:
        return torch.empty((0,), device=freqs.device, dtype=torch.float32)
    f = freqs.to(torch.float32)
    return base * torch.sqrt(1.0 + (f * f).sum(dim=1))


def count_optimizer_state_elements(optimizer) -> int:
    """cresso_v5.py:529-535."""
    total = 0
    for state in optimizer.state.values():
        for value in state.values():
            if torch.is_tensor(value):
                total += value.numel()
    return int(total)


def theoretical_state_elements(shape: Sequence[int], rank: int, spectral: bool = True, hash_bins: int = 128,
                               hash_tables: int = 2, micro_field_max_size: int = 0, hard_channel_min_size: int = 16,
                               thin_matrix_hard_cutoff: int = 8, thin_matrix_max_width: int = 64,
                               thin_matrix_min_aspect: float = 4.0, thin_matrix_route: str = "scalar") -> int:
    """Persistent state size per tensor (cresso_v5.py:573-609):
    spectral R*ndim + 12R + 3BT (hard channel) + 4, scalar 8, micro 3N + 4."""
    dims = tuple(int(d) for d in shape)
    ndim = len(dims)
    n = 1
    for d in dims:
        n *= d
    if int(micro_field_max_size) > 0 and n <= int(micro_field_max_size) and ndim > 0:
        return int(3 * n + 4)
    spectral = bool(spectral) and not thin_matrix_uses_scalar_route(
        dims, thin_matrix_route, thin_matrix_max_width, thin_matrix_min_aspect)
    if spectral:
        thin = ndim == 2 and int(thin_matrix_hard_cutoff) > 0 and min(dims) <= int(thin_matrix_hard_cutoff)
        hard = n >= int(hard_channel_min_size) and not thin
        return int(int(rank) * ndim + 12 * int(rank) + (3 * int(hash_bins) * int(hash_tables) if hard else 0) + 4)
    return 8


def iter_params(params: Iterable) -> list:
    return list(params)
