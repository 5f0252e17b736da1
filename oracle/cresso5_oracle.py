"""Oracle restatement of the CRESSO5 step (reference ``cresso_v5.py``, PyTorch path).

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this file;
it is the checker the CUDA path is compared against.

Every function cites the reference line range it restates.  Arithmetic follows
the reference operation by operation (same torch ops, same order, same dtypes)
so that on CPU this module reproduces the reference bit for bit; the committed
golden vectors in ``tests/golden`` (made by running the reference itself) pin
that claim.  It runs on any torch device and in float32 or float64, which gives
the tests a float64 "truth" run to measure the float32 noise floor.

Routes: spectral (``cresso_v5.py:945-1353``), scalar (``:1434-1582``) and the
micro field (``micro_field_max_size > 0``, ``:1355-1432``).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
from torch import Tensor

# Defaults of CRESSO5.__init__ (cresso_v5.py:621-681), without the API-only keys.
DEFAULTS: Dict[str, object] = dict(
    lr=2.0e-3, rank=8, max_frequency=5, weight_decay=0.0, energy_power=1.20, dt=0.15,
    impulse_friction=0.18, contact_gain=0.16, restoring=0.62, cubic=0.006, metric_dt=0.09,
    metric_friction=0.22, metric_coupling=0.36, local_sharpness=0.0,
    instant_metric_coupling=0.55, instant_metric_power=1.0, root_channel_mix=0.16,
    echo_mix=0.06, transport_mix=0.18, hash_bins=128, hash_tables=2, hash_decay=0.92,
    hash_impulse_decay=0.78, hash_metric_coupling=0.42, hash_drive_mix=0.22,
    direct_force_mix=0.18, residual_feedback_mix=0.06, micro_field_max_size=0,
    micro_decay=0.94, micro_impulse_decay=0.82, micro_drive_mix=0.35, reservoir_decay=0.95,
    refractory_decay=0.90, refractory_gain=0.55, confidence_decay=0.92, confidence_gain=0.50,
    surprise_gain=0.18, surprise_decay=0.95, prediction_mix=0.16, novelty_mix=0.04,
    warmup_steps=10, surprise_brake=0.18, target_update_rms=1.0, min_gain=0.04, max_gain=6.0,
    drive_clip=4.0, spike_mix=0.25, min_spectral_size=1024, basis_cache_limit_elements=2_000_000,
    hard_channel_min_size=16, thin_matrix_hard_cutoff=8, thin_matrix_max_width=64,
    thin_matrix_min_aspect=4.0, thin_matrix_route="scalar", maximize=False, eps=1e-8,
)


def hparams(**overrides) -> Dict[str, object]:
    hp = dict(DEFAULTS)
    for k, v in overrides.items():
        if k not in hp and k != "cuda_ops":
            raise KeyError(k)
        hp[k] = v
    return hp


# ---------------------------------------------------------------------------
# Integer helpers (bit-exact)
# ---------------------------------------------------------------------------

def hash_unit(n: int, salt: int = 0) -> float:
    """24-bit integer mix mapped to [0, 1).  cresso_v5.py:127-135."""
    x = (int(n) + 1) * 0x9E3779B1 + (int(salt) + 11) * 0x85EBCA77
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return float(x & 0xFFFFFF) / float(1 << 24)


def hash_index_np(n: int, bins: int, salt: int = 0, offset: int = 0) -> np.ndarray:
    """Salted 3-round int64 coordinate hash of flat indices ``offset .. offset+n-1``.

    Restates cresso_v5.py:495-516.  numpy int64 arithmetic wraps like torch's,
    ``>>`` is arithmetic on signed int64 and ``np.remainder`` takes the sign of
    the divisor like ``torch.remainder``.
    """
    bins = int(bins)
    if bins <= 0:
        return np.empty((n,), dtype=np.int64)
    s = int(salt) + 1
    i = np.arange(offset, offset + n, dtype=np.int64)
    with np.errstate(over="ignore"):
        h = i * np.int64(1103515245 + 97 * s) + np.int64(12345 + 0x9E3779B1 * s)
        h = h ^ (h >> np.int64(16))
        h = h * np.int64(_wrap64(2246822519 + 1315423911 * s))
        h = h ^ (h >> np.int64(13))
        h = h * np.int64(_wrap64(3266489917 + 374761393 * s))
        h = h ^ (h >> np.int64(16))
    return np.remainder(h, np.int64(bins))


def _wrap64(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= (1 << 63) else v


def hash_index_tensor(shape: Sequence[int], bins: int, device, salt: int = 0) -> Tensor:
    """Torch form of the coordinate hash, same ops as cresso_v5.py:495-516."""
    bins = int(bins)
    n = 1
    for d in shape:
        n *= int(d)
    if bins <= 0:
        return torch.empty(tuple(shape), device=device, dtype=torch.long)
    i = torch.arange(n, device=device, dtype=torch.long)
    s = int(salt) + 1
    h = i * (1103515245 + 97 * s) + (12345 + 0x9E3779B1 * s)
    h = h ^ (h >> 16)
    h = h * (2246822519 + 1315423911 * s)
    h = h ^ (h >> 13)
    h = h * (3266489917 + 374761393 * s)
    h = h ^ (h >> 16)
    return torch.remainder(h, bins).view(tuple(shape))


def multiscale_frequencies(rank: int, ndim: int, max_frequency: int) -> List[Tuple[int, ...]]:
    """Deterministic frequency pack.  cresso_v5.py:145-227.

    Order: the zero mode, axis-local modes, diagonal / anti-diagonal modes,
    pairwise mixed modes, then hashed modes with an exhaustion guard.
    """
    rank, ndim, maxf = int(rank), int(ndim), max(0, int(max_frequency))
    if rank <= 0:
        return []
    out: List[Tuple[int, ...]] = [tuple([0] * ndim)]
    seen = set(out)

    def push(t: Tuple[int, ...]) -> bool:
        if t not in seen:
            out.append(t)
            seen.add(t)
        return len(out) >= rank

    if maxf <= 0:
        return (out * rank)[:rank] if out else []
    for f in range(1, maxf + 1):
        for axis in range(ndim):
            v = [0] * ndim
            v[axis] = f
            if push(tuple(v)):
                return out[:rank]
    for f in range(1, maxf + 1):
        if push(tuple([f] * ndim)):
            return out[:rank]
        if ndim > 1:
            if push(tuple(f if i % 2 == 0 else max(1, maxf + 1 - f) for i in range(ndim))):
                return out[:rank]
    if ndim > 1:
        for f1 in range(1, maxf + 1):
            for f2 in range(1, maxf + 1):
                for a in range(ndim):
                    v = [0] * ndim
                    v[a] = f1
                    v[(a + 1) % ndim] = f2
                    if push(tuple(v)):
                        return out[:rank]
    primes = [2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37]
    n = 1
    attempts = 0
    guard = max(64, 10 * rank * max(1, ndim))
    while len(out) < rank:
        v = []
        active = 0
        for axis in range(ndim):
            f = (n * primes[axis % len(primes)] + axis * axis + 3 * axis + 1) % (maxf + 1)
            active += int(f != 0)
            v.append(int(f))
        if active == 0:
            v[n % ndim] = 1 + (n % maxf)
        elif active == 1 and ndim > 1:
            v[(n + 1) % ndim] = 1 + ((n // 2) % maxf)
        t = tuple(v)
        if t not in seen or attempts >= guard:
            out.append(t)
            seen.add(t)
        n += 1
        attempts += 1
    return out[:rank]


def freqs_tensor(rank: int, ndim: int, max_frequency: int, device=None) -> Tensor:
    modes = multiscale_frequencies(rank, ndim, max_frequency)
    if not modes:
        return torch.empty((0, ndim), dtype=torch.long, device=device)
    return torch.tensor(modes, dtype=torch.long, device=device)


def omega_from_freqs(freqs: Tensor, base: float = 1.0) -> Tensor:
    """omega = base * sqrt(1 + |f|^2).  cresso_v5.py:230-234."""
    if freqs.numel() == 0:
        return torch.empty((0,), device=freqs.device, dtype=torch.float32)
    f = freqs.to(torch.float32)
    return base * torch.sqrt(1.0 + (f * f).sum(dim=1))


# ---------------------------------------------------------------------------
# Basis (cresso_v5.py:138-376)
# ---------------------------------------------------------------------------

def _normalize_basis(x: Tensor, zero_mean: bool = False) -> Tensor:
    """cresso_v5.py:138-142."""
    if zero_mean:
        x = x - x.mean()
    rms = torch.sqrt(x.pow(2).mean() + 1e-12)
    return x / rms.clamp_min(1e-6)


def _axis_coord(dim: int, device, dtype, centered: bool = False) -> Tensor:
    """cresso_v5.py:237-239."""
    u = (torch.arange(dim, device=device, dtype=dtype) + 0.5) / float(dim)
    return u - 0.5 if centered else u


def _phase(shape, fr: List[int], mode: int, dtype, device, chirp: bool) -> Tensor:
    """Additive (optionally chirped) phase field.  cresso_v5.py:272-292."""
    nd = len(shape)
    phase: Optional[Tensor] = None
    for axis, dim in enumerate(shape):
        f = fr[axis] if fr else 0
        if f == 0 and not chirp:
            continue
        u = _axis_coord(dim, device, dtype)
        comp = math.pi * float(f) * u
        if chirp:
            c = 0.25 + 1.75 * hash_unit(mode, 17 + axis)
            comp = comp + math.pi * c * float(max(1, f)) * (u - 0.5).pow(2)
        view = [1] * nd
        view[axis] = dim
        comp = comp.view(view)
        phase = comp if phase is None else phase + comp
    if phase is None:
        return torch.zeros(shape, device=device, dtype=dtype)
    return phase.expand(shape)


def basis_pair(shape: Sequence[int], freqs: Tensor, mode: int, dtype) -> Tuple[Tensor, Tensor]:
    """Normalised (cos, sin) carrier of one mode.  cresso_v5.py:295-348.

    kind = mode % 4: 0 additive phase, 1 per-axis products, 2 chirped phase,
    3 chirped phase under a separable Gaussian window.  A zero frequency vector
    gives the unnormalised pair (1, 0).
    """
    shape = tuple(int(d) for d in shape)
    device = freqs.device
    fr = [int(v) for v in freqs[mode].tolist()] if freqs.numel() else []
    if sum(abs(v) for v in fr) == 0:
        return torch.ones(shape, device=device, dtype=dtype), torch.zeros(shape, device=device, dtype=dtype)
    kind = mode % 4
    nd = len(shape)
    if kind == 0 or kind == 2:
        ph = _phase(shape, fr, mode, dtype, device, chirp=(kind == 2))
        return _normalize_basis(torch.cos(ph), True), _normalize_basis(torch.sin(ph), True)
    if kind == 1:
        cb: Optional[Tensor] = None
        sb: Optional[Tensor] = None
        for axis, dim in enumerate(shape):
            f = fr[axis]
            if f == 0:
                continue
            u = _axis_coord(dim, device, dtype)
            ph = math.pi * float(f) * u
            view = [1] * nd
            view[axis] = dim
            c = torch.cos(ph).view(view)
            s = torch.sin(ph).view(view)
            cb = c if cb is None else cb * c
            sb = s if sb is None else sb * s
        assert cb is not None and sb is not None
        return _normalize_basis(cb.expand(shape), True), _normalize_basis(sb.expand(shape), True)
    ph = _phase(shape, fr, mode, dtype, device, chirp=True)
    window: Optional[Tensor] = None
    for axis, dim in enumerate(shape):
        u = _axis_coord(dim, device, dtype)
        center = 0.15 + 0.70 * hash_unit(mode, 101 + axis)
        width = 0.18 + 0.20 * hash_unit(mode, 151 + axis)
        w = torch.exp(-0.5 * ((u - center) / width).pow(2))
        view = [1] * nd
        view[axis] = dim
        w = w.view(view)
        window = w if window is None else window * w
    assert window is not None
    window = window.expand(shape)
    return _normalize_basis(window * torch.cos(ph), True), _normalize_basis(window * torch.sin(ph), True)


class BasisSet:
    """All carriers of one (shape, freqs, dtype); built once per step like the
    reference's transient list cache (cresso_v5.py:380-415).  The values do not
    depend on whether the reference cached them."""

    def __init__(self, shape, freqs: Tensor, dtype):
        self.shape = tuple(int(d) for d in shape)
        self.pairs = [basis_pair(self.shape, freqs, r, dtype) for r in range(int(freqs.shape[0]))]

    def project(self, x: Tensor) -> Tuple[Tensor, Tensor]:
        """c_r = mean(x * cos_r), s_r = mean(x * sin_r).  cresso_v5.py:351-359, 438-443."""
        rank = len(self.pairs)
        c = torch.empty(rank, device=x.device, dtype=x.dtype)
        s = torch.empty(rank, device=x.device, dtype=x.dtype)
        for r, (bc, bs) in enumerate(self.pairs):
            c[r] = (x * bc).mean()
            s[r] = (x * bs).mean()
        return c, s

    def reconstruct(self, c: Tensor, s: Tensor, dtype, gates: Optional[Tensor] = None) -> Tensor:
        """shrink * sum_r g_r (c_r cos_r + s_r sin_r).  cresso_v5.py:362-376, 480-491."""
        rank = int(c.numel())
        out = torch.zeros(self.shape, device=c.device, dtype=dtype)
        if rank == 0:
            return out
        shrink = 1.0 / math.sqrt(max(1.0, 0.7 * math.log2(rank + 1.0)))
        for r, (bc, bs) in enumerate(self.pairs):
            g = 1.0 if gates is None else float(gates[r].item())
            if g == 0.0:
                continue
            out.add_(bc, alpha=float(c[r].item()) * shrink * g)
            out.add_(bs, alpha=float(s[r].item()) * shrink * g)
        return out


def project(x: Tensor, freqs: Tensor) -> Tuple[Tensor, Tensor]:
    return BasisSet(tuple(x.shape), freqs, x.dtype).project(x)


def reconstruct(c: Tensor, s: Tensor, freqs: Tensor, shape, dtype, gates: Optional[Tensor] = None) -> Tensor:
    return BasisSet(shape, freqs, dtype).reconstruct(c, s, dtype, gates)


# ---------------------------------------------------------------------------
# Field helpers
# ---------------------------------------------------------------------------

def hash_reduce_mean(x: Tensor, idx: Tensor, bins: int) -> Tensor:
    """Per-bin mean, empty bin -> 0.  cresso_v5.py:519-526."""
    fi = idx.reshape(-1)
    fx = x.reshape(-1)
    out = torch.zeros(int(bins), device=x.device, dtype=x.dtype)
    out.scatter_add_(0, fi, fx)
    cnt = torch.zeros(int(bins), device=x.device, dtype=x.dtype)
    cnt.scatter_add_(0, fi, torch.ones_like(fx, dtype=x.dtype))
    return out / cnt.clamp_min(1.0)


def instant_axis_metric(rel: Tensor, power: float, coupling: float, eps: float) -> Tensor:
    """Stateless axial current metric.  cresso_v5.py:243-262."""
    if coupling == 0.0 or rel.ndim == 0 or rel.numel() <= 1:
        return torch.ones_like(rel)
    nd = rel.ndim
    power = max(float(power), 0.25)
    dens = rel.clamp_min(eps).pow(power).clamp(max=1.0e6)
    acc: Optional[Tensor] = None
    for axis in range(nd):
        red = tuple(i for i in range(nd) if i != axis)
        ax = dens.mean(dim=red, keepdim=True) if red else dens
        ax = ax / ax.mean().clamp_min(eps)
        term = torch.log(ax.clamp_min(eps))
        acc = term if acc is None else acc + term
    assert acc is not None
    return torch.exp((float(coupling) / (nd * power)) * acc).clamp(0.08, 12.0)


def rms_normalize(x: Tensor, target, eps: float) -> Tensor:
    """cresso_v5.py:265-269."""
    rms = torch.sqrt(x.pow(2).mean() + eps)
    if torch.is_tensor(target):
        return x * (target.to(dtype=x.dtype, device=x.device) / rms.clamp_min(eps))
    return x * (float(target) / rms.clamp_min(eps))


def reservoir(old: Tensor, cur: Tensor, decay: float, step: int) -> Tensor:
    """EMA with a copy on the first step; keeps tensor identity.  cresso_v5.py:900-905."""
    if step <= 1:
        old.copy_(cur.detach().to(device=old.device, dtype=old.dtype))
        return old
    old.mul_(float(decay)).add_(cur.detach().to(device=old.device, dtype=old.dtype), alpha=1.0 - float(decay))
    return old


def work_dtype(dtype):
    """cresso_v5.py:119-124 (work and state dtype are the same rule)."""
    return torch.float32 if dtype in (torch.float16, torch.bfloat16) else dtype


# ---------------------------------------------------------------------------
# Routing and state size (cresso_v5.py:529-609, 847-855)
# ---------------------------------------------------------------------------

def is_lora_thin(shape, max_width: int = 64, min_aspect: float = 4.0) -> bool:
    """cresso_v5.py:545-557."""
    dims = tuple(int(d) for d in shape)
    if len(dims) != 2 or int(max_width) <= 0:
        return False
    short, long_ = min(dims), max(dims)
    if short <= 0:
        return False
    return short <= int(max_width) and (long_ / short) >= float(min_aspect)


def thin_uses_scalar(shape, route: str = "scalar", max_width: int = 64, min_aspect: float = 4.0) -> bool:
    """cresso_v5.py:538-570."""
    r = str(route).lower()
    if r not in ("scalar", "spectral"):
        raise ValueError("thin_matrix_route must be one of 'scalar' or 'spectral'")
    return r == "scalar" and is_lora_thin(shape, max_width, min_aspect)


def uses_spectral(shape, hp) -> bool:
    """cresso_v5.py:847-855."""
    n = int(np.prod(shape)) if len(shape) else 1
    if not (n >= int(hp["min_spectral_size"]) and int(hp["rank"]) > 0 and len(shape) > 0):
        return False
    return not thin_uses_scalar(shape, hp["thin_matrix_route"], hp["thin_matrix_max_width"], hp["thin_matrix_min_aspect"])


def count_state_elements(states: Dict) -> int:
    """cresso_v5.py:529-535."""
    return int(sum(v.numel() for st in states.values() for v in st.values() if torch.is_tensor(v)))


def theoretical_state_elements(shape, rank, spectral=True, hash_bins=128, hash_tables=2,
                               micro_field_max_size=0, hard_channel_min_size=16,
                               thin_matrix_hard_cutoff=8, thin_matrix_max_width=64,
                               thin_matrix_min_aspect=4.0, thin_matrix_route="scalar") -> int:
    """cresso_v5.py:573-609."""
    dims = tuple(int(d) for d in shape)
    nd = len(dims)
    n = int(np.prod(dims)) if dims else 1
    if int(micro_field_max_size) > 0 and n <= int(micro_field_max_size) and nd > 0:
        return 3 * n + 4
    spectral = bool(spectral) and not thin_uses_scalar(dims, thin_matrix_route, thin_matrix_max_width, thin_matrix_min_aspect)
    if spectral:
        thin = nd == 2 and int(thin_matrix_hard_cutoff) > 0 and min(dims) <= int(thin_matrix_hard_cutoff)
        hard = n >= int(hard_channel_min_size) and not thin
        return int(rank) * nd + 12 * int(rank) + (3 * int(hash_bins) * int(hash_tables) if hard else 0) + 4
    return 8


# ---------------------------------------------------------------------------
# State creation (cresso_v5.py:857-891)
# ---------------------------------------------------------------------------

def init_common(device, dtype) -> Dict:
    return dict(step=0,
                force_rms=torch.zeros((), device=device, dtype=dtype),
                drive_energy=torch.ones((), device=device, dtype=dtype),
                surprise=torch.zeros((), device=device, dtype=dtype),
                action=torch.zeros((), device=device, dtype=dtype))


def init_spectral(param: Tensor, hp, dtype) -> Dict:
    st = init_common(param.device, dtype)
    rank = int(hp["rank"])
    freqs = freqs_tensor(rank, param.ndim, int(hp["max_frequency"]), param.device)
    st["freqs"] = freqs
    st["omega"] = omega_from_freqs(freqs).to(device=param.device, dtype=dtype)
    for name in ("q_cos", "q_sin", "p_cos", "p_sin", "metric_cos", "metric_sin",
                 "metric_p_cos", "metric_p_sin", "calcium_cos", "calcium_sin", "mode_confidence"):
        st[name] = torch.zeros(rank, device=param.device, dtype=dtype)
    bins = int(hp["hash_bins"])
    tables = int(hp["hash_tables"])
    cutoff = int(hp["thin_matrix_hard_cutoff"])
    thin = param.ndim == 2 and cutoff > 0 and min(param.shape) <= cutoff
    if bins > 0 and param.numel() >= int(hp["hard_channel_min_size"]) and not thin:
        st["hash_energy"] = torch.ones(tables, bins, device=param.device, dtype=dtype)
        st["hash_impulse"] = torch.zeros(tables, bins, device=param.device, dtype=dtype)
        st["hash_refractory"] = torch.zeros(tables, bins, device=param.device, dtype=dtype)
    return st


def init_micro(param: Tensor, dtype) -> Dict:
    """Per-element energy / impulse / refractory fields.  cresso_v5.py:893-898."""
    st = init_common(param.device, dtype)
    st["micro_energy"] = torch.ones_like(param.detach(), dtype=dtype, memory_format=torch.preserve_format)
    st["micro_impulse"] = torch.zeros_like(param.detach(), dtype=dtype, memory_format=torch.preserve_format)
    st["micro_refractory"] = torch.zeros_like(param.detach(), dtype=dtype, memory_format=torch.preserve_format)
    return st


def init_scalar(param: Tensor, dtype) -> Dict:
    st = init_common(param.device, dtype)
    for name in ("q", "impulse", "metric_q", "metric_impulse"):
        st[name] = torch.zeros((), device=param.device, dtype=dtype)
    return st


def base_force(param: Tensor, grad: Tensor, hp, dtype) -> Tensor:
    """f = g (+ wd p).  cresso_v5.py:907-912."""
    f = grad.to(dtype=dtype)
    wd = float(hp["weight_decay"])
    if wd != 0.0:
        f = f + wd * param.detach().to(dtype=dtype)
    return f


def contact_update_pair(q, p, port, omega, calcium, action, surprise, hp, rank):
    """Refractory contact oscillator half-update.  cresso_v5.py:914-943."""
    dt = float(hp["dt"])
    rd = float(hp["refractory_decay"])
    calcium.mul_(rd).add_(port.abs(), alpha=1.0 - rd)
    rgate = 1.0 / (1.0 + float(hp["refractory_gain"]) * calcium)
    s = surprise.to(q.dtype)
    plasticity = 1.0 + float(hp["surprise_gain"]) * s / (1.0 + s)
    brake = 1.0 / (1.0 + float(hp["surprise_brake"]) * s)
    gp = port * rgate * plasticity * brake
    energy = 0.5 * (p.pow(2).mean() + ((omega * q).pow(2)).mean()) if rank > 0 else torch.zeros_like(action)
    port_power = (gp * p).mean() if rank > 0 else torch.zeros_like(action)
    action.mul_(0.985).add_((port_power - energy).to(action.dtype), alpha=dt)
    friction = float(hp["impulse_friction"]) + float(hp["contact_gain"]) * torch.tanh(action.abs()).to(p.dtype)
    p.mul_(torch.clamp(1.0 - dt * friction, min=0.0))
    p.add_(gp - float(hp["restoring"]) * (omega * omega) * q - float(hp["cubic"]) * q.pow(3), alpha=dt)
    q.add_(p, alpha=dt)
    q.clamp_(-8.0, 8.0)
    return action


# ---------------------------------------------------------------------------
# Spectral step (cresso_v5.py:945-1353)
# ---------------------------------------------------------------------------

def spectral_step(param: Tensor, grad: Tensor, st: Dict, hp) -> None:
    dtype = work_dtype(param.dtype)
    if len(st) == 0:
        st.update(init_spectral(param, hp, work_dtype(dtype)))
    st["step"] += 1
    step = int(st["step"])
    eps = float(hp["eps"])

    force = base_force(param, grad, hp, dtype)
    frn = torch.sqrt(force.pow(2).mean() + eps)
    st["force_rms"] = reservoir(st["force_rms"], frn, hp["reservoir_decay"], step)
    scale = st["force_rms"].to(dtype).clamp_min(eps)

    freqs = st["freqs"]
    rank = int(st["omega"].numel())
    omega = st["omega"].to(dtype=st["q_cos"].dtype)
    basis = BasisSet(tuple(param.shape), freqs, dtype)
    cutoff = int(hp["thin_matrix_hard_cutoff"])
    thin = param.ndim == 2 and cutoff > 0 and min(param.shape) <= cutoff
    hard = param.numel() >= int(hp["hard_channel_min_size"]) and not thin

    rel = (force.abs() / scale + eps).clamp(max=1.0e4)
    bins = int(hp["hash_bins"])
    tables = int(hp["hash_tables"])
    hash_idx: Optional[List[Tensor]] = None
    hash_metric = 1.0
    hash_pred = 0.0
    ds: Optional[Tensor] = None
    if hard and bins > 0 and "hash_energy" in st:
        # Multi-table hash metric (cresso_v5.py:995-1056).
        hash_idx = []
        logsum: Optional[Tensor] = None
        ds = rel.pow(float(hp["energy_power"]))
        for t in range(tables):
            idx = hash_index_tensor(tuple(param.shape), bins, param.device, salt=t)
            hash_idx.append(idx)
            cell = hash_reduce_mean(ds, idx, bins)
            e = st["hash_energy"][t]
            if step <= 1:
                e.copy_(cell.to(e.dtype))
            else:
                e.mul_(float(hp["hash_decay"])).add_(cell.to(e.dtype), alpha=1.0 - float(hp["hash_decay"]))
            hm = (e.to(dtype) / e.to(dtype).mean().clamp_min(eps)).clamp_min(eps)
            hmp = hm.pow(float(hp["hash_metric_coupling"]) / max(0.25, float(hp["energy_power"])))
            term = torch.log(hmp[idx].clamp(0.08, 12.0).clamp_min(eps))
            logsum = term if logsum is None else logsum + term
        assert logsum is not None
        hash_metric = torch.exp(logsum / float(tables)).clamp(0.08, 12.0)
    if ds is None:
        ds = rel.pow(float(hp["energy_power"]))
    density = torch.log1p(ds)
    density = density / density.mean().clamp_min(eps) - 1.0

    # Spectral metric oscillator (cresso_v5.py:1061-1093).
    mc_port, ms_port = basis.project(density)
    mc_port = mc_port.to(st["metric_cos"].dtype)
    ms_port = ms_port.to(st["metric_sin"].dtype)
    mdt = float(hp["metric_dt"])
    mf = float(hp["metric_friction"])
    for qn, pn, port in (("metric_cos", "metric_p_cos", mc_port), ("metric_sin", "metric_p_sin", ms_port)):
        mq, mp = st[qn], st[pn]
        mp.mul_(max(0.0, 1.0 - mdt * mf))
        mp.add_(port - (omega * omega) * mq, alpha=mdt)
        mq.add_(mp, alpha=mdt)
        mq.clamp_(-3.0, 3.0)
    log_metric = basis.reconstruct(st["metric_cos"].to(dtype), st["metric_sin"].to(dtype), dtype).clamp(-3.0, 3.0)
    metric = torch.exp(float(hp["metric_coupling"]) * log_metric).clamp(0.06, 16.0)

    # Local and instant metrics, tangent force (cresso_v5.py:1095-1123).
    ls = float(hp["local_sharpness"])
    local = (1.0 + ls * torch.sqrt(rel.clamp(max=100.0))).clamp(1.0, 8.0) if ls != 0.0 else 1.0
    ic = float(hp["instant_metric_coupling"]) if hard else 0.0
    instant = instant_axis_metric(rel, float(hp["instant_metric_power"]), ic, eps)
    tangent = (force / (scale * metric * local * instant * hash_metric + eps)).clamp(-1.0e4, 1.0e4)

    # Prediction, surprise, port projection (cresso_v5.py:1125-1138).
    qc, qs, conf = st["q_cos"], st["q_sin"], st["mode_confidence"]
    gates = torch.sigmoid(float(hp["confidence_gain"]) * conf).to(dtype)
    pred = basis.reconstruct(qc.to(dtype), qs.to(dtype), dtype, gates=gates)
    error = tangent - pred
    sn = torch.sqrt(error.pow(2).mean() + eps)
    st["surprise"] = reservoir(st["surprise"], sn, hp["surprise_decay"], step)
    surprise = st["surprise"]
    port_src = error + float(hp["transport_mix"]) * tangent
    pc, ps = basis.project(port_src)
    pc = pc.to(qc.dtype)
    ps = ps.to(qs.dtype)

    # Hash impulse reservoirs (cresso_v5.py:1140-1184).
    if hash_idx is not None and "hash_impulse" in st:
        acc: Optional[Tensor] = None
        for t, idx in enumerate(hash_idx):
            cell = hash_reduce_mean(port_src, idx, bins).to(st["hash_impulse"].dtype)
            href = st["hash_refractory"][t]
            himp = st["hash_impulse"][t]
            href.mul_(float(hp["hash_decay"])).add_(cell.abs(), alpha=1.0 - float(hp["hash_decay"]))
            hg = 1.0 / (1.0 + float(hp["refractory_gain"]) * href)
            himp.mul_(float(hp["hash_impulse_decay"])).add_(cell * hg, alpha=1.0 - float(hp["hash_impulse_decay"]))
            got = himp.to(dtype)[idx]
            acc = got if acc is None else acc + got
        assert acc is not None
        hash_pred = acc / float(len(hash_idx))

    # Confidence (cresso_v5.py:1186-1202).
    pe = torch.sqrt(pc.pow(2) + ps.pow(2) + eps)
    support = (pc * qc + ps * qs) / (pe * torch.sqrt(qc.pow(2) + qs.pow(2) + eps) + eps)
    cd = float(hp["confidence_decay"])
    conf.mul_(cd).add_(support.clamp(-1.0, 1.0), alpha=1.0 - cd)
    conf.clamp_(-4.0, 4.0)

    # Contact oscillators, cos half then sin half (cresso_v5.py:1204-1250).
    action = st["action"]
    action = contact_update_pair(qc, st["p_cos"], pc, omega, st["calcium_cos"], action, surprise, hp, rank)
    st["action"] = contact_update_pair(qs, st["p_sin"], ps, omega, st["calcium_sin"], action, surprise, hp, rank)

    # Second prediction and echo (cresso_v5.py:1252-1258).
    gates = torch.sigmoid(float(hp["confidence_gain"]) * conf).to(dtype)
    pred = basis.reconstruct(qc.to(dtype), qs.to(dtype), dtype, gates=gates)
    error = tangent - pred
    echo_raw: Optional[Tensor] = None
    if hard and float(hp["echo_mix"]) != 0.0:
        ec, es = basis.project(tangent)
        echo_raw = basis.reconstruct(ec, es, dtype)

    # Drive shaping and update (cresso_v5.py:1303-1353).
    _drive_and_apply(param, tangent, pred, error, echo_raw, hash_pred, hard, st, hp, step, dtype, spectral=True)


def _drive_and_apply(param, tangent, pred, error, echo_raw, hash_pred, hard, st, hp, step, dtype, spectral):
    eps = float(hp["eps"])
    frms = torch.sqrt(tangent.pow(2).mean() + eps)
    prms = torch.sqrt(pred.pow(2).mean() + eps)
    align = ((tangent * pred).mean() / (frms * prms + eps)).clamp(-1.0, 1.0)
    align_gate = torch.where(prms > math.sqrt(eps), ((align + 1.0) * 0.5).clamp(0.0, 1.0),
                             torch.zeros((), device=param.device, dtype=dtype))
    ws = int(hp["warmup_steps"])
    warm = 1.0 if ws == 0 else (1.0 - math.exp(-step / max(1, ws)))
    s = st["surprise"].to(dtype)
    if spectral:
        mix = float(hp["prediction_mix"]) * warm * align_gate * (1.0 / (1.0 + s))
    else:
        mix = float(hp["prediction_mix"]) * warm * align_gate / (1.0 + s)
    clip = float(hp["drive_clip"])
    bounded = torch.tanh(tangent / clip) * clip
    rational = tangent / (1.0 + tangent.abs() / clip)
    root = tangent.sign() * torch.sqrt(tangent.abs().clamp(max=clip * clip) + eps)
    root = rms_normalize(root, torch.sqrt(rational.pow(2).mean() + eps), eps)
    spike = float(hp["spike_mix"]) / (1.0 + s)
    base = (1.0 - spike) * rational + spike * bounded
    if spectral:
        root_mix = (float(hp["root_channel_mix"]) if hard else 0.0) / (1.0 + 0.5 * s)
    else:
        root_mix = float(hp["root_channel_mix"]) / (1.0 + 0.5 * s)
    shaped = (1.0 - root_mix) * base + root_mix * root
    novelty = torch.tanh(error / (clip * (1.0 + st["surprise"].to(dtype)))) * clip
    direct_mix = float(hp["direct_force_mix"]) / (1.0 + 0.35 * s)
    if spectral:
        shaped_rms = torch.sqrt(shaped.pow(2).mean() + eps)
        if hard and float(hp["echo_mix"]) != 0.0:
            echo = rms_normalize(echo_raw, shaped_rms, eps)
        else:
            echo = 0.0
        if torch.is_tensor(hash_pred):
            hash_pred = rms_normalize(hash_pred, shaped_rms, eps)
        direct = tangent * (shaped_rms / frms.clamp_min(eps))
    else:
        direct = rms_normalize(tangent, torch.sqrt(shaped.pow(2).mean() + eps), eps)
    core = (1.0 - direct_mix) * shaped + direct_mix * direct
    residual_mix = float(hp["residual_feedback_mix"]) / (1.0 + s)
    residual = rms_normalize(error, torch.sqrt(core.pow(2).mean() + eps), eps)
    if spectral:
        drive = ((1.0 - mix) * core + mix * pred + float(hp["novelty_mix"]) * novelty
                 + residual_mix * residual
                 + (float(hp["echo_mix"]) if hard else 0.0) * echo
                 + (float(hp["hash_drive_mix"]) if hard else 0.0) * hash_pred)
    else:
        drive = (1.0 - mix) * core + mix * pred + float(hp["novelty_mix"]) * novelty + residual_mix * residual
    den = drive.pow(2).mean().to(st["drive_energy"].dtype)
    st["drive_energy"] = reservoir(st["drive_energy"], den, hp["reservoir_decay"], step)
    gain = (float(hp["target_update_rms"]) / torch.sqrt(st["drive_energy"].to(dtype) + eps)).clamp(
        float(hp["min_gain"]), float(hp["max_gain"]))
    param.add_((drive * gain).to(dtype=param.dtype), alpha=-float(hp["lr"]))


# ---------------------------------------------------------------------------
# Thin / small tensor scalar route (cresso_v5.py:1434-1582, torch branch 1505-1582)
# ---------------------------------------------------------------------------

def scalar_step(param: Tensor, grad: Tensor, st: Dict, hp) -> None:
    dtype = work_dtype(param.dtype)
    if len(st) == 0:
        st.update(init_scalar(param, work_dtype(dtype)))
    st["step"] += 1
    step = int(st["step"])
    eps = float(hp["eps"])
    force = base_force(param, grad, hp, dtype)
    frn = torch.sqrt(force.pow(2).mean() + eps)
    st["force_rms"] = reservoir(st["force_rms"], frn, hp["reservoir_decay"], step)
    scale = st["force_rms"].to(dtype).clamp_min(eps)

    density = torch.log1p((force.abs() / scale + eps).pow(float(hp["energy_power"]))).mean()
    mport = (density - st["metric_q"].to(dtype).tanh()).to(st["metric_q"].dtype)
    mdt = float(hp["metric_dt"])
    mq, mp = st["metric_q"], st["metric_impulse"]
    mp.mul_(max(0.0, 1.0 - mdt * float(hp["metric_friction"])))
    mp.add_(mport - mq, alpha=mdt)
    mq.add_(mp, alpha=mdt)
    mq.clamp_(-3.0, 3.0)
    metric = torch.exp(float(hp["metric_coupling"]) * mq.to(dtype)).clamp(0.06, 16.0)
    rel = (force.abs() / scale + eps).clamp(max=1.0e4)
    ls = float(hp["local_sharpness"])
    local = (1.0 + ls * torch.sqrt(rel.clamp(max=100.0))).clamp(1.0, 8.0) if ls != 0.0 else 1.0
    instant = instant_axis_metric(rel, float(hp["instant_metric_power"]), float(hp["instant_metric_coupling"]), eps)
    tangent = (force / (scale * metric * local * instant + eps)).clamp(-1.0e4, 1.0e4)

    q, imp = st["q"], st["impulse"]
    pred = q.to(dtype).expand_as(tangent)
    error = tangent - pred
    sn = torch.sqrt(error.pow(2).mean() + eps)
    st["surprise"] = reservoir(st["surprise"], sn, hp["surprise_decay"], step)
    port = error.mean().to(q.dtype)
    dt = float(hp["dt"])
    s = st["surprise"].to(q.dtype)
    plasticity = 1.0 + float(hp["surprise_gain"]) * s / (1.0 + s)
    brake = 1.0 / (1.0 + float(hp["surprise_brake"]) * s)
    action = st["action"]
    energy = 0.5 * (imp.pow(2) + q.pow(2))
    action.mul_(0.985).add_((port * imp - energy).to(action.dtype), alpha=dt)
    friction = float(hp["impulse_friction"]) + float(hp["contact_gain"]) * torch.tanh(action.abs()).to(imp.dtype)
    imp.mul_(torch.clamp(1.0 - dt * friction, min=0.0))
    imp.add_(plasticity * brake * port - float(hp["restoring"]) * q - float(hp["cubic"]) * q.pow(3), alpha=dt)
    q.add_(imp, alpha=dt)
    q.clamp_(-8.0, 8.0)

    pred = q.to(dtype).expand_as(tangent)
    error = tangent - pred
    _drive_and_apply(param, tangent, pred, error, None, 0.0, False, st, hp, step, dtype, spectral=False)


# ---------------------------------------------------------------------------
# Micro-field route for small tensors (cresso_v5.py:1355-1432)
# ---------------------------------------------------------------------------

def micro_step(param: Tensor, grad: Tensor, st: Dict, hp) -> None:
    dtype = work_dtype(param.dtype)
    if len(st) == 0:
        st.update(init_micro(param, work_dtype(dtype)))
    st["step"] += 1
    step = int(st["step"])
    eps = float(hp["eps"])
    force = base_force(param, grad, hp, dtype)
    frn = torch.sqrt(force.pow(2).mean() + eps)
    st["force_rms"] = reservoir(st["force_rms"], frn, hp["reservoir_decay"], step)
    scale = st["force_rms"].to(dtype).clamp_min(eps)
    rel = (force.abs() / scale + eps).clamp(max=1.0e4)

    # energy field and its metric (cresso_v5.py:1380-1392)
    e, imp, ref = st["micro_energy"], st["micro_impulse"], st["micro_refractory"]
    density = rel.pow(float(hp["energy_power"]))
    if step <= 1:
        e.copy_(density.to(e.dtype))
    else:
        e.mul_(float(hp["micro_decay"])).add_(density.to(e.dtype), alpha=1.0 - float(hp["micro_decay"]))
    expo = float(hp["hash_metric_coupling"]) / max(0.25, float(hp["energy_power"]))
    metric = (e.to(dtype) / e.to(dtype).mean().clamp_min(eps)).pow(expo).clamp(0.08, 12.0)
    instant = instant_axis_metric(rel, float(hp["instant_metric_power"]),
                                  min(0.35, float(hp["instant_metric_coupling"])), eps)
    tangent = (force / (scale * metric * instant + eps)).clamp(-1.0e4, 1.0e4)

    # refractory-gated impulse, prediction, surprise (cresso_v5.py:1394-1404)
    ref.mul_(float(hp["refractory_decay"])).add_(tangent.abs().to(ref.dtype), alpha=1.0 - float(hp["refractory_decay"]))
    gate = 1.0 / (1.0 + float(hp["refractory_gain"]) * ref.to(dtype))
    port = tangent * gate
    imp.mul_(float(hp["micro_impulse_decay"])).add_(port.to(imp.dtype), alpha=1.0 - float(hp["micro_impulse_decay"]))
    pred = imp.to(dtype)
    error = tangent - pred
    sn = torch.sqrt(error.pow(2).mean() + eps)
    st["surprise"] = reservoir(st["surprise"], sn, hp["surprise_decay"], step)

    # drive and update (cresso_v5.py:1406-1432)
    clip = float(hp["drive_clip"])
    bounded = torch.tanh(tangent / clip) * clip
    rational = tangent / (1.0 + tangent.abs() / clip)
    s = st["surprise"].to(dtype)
    spike = float(hp["spike_mix"]) / (1.0 + s)
    shaped = (1.0 - spike) * rational + spike * bounded
    pred_norm = rms_normalize(pred, torch.sqrt(shaped.pow(2).mean() + eps), eps)
    direct_mix = float(hp["direct_force_mix"]) / (1.0 + 0.35 * s)
    micro_mix = float(hp["micro_drive_mix"]) / (1.0 + 0.25 * s)
    residual_mix = float(hp["residual_feedback_mix"]) / (1.0 + s)
    direct = rms_normalize(tangent, torch.sqrt(shaped.pow(2).mean() + eps), eps)
    residual = rms_normalize(error, torch.sqrt(shaped.pow(2).mean() + eps), eps)
    core = (1.0 - direct_mix - 0.5 * micro_mix).clamp(0.0, 1.0)
    drive = core * shaped + direct_mix * direct + micro_mix * pred_norm + residual_mix * residual
    den = drive.pow(2).mean().to(st["drive_energy"].dtype)
    st["drive_energy"] = reservoir(st["drive_energy"], den, hp["reservoir_decay"], step)
    gain = (float(hp["target_update_rms"]) / torch.sqrt(st["drive_energy"].to(dtype) + eps)).clamp(
        float(hp["min_gain"]), float(hp["max_gain"]))
    param.add_((drive * gain).to(dtype=param.dtype), alpha=-float(hp["lr"]))


# ---------------------------------------------------------------------------
# Optimizer-shaped driver
# ---------------------------------------------------------------------------

class OracleCRESSO5:
    """Minimal driver with the reference's per-parameter loop (cresso_v5.py:821-845).

    ``state`` maps each parameter to a dict with the reference's keys.
    """

    def __init__(self, params, **kwargs):
        self.params = list(params)
        self.hp = hparams(**{k: v for k, v in kwargs.items() if k != "cuda_ops"})
        self.state: Dict[Tensor, Dict] = {}

    @torch.no_grad()
    def step(self):
        for p in self.params:
            if p.grad is None or not torch.is_floating_point(p):
                continue
            g = p.grad.detach()
            if self.hp["maximize"]:
                g = -g
            st = self.state.setdefault(p, {})
            if int(self.hp["micro_field_max_size"]) > 0 and p.ndim > 0 and p.numel() <= int(self.hp["micro_field_max_size"]):
                micro_step(p, g, st, self.hp)
            elif uses_spectral(tuple(p.shape), self.hp):
                spectral_step(p, g, st, self.hp)
            else:
                scalar_step(p, g, st, self.hp)
