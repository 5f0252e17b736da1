"""CRESSO5 on B200: the drop-in optimizer class.

``CRESSO5`` keeps the reference API of ``cresso_v5.CRESSO5``
(cresso_v5.py:612-1585): the same constructor keywords, validation and
``param_groups`` keys, ``step(closure=None)``, the persistent state layout
(keys, shapes, dtypes; cresso_v5.py:857-891) and therefore
``state_dict()`` / ``load_state_dict()`` compatibility in both directions.

The step itself runs as fused sm_100a CUDA kernels through the C ABI of
``libcresso_b200.so``: per parameter group and device, all spectral-route
tensors go through one grouped five-pass step and all scalar-route tensors
through one grouped launch.  There is no PyTorch fallback: ``cuda_ops`` accepts
``"auto"`` / ``"required"`` / ``True`` and always means required; ``"off"`` /
``False`` raise ``ValueError`` (the reference PyTorch path lives in the
reference package).
"""

from __future__ import annotations

from typing import Callable, Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch
from torch import Tensor
from torch.optim import Optimizer

from . import _lib
from ._host import (
    count_optimizer_state_elements,
    frequencies_tensor,
    hard_enabled,
    multiscale_frequencies,
    normalize_thin_matrix_route,
    omega_from_freqs,
    theoretical_state_elements,
    uses_spectral_route,
    validate_scalar,
)

__all__ = ["CRESSO5", "CRESSO", "count_optimizer_state_elements", "theoretical_state_elements"]

# parameter element types of the CUDA path and their descriptor codes; the work and the
# state are float32 for all three (cresso_v5.py:119-124)
_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}

_SPECTRAL_RANK_STATE = ("q_cos", "q_sin", "p_cos", "p_sin", "metric_cos", "metric_sin", "metric_p_cos",
                        "metric_p_sin", "calcium_cos", "calcium_sin", "mode_confidence")


def _items_ident(items: list) -> tuple:
    """What a cached descriptor table depends on: the parameter objects, their
    storage addresses and their state dicts (the cache entry holds references to
    all of them, so no id can be reused while it lives)."""
    ps = [it[0] for it in items]
    return tuple(map(id, ps)), tuple([p.data_ptr() for p in ps]), tuple([id(it[2]) for it in items])


class CRESSO5(Optimizer):
    """Contact-Refractory Axial-Spectral Optimizer (B200-native step).

    Large tensors evolve a compact contact-dissipative multiwave state
    (rank-R spectral oscillators, T x B hash-cell reservoirs, four scalars);
    LoRA-thin and small tensors use the scalar contact route, and with
    ``micro_field_max_size > 0`` tensors up to that size keep per-element
    micro fields.  Parameters may be float32, float16, bfloat16 (float32 work
    and state) or float64 (float64 work and state), on CUDA devices only.

    The state tensors are updated in place, and the descriptor tables that point
    the kernels at them are cached across steps (keyed on the parameters, their
    storage addresses and their state dicts).  Change state through
    ``load_state_dict`` (which drops the caches) or in place; a caller that
    rebinds a state tensor inside a state dict (``opt.state[p]["q_cos"] = t``),
    or gives a parameter a new shape over the same storage, calls
    ``invalidate_caches()`` afterwards.
    """

    def __init__(
        self,
        params: Iterable[Tensor],
        lr: float = 2.0e-3,
        rank: int = 8,
        max_frequency: int = 5,
        weight_decay: float = 0.0,
        energy_power: float = 1.20,
        dt: float = 0.15,
        impulse_friction: float = 0.18,
        contact_gain: float = 0.16,
        restoring: float = 0.62,
        cubic: float = 0.006,
        metric_dt: float = 0.09,
        metric_friction: float = 0.22,
        metric_coupling: float = 0.36,
        local_sharpness: float = 0.0,
        instant_metric_coupling: float = 0.55,
        instant_metric_power: float = 1.0,
        root_channel_mix: float = 0.16,
        echo_mix: float = 0.06,
        transport_mix: float = 0.18,
        hash_bins: int = 128,
        hash_tables: int = 2,
        hash_decay: float = 0.92,
        hash_impulse_decay: float = 0.78,
        hash_metric_coupling: float = 0.42,
        hash_drive_mix: float = 0.22,
        direct_force_mix: float = 0.18,
        residual_feedback_mix: float = 0.06,
        micro_field_max_size: int = 0,
        micro_decay: float = 0.94,
        micro_impulse_decay: float = 0.82,
        micro_drive_mix: float = 0.35,
        reservoir_decay: float = 0.95,
        refractory_decay: float = 0.90,
        refractory_gain: float = 0.55,
        confidence_decay: float = 0.92,
        confidence_gain: float = 0.50,
        surprise_gain: float = 0.18,
        surprise_decay: float = 0.95,
        prediction_mix: float = 0.16,
        novelty_mix: float = 0.04,
        warmup_steps: int = 10,
        surprise_brake: float = 0.18,
        target_update_rms: float = 1.0,
        min_gain: float = 0.04,
        max_gain: float = 6.0,
        drive_clip: float = 4.0,
        spike_mix: float = 0.25,
        min_spectral_size: int = 1024,
        basis_cache_limit_elements: int = 2_000_000,
        cuda_ops: str | bool = "auto",
        hard_channel_min_size: int = 16,
        thin_matrix_hard_cutoff: int = 8,
        thin_matrix_max_width: int = 64,
        thin_matrix_min_aspect: float = 4.0,
        thin_matrix_route: str = "scalar",
        maximize: bool = False,
        eps: float = 1e-8,
    ) -> None:
        # Validation of cresso_v5.py:682-758.
        for name, value, lower, upper in [
            ("lr", lr, 0.0, None), ("weight_decay", weight_decay, 0.0, None),
            ("energy_power", energy_power, 0.25, None), ("dt", dt, 0.0, 1.0),
            ("impulse_friction", impulse_friction, 0.0, None), ("contact_gain", contact_gain, 0.0, None),
            ("restoring", restoring, 0.0, None), ("cubic", cubic, 0.0, None), ("metric_dt", metric_dt, 0.0, 1.0),
            ("metric_friction", metric_friction, 0.0, None), ("metric_coupling", metric_coupling, 0.0, None),
            ("local_sharpness", local_sharpness, 0.0, None),
            ("instant_metric_coupling", instant_metric_coupling, 0.0, None),
            ("instant_metric_power", instant_metric_power, 0.25, None),
            ("root_channel_mix", root_channel_mix, 0.0, 1.0), ("echo_mix", echo_mix, 0.0, 1.0),
            ("transport_mix", transport_mix, 0.0, 1.0), ("hash_decay", hash_decay, 0.0, 1.0),
            ("hash_impulse_decay", hash_impulse_decay, 0.0, 1.0),
            ("hash_metric_coupling", hash_metric_coupling, 0.0, None), ("hash_drive_mix", hash_drive_mix, 0.0, 1.0),
            ("direct_force_mix", direct_force_mix, 0.0, 1.0),
            ("residual_feedback_mix", residual_feedback_mix, 0.0, 1.0), ("micro_decay", micro_decay, 0.0, 1.0),
            ("micro_impulse_decay", micro_impulse_decay, 0.0, 1.0), ("micro_drive_mix", micro_drive_mix, 0.0, 1.0),
            ("reservoir_decay", reservoir_decay, 0.0, 1.0), ("refractory_decay", refractory_decay, 0.0, 1.0),
            ("refractory_gain", refractory_gain, 0.0, None), ("confidence_decay", confidence_decay, 0.0, 1.0),
            ("confidence_gain", confidence_gain, 0.0, None), ("surprise_gain", surprise_gain, 0.0, None),
            ("surprise_decay", surprise_decay, 0.0, 1.0), ("prediction_mix", prediction_mix, 0.0, 1.0),
            ("novelty_mix", novelty_mix, 0.0, 1.0), ("surprise_brake", surprise_brake, 0.0, None),
            ("target_update_rms", target_update_rms, 0.0, None), ("min_gain", min_gain, 0.0, None),
            ("max_gain", max_gain, 0.0, None), ("drive_clip", drive_clip, 0.1, None),
            ("spike_mix", spike_mix, 0.0, 1.0), ("eps", eps, 0.0, None),
        ]:
            validate_scalar(name, value, lower, upper)
        if int(rank) < 0:
            raise ValueError("rank must be non-negative")
        if int(max_frequency) < 0:
            raise ValueError("max_frequency must be non-negative")
        if int(hash_bins) < 0:
            raise ValueError("hash_bins must be non-negative")
        if int(hash_tables) < 1:
            raise ValueError("hash_tables must be >= 1")
        if int(min_spectral_size) < 1:
            raise ValueError("min_spectral_size must be >= 1")
        if int(micro_field_max_size) < 0:
            raise ValueError("micro_field_max_size must be >= 0")
        if int(basis_cache_limit_elements) < 0:
            raise ValueError("basis_cache_limit_elements must be >= 0")
        if int(hard_channel_min_size) < 0:
            raise ValueError("hard_channel_min_size must be >= 0")
        if int(thin_matrix_hard_cutoff) < 0:
            raise ValueError("thin_matrix_hard_cutoff must be >= 0")
        if int(thin_matrix_max_width) < 0:
            raise ValueError("thin_matrix_max_width must be >= 0")
        validate_scalar("thin_matrix_min_aspect", thin_matrix_min_aspect, 1.0, None)
        if int(warmup_steps) < 0:
            raise ValueError("warmup_steps must be non-negative")
        if min_gain > max_gain:
            raise ValueError("min_gain must be <= max_gain")
        route = normalize_thin_matrix_route(thin_matrix_route)
        mode = ("auto" if cuda_ops else "off") if isinstance(cuda_ops, bool) else str(cuda_ops).lower()
        if mode not in {"auto", "required", "off"}:
            raise ValueError("cuda_ops must be one of 'auto', 'required', or 'off'")
        if mode == "off":
            raise ValueError(
                "cresso_b200.CRESSO5 runs only the fused CUDA path; cuda_ops='off' selects the reference "
                "PyTorch implementation (cresso_v5.CRESSO5), which this package does not contain")
        defaults = dict(
            lr=float(lr), rank=int(rank), max_frequency=int(max_frequency), weight_decay=float(weight_decay),
            energy_power=float(energy_power), dt=float(dt), impulse_friction=float(impulse_friction),
            contact_gain=float(contact_gain), restoring=float(restoring), cubic=float(cubic),
            metric_dt=float(metric_dt), metric_friction=float(metric_friction),
            metric_coupling=float(metric_coupling), local_sharpness=float(local_sharpness),
            instant_metric_coupling=float(instant_metric_coupling),
            instant_metric_power=float(instant_metric_power), root_channel_mix=float(root_channel_mix),
            echo_mix=float(echo_mix), transport_mix=float(transport_mix), hash_bins=int(hash_bins),
            hash_tables=int(hash_tables), hash_decay=float(hash_decay),
            hash_impulse_decay=float(hash_impulse_decay), hash_metric_coupling=float(hash_metric_coupling),
            hash_drive_mix=float(hash_drive_mix), direct_force_mix=float(direct_force_mix),
            residual_feedback_mix=float(residual_feedback_mix), micro_field_max_size=int(micro_field_max_size),
            micro_decay=float(micro_decay), micro_impulse_decay=float(micro_impulse_decay),
            micro_drive_mix=float(micro_drive_mix), reservoir_decay=float(reservoir_decay),
            refractory_decay=float(refractory_decay), refractory_gain=float(refractory_gain),
            confidence_decay=float(confidence_decay), confidence_gain=float(confidence_gain),
            surprise_gain=float(surprise_gain), surprise_decay=float(surprise_decay),
            prediction_mix=float(prediction_mix), novelty_mix=float(novelty_mix), warmup_steps=int(warmup_steps),
            surprise_brake=float(surprise_brake), target_update_rms=float(target_update_rms),
            min_gain=float(min_gain), max_gain=float(max_gain), drive_clip=float(drive_clip),
            spike_mix=float(spike_mix), min_spectral_size=int(min_spectral_size),
            basis_cache_limit_elements=int(basis_cache_limit_elements), cuda_ops=mode,
            hard_channel_min_size=int(hard_channel_min_size), thin_matrix_hard_cutoff=int(thin_matrix_hard_cutoff),
            thin_matrix_max_width=int(thin_matrix_max_width), thin_matrix_min_aspect=float(thin_matrix_min_aspect),
            thin_matrix_route=route, maximize=bool(maximize), eps=float(eps),
        )
        super().__init__(params, defaults)
        self._shape_ws: Dict[tuple, Tensor] = {}
        self._hash_cache: Dict[tuple, Tuple[Tensor, int]] = {}
        self._scratch: Dict[tuple, Tensor] = {}
        # device-side failure reports: per device an int32 word that the spectral kernels OR
        # failure bits into (never cleared), and a pinned host copy of it taken after every
        # step, read without synchronising at the start of the next step
        self._status_dev: Dict[object, Tensor] = {}
        self._status_host: Dict[object, tuple] = {}
        # host-side caches for groups of many small tensors (LoRA adapters): the route of
        # each (shape, shard, routing settings), and per device the scalar-route descriptor
        # table of the last step with the identities it was built from
        self._route_cache: Dict[tuple, bool] = {}
        self._scalar_descs: Dict[object, tuple] = {}
        self._micro_descs: Dict[object, tuple] = {}
        self._fast: Dict[int, tuple] = {}  # per param group: the routing of the last full pass
        self._spectral_desc_cache: Dict[object, tuple] = {}
        self._num_sms: Dict[object, int] = {}

    # ------------------------------------------------------------------ state
    def _init_common(self, state: dict, device, dtype) -> None:
        """cresso_v5.py:857-862."""
        state["step"] = 0
        state["force_rms"] = torch.zeros((), device=device, dtype=dtype)
        state["drive_energy"] = torch.ones((), device=device, dtype=dtype)
        state["surprise"] = torch.zeros((), device=device, dtype=dtype)
        state["action"] = torch.zeros((), device=device, dtype=dtype)

    def _geometry(self, param: Tensor):
        """(global shape, row0, rows, col0, cols) of the block of the tensor this
        rank holds.  An unsharded tensor is its own global tensor; a row-sharded
        one (see cresso_b200.distributed) carries its global shape and offset."""
        spec = getattr(param, "_cresso_shard", None)
        if spec is None:
            shape = tuple(int(d) for d in param.shape)
            if len(shape) >= 2:  # rank >= 3: the leading axes flattened into rows
                rows = 1
                for d in shape[:-1]:
                    rows *= d
                return shape, 0, rows, 0, shape[-1]
            n = shape[-1] if shape else 1
            return shape, 0, 1, 0, n
        gshape, offset = spec
        gshape = tuple(int(d) for d in gshape)
        if len(gshape) == 2:
            if tuple(param.shape) != (param.shape[0], gshape[1]) or param.ndim != 2:
                raise RuntimeError("a row shard of a 2-D tensor must keep the full row width")
            return gshape, int(offset), int(param.shape[0]), 0, gshape[1]
        if len(gshape) == 1 and param.ndim == 1:
            return gshape, 0, 1, int(offset), int(param.shape[0])
        raise RuntimeError("only 1-D and 2-D tensors can be sharded")

    def _init_spectral(self, param: Tensor, group: dict, dtype, shape: Optional[tuple] = None) -> None:
        """cresso_v5.py:864-883 (same keys, shapes and dtypes).  `shape` is the
        global shape of a sharded tensor (defaults to the parameter's)."""
        shape = tuple(param.shape) if shape is None else tuple(shape)
        numel = 1
        for d in shape:
            numel *= int(d)
        state = self.state[param]
        self._init_common(state, param.device, dtype)
        rank = int(group["rank"])
        freqs = frequencies_tensor(rank, len(shape), int(group["max_frequency"]), param.device)
        state["freqs"] = freqs
        state["omega"] = omega_from_freqs(freqs).to(device=param.device, dtype=dtype)
        for name in _SPECTRAL_RANK_STATE:
            state[name] = torch.zeros(rank, device=param.device, dtype=dtype)
        bins = int(group.get("hash_bins", 0))
        tables = int(group.get("hash_tables", 1))
        cutoff = int(group.get("thin_matrix_hard_cutoff", 0))
        thin = len(shape) == 2 and cutoff > 0 and min(shape) <= cutoff
        if bins > 0 and numel >= int(group.get("hard_channel_min_size", 0)) and not thin:
            state["hash_energy"] = torch.ones(tables, bins, device=param.device, dtype=dtype)
            state["hash_impulse"] = torch.zeros(tables, bins, device=param.device, dtype=dtype)
            state["hash_refractory"] = torch.zeros(tables, bins, device=param.device, dtype=dtype)

    def _init_scalar(self, param: Tensor, dtype) -> None:
        """cresso_v5.py:885-891."""
        state = self.state[param]
        self._init_common(state, param.device, dtype)
        for name in ("q", "impulse", "metric_q", "metric_impulse"):
            state[name] = torch.zeros((), device=param.device, dtype=dtype)

    def _init_micro(self, param: Tensor, dtype) -> None:
        """cresso_v5.py:893-898: per-element float32 fields of the parameter's shape."""
        state = self.state[param]
        self._init_common(state, param.device, dtype)
        state["micro_energy"] = torch.ones_like(param, dtype=dtype, memory_format=torch.preserve_format)
        state["micro_impulse"] = torch.zeros_like(param, dtype=dtype, memory_format=torch.preserve_format)
        state["micro_refractory"] = torch.zeros_like(param, dtype=dtype, memory_format=torch.preserve_format)

    def _use_spectral_route(self, param: Tensor, group: dict) -> bool:
        return uses_spectral_route(self._geometry(param)[0], group)

    # ------------------------------------------------------------- caches
    def _workspace(self, device, shape: tuple, group: dict, freqs: Tensor) -> Tensor:
        """Per-shape carrier tables / stats / Gram / hash counts, kept across steps
        (a transient cache, never part of the state; cresso_v5.py:380-415)."""
        rank, maxf = int(group["rank"]), int(group["max_frequency"])
        bins, tables = int(group["hash_bins"]), int(group["hash_tables"])
        if bins <= 0:
            bins, tables = 0, 0
        key = (device, shape, rank, maxf, bins, tables)
        ws = self._shape_ws.get(key)
        if ws is not None:
            return ws
        L = _lib.lib()
        dims = _lib.i64_array(shape)
        nbytes = np.zeros(1, dtype=np.int64)
        _lib.check(L.cresso_shape_workspace_bytes(len(shape), dims, rank, bins, tables,
                                                  nbytes.ctypes.data_as(_lib._pi64)), "shape_workspace_bytes")
        ws = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=device)
        fr = np.ascontiguousarray(np.asarray(multiscale_frequencies(rank, len(shape), maxf), dtype=np.int64))
        stored = freqs.detach().to("cpu", torch.int64).numpy()
        if stored.shape != fr.shape or not np.array_equal(stored, fr):
            raise RuntimeError("state['freqs'] differs from the deterministic CRESSO5 frequency pack")
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_shape_workspace_init(len(shape), dims, rank, fr.ctypes.data_as(_lib._pi64), bins, tables,
                                                 _lib.ptr(ws), stream), "shape_workspace_init")
        self._shape_ws[key] = ws
        return ws

    def _workspace64(self, device, shape: tuple, group: dict, freqs: Tensor) -> Tensor:
        """Float64 carrier tables and stats of a shape (float64 parameters), kept across steps."""
        rank, maxf = int(group["rank"]), int(group["max_frequency"])
        key = (device, shape, rank, maxf, "f64")
        ws = self._shape_ws.get(key)
        if ws is not None:
            return ws
        L = _lib.lib()
        dims = _lib.i64_array(shape)
        nbytes = np.zeros(1, dtype=np.int64)
        _lib.check(L.cresso_shape_workspace64_bytes(len(shape), dims, rank, nbytes.ctypes.data_as(_lib._pi64)),
                   "shape_workspace64_bytes")
        ws = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=device)
        fr = np.ascontiguousarray(np.asarray(multiscale_frequencies(rank, len(shape), maxf), dtype=np.int64))
        stored = freqs.detach().to("cpu", torch.int64).numpy()
        if stored.shape != fr.shape or not np.array_equal(stored, fr):
            raise RuntimeError("state['freqs'] differs from the deterministic CRESSO5 frequency pack")
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_shape_workspace64_init(len(shape), dims, rank, fr.ctypes.data_as(_lib._pi64),
                                                   _lib.ptr(ws), stream), "shape_workspace64_init")
        self._shape_ws[key] = ws
        return ws

    def _hash_index_cache(self, device, bins: int, tables: int, n: int) -> Tuple[Tensor, int]:
        key = (device, bins, tables)
        cur = self._hash_cache.get(key)
        if cur is not None and cur[1] >= n:
            return cur
        L = _lib.lib()
        cap = max(n, cur[1] * 2 if cur is not None else 0)
        cap = (cap + 255) // 256 * 256  # table rows stay 16-byte aligned for the staged copies
        nbytes = np.zeros(1, dtype=np.int64)
        _lib.check(L.cresso_hash_cache_bytes(cap, bins, tables, nbytes.ctypes.data_as(_lib._pi64)), "hash_cache_bytes")
        buf = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_hash_cache_init(cap, bins, tables, _lib.ptr(buf), stream), "hash_cache_init")
        self._hash_cache[key] = (buf, cap)
        return self._hash_cache[key]

    def _scratch_buffer(self, device, kind: str, nbytes: int) -> Tensor:
        key = (device, kind)
        buf = self._scratch.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._scratch[key] = buf
        return buf

    # --------------------------------------------------------------- step
    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.check_device_status(block=False)
        spectral_devices: set = set()
        for gi, group in enumerate(self.param_groups):
            self._run_routed(group, self._route_group(gi, group), spectral_devices)
        self._publish_status(spectral_devices)
        return loss

    def _route_group(self, gi: int, group: dict):
        """(spectral, scalar, micro, spectral64): per route, per device, the
        (param, grad, state) items of the group's parameters with a gradient."""
        route_sig = (group["min_spectral_size"], group["rank"], group.get("thin_matrix_route", "scalar"),
                     group.get("thin_matrix_max_width", 64), group.get("thin_matrix_min_aspect", 4.0),
                     group.get("micro_field_max_size", 0))
        routed = self._route_fast(gi, group, route_sig)
        if routed is None:
            routed = self._route_full(gi, group, route_sig)
        return routed

    def _run_routed(self, group: dict, routed, spectral_devices: set, select=None, tag=None) -> None:
        """Launches the routes of one group; `select` (a set of parameter ids) limits
        the step to those parameters, and `tag` keys their descriptor tables apart
        from the tables of other selections."""
        spectral, scalar, micro_items, spectral64 = routed
        hp = None
        for kind, per_device in enumerate((spectral, scalar, micro_items, spectral64)):
            for device, items in per_device.items():
                if select is not None:
                    items = [it for it in items if id(it[0]) in select]
                    if not items:
                        continue
                hp = _lib.pack_hparams(group) if hp is None else hp
                if kind == 0:
                    self._run_spectral(group, hp, device, items, tag)
                    spectral_devices.add(device)
                elif kind == 1:
                    self._run_scalar(hp, device, items, tag)
                elif kind == 2:
                    self._run_micro(hp, device, items, tag)
                else:
                    self._run_spectral64(group, hp, device, items)

    def invalidate_caches(self) -> None:
        """Drops the cached routing and descriptor tables; the next step rebuilds
        them from the current parameters and state tensors."""
        self._fast.clear()
        self._scalar_descs.clear()
        self._micro_descs.clear()
        self._spectral_desc_cache.clear()

    def load_state_dict(self, state_dict) -> None:  # type: ignore[override]
        super().load_state_dict(state_dict)
        self.invalidate_caches()

    # ------------------------------------------------------- failure reports
    def _status_word(self, device) -> Tensor:
        """The device's int32 failure word (zeroed once, never cleared afterwards)."""
        w = self._status_dev.get(device)
        if w is None:
            w = self._status_dev[device] = torch.zeros(1, dtype=torch.int32, device=device)
        return w

    def _publish_status(self, devices) -> None:
        """Queues, after this step's work on each device, a copy of its failure word
        into pinned host memory; check_device_status reads it."""
        for device in devices:
            word = self._status_word(device)
            if word.device.type != "cuda":  # host-side word (multi-process tests on CPU ranks)
                self._status_host[device] = (word.clone(), None)
                continue
            entry = self._status_host.get(device)
            if entry is None:
                entry = self._status_host[device] = (torch.zeros(1, dtype=torch.int32, pin_memory=True),
                                                     torch.cuda.Event())
            host, ev = entry
            stream = torch.cuda.current_stream(device)
            # a kernel writes the pinned word (no copy engine: a copy could queue behind
            # the caller's prefetch of the next step's gradients)
            _lib.check(_lib.lib().cresso_status_copy(_lib.ptr(word), _lib.ptr(host), stream.cuda_stream),
                       "status_copy")
            ev.record(stream)

    def check_device_status(self, block: bool = True) -> None:
        """Raises RuntimeError if a spectral kernel of an earlier step reported a
        device-side failure: a bounded wait inside a pass kernel that gave up (the
        results and state of that step are invalid; bit 1), or tensor-core work still
        in flight after such a give-up (later steps are not to be trusted either;
        bit 2).  step() calls it without blocking, so a failure surfaces at the first
        step() after the failed step's copy of the word reached the host; with
        block=True (the default) it waits for the last step's copy."""
        for device, (host, ev) in self._status_host.items():
            if ev is None:
                pass
            elif block:
                ev.synchronize()
            elif not ev.query():
                continue
            v = int(host[0])
            if v:
                what = "; ".join(msg for bit, msg in _lib.DEVICE_STATUS.items() if v & bit)
                raise RuntimeError(f"CRESSO5 device failure on {device} (status {v}): {what}")

    def _route_fast(self, gi: int, group: dict, route_sig: tuple):
        """The routing of the group's last full pass, reused when nothing it depends on
        has changed: the same parameter objects (contiguous, same dtype) with the same
        state dicts, every parameter with a contiguous strided gradient of its dtype on
        its device, and the same routing settings.  Anything else returns None (before
        any state is touched) and the full pass runs."""
        cached = self._fast.get(gi)
        if cached is None:
            return None
        sig, ids, params, states, dtypes, devices, slots = cached
        plist = group["params"]
        if sig != route_sig or len(plist) != len(params) or tuple(map(id, plist)) != ids:
            return None
        grads = [p.grad for p in params]
        state = self.state
        for p, g, st, dt, dev in zip(params, grads, states, dtypes, devices):
            if (g is None or g.dtype is not dt or g.layout is not torch.strided or not g.is_contiguous()
                    or g.device != dev or not p.is_contiguous() or state.get(p) is not st):
                return None
        for st in states:
            st["step"] += 1
        routed: Tuple[Dict[torch.device, list], ...] = ({}, {}, {}, {})
        for (kind, i), p, g, st, dev in zip(slots, params, grads, states, devices):
            routed[kind].setdefault(dev, []).append((p, g, st))
        return routed

    def _route_full(self, gi: int, group: dict, route_sig: tuple):
        """Checks and routes every parameter of the group (cresso_v5.py:822-845) and
        creates missing state; records the routing for _route_fast when every
        parameter took part."""
        routed: Tuple[Dict[torch.device, list], ...] = ({}, {}, {}, {})  # spectral, scalar, micro, spectral64
        SPEC, SCAL, MICRO, SPEC64 = 0, 1, 2, 3
        micro = int(group.get("micro_field_max_size", 0))
        slots = []
        complete = True
        for param in group["params"]:
            grad = param.grad  # step() runs under no_grad: no detach needed
            if grad is None or not torch.is_floating_point(param):
                complete = False
                continue
            if grad.is_sparse:
                raise RuntimeError("CRESSO5 does not support sparse gradients")
            if not param.is_cuda:
                raise RuntimeError(
                    "CRESSO5 cuda_ops='required' requires every optimized parameter to be a CUDA parameter")
            if param.dtype not in _DTYPES:
                raise RuntimeError("CRESSO5 B200 path supports float32, float16, bfloat16 and float64 "
                                   f"parameters (got {param.dtype})")
            if not param.is_contiguous():
                raise RuntimeError("CRESSO5 B200 path updates parameters in place and needs them contiguous")
            if grad.dtype is not param.dtype or grad.device != param.device:
                raise RuntimeError("CRESSO5: grad must match its parameter's dtype and device")
            if not grad.is_contiguous():
                grad = grad.contiguous()
            state = self.state[param]
            # work and state type: float64 for float64 parameters, else float32 (cresso_v5.py:119-124)
            wdt = torch.float64 if param.dtype is torch.float64 else torch.float32
            if micro > 0 and param.ndim > 0 and param.numel() <= micro:  # cresso_v5.py:839-840
                if getattr(param, "_cresso_shard", None) is not None:
                    raise RuntimeError("micro-field tensors are not sharded: pass them whole")
                if len(state) == 0:
                    self._init_micro(param, wdt)
                kind = MICRO
            else:
                rkey = (param.shape, getattr(param, "_cresso_shard", None), route_sig)
                spectral_route = self._route_cache.get(rkey)
                if spectral_route is None:
                    spectral_route = self._route_cache[rkey] = self._use_spectral_route(param, group)
                if spectral_route:
                    # float64 tensors, and tensors of every type at rank > 16: the float64-arithmetic
                    # pipeline (float32 state for float32 / float16 / bfloat16 parameters)
                    wide = int(group["rank"]) > _lib.MAX_RANK
                    if param.dtype is torch.float64 or wide:
                        if wide and int(group["rank"]) > _lib.MAX_RANK_WIDE:
                            raise RuntimeError(f"CRESSO5 B200 path supports rank <= {_lib.MAX_RANK_WIDE} "
                                               f"(got {group['rank']})")
                        if getattr(param, "_cresso_shard", None) is not None:
                            raise RuntimeError("float64 and rank > 16 spectral tensors are not sharded: pass them "
                                               "whole")
                        if len(state) == 0:
                            self._init_spectral(param, group, wdt)
                        kind = SPEC64
                    else:
                        if len(state) == 0:
                            self._init_spectral(param, group, torch.float32, self._geometry(param)[0])
                        kind = SPEC
                else:
                    if getattr(param, "_cresso_shard", None) is not None:
                        raise RuntimeError("scalar-route (small / LoRA-thin) tensors are not sharded: pass them "
                                           "whole")
                    if len(state) == 0:
                        self._init_scalar(param, wdt)
                    kind = SCAL
            state["step"] += 1
            routed[kind].setdefault(param.device, []).append((param, grad, state))
            slots.append((kind, param, state))
        if complete and slots:
            params = tuple(p for _, p, _ in slots)
            self._fast[gi] = (route_sig, tuple(map(id, group["params"])), params, tuple(st for _, _, st in slots),
                              tuple(p.dtype for p in params), tuple(p.device for p in params),
                              tuple((k, i) for i, (k, _, _) in enumerate(slots)))
        else:
            self._fast.pop(gi, None)
        return routed

    def _spectral_descs(self, group: dict, device, items: list, tag=None) -> np.ndarray:
        """Descriptor table of the spectral group.  Like the small-route tables it is
        reused while the parameters, their storage, their state dicts and the settings
        it depends on stay the same, refreshing gradient pointers and step counters;
        the entry holds every object whose memory it points at."""
        F = _lib.DESC_INDEX
        bins, tables = int(group["hash_bins"]), int(group["hash_tables"])
        settings = (group["rank"], group["max_frequency"], bins, tables, group.get("hard_channel_min_size"),
                    group.get("thin_matrix_hard_cutoff"))
        ident = (settings, _items_ident(items))
        key = (device, id(group), tag)
        cached = self._spectral_desc_cache.get(key)
        if cached is not None and cached[0] == ident:
            descs = cached[1]
        else:
            descs, keep = self._build_spectral_descs(group, device, items)
            self._spectral_desc_cache[key] = (ident, descs, keep, group)
        descs[:, F["grad"]] = [g.data_ptr() for _, g, _ in items]
        descs[:, F["step"]] = [st["step"] for _, _, st in items]
        return descs

    def _build_spectral_descs(self, group: dict, device, items: list):
        F = _lib.DESC_INDEX
        descs = _lib.new_descs(len(items))
        keep = []
        bins, tables = int(group["hash_bins"]), int(group["hash_tables"])
        for i, (p, g, st) in enumerate(items):
            shape, row0, rows, col0, cols = self._geometry(p)
            numel = 1
            for dd in shape:
                numel *= dd
            d = descs[i]
            d[F["ndim"]] = len(shape)
            for a, sz in enumerate(shape):
                d[F["shape0"] + a] = sz
            d[F["row0"]] = row0
            d[F["rows"]] = rows
            d[F["col0"]] = col0
            d[F["cols"]] = cols
            d[F["step"]] = int(st["step"])
            d[F["param"]] = p.data_ptr()
            d[F["grad"]] = g.data_ptr()
            d[F["dtype"]] = _DTYPES[p.dtype]
            ws = self._workspace(device, shape, group, st["freqs"])
            d[F["shape_ws"]] = ws.data_ptr()
            held = [p, st, ws]
            if "hash_energy" in st and bins > 0 and hard_enabled(shape, group):
                buf, cap = self._hash_index_cache(device, bins, tables, numel)
                d[F["hash_cache"]] = buf.data_ptr()
                d[F["hash_cache_n"]] = cap
                held.append(buf)
                for name in ("hash_energy", "hash_impulse", "hash_refractory"):
                    d[F[name]] = st[name].data_ptr()
                    held.append(st[name])
            for name in ("omega",) + _SPECTRAL_RANK_STATE + ("force_rms", "drive_energy", "surprise", "action"):
                d[F[name]] = st[name].data_ptr()
                held.append(st[name])
            keep.append(held)
        return descs, keep

    def _run_spectral(self, group: dict, hp: np.ndarray, device, items: list, tag=None) -> None:
        run, scratch, layout = self._spectral_setup(group, hp, device, items, tag)
        self._spectral_stages(run, scratch, layout)

    def _spectral_setup(self, group: dict, hp: np.ndarray, device, items: list, tag=None,
                        scratch_kind: str = "spectral"):
        """Descriptor table, scratch and layout of a spectral group; returns
        (run(begin, end) launching a stage range, scratch, layout)."""
        if int(group["rank"]) > _lib.MAX_RANK:  # routing sends such tensors to the float64 pipeline
            raise RuntimeError(f"CRESSO5: rank {group['rank']} > {_lib.MAX_RANK} reached the fused spectral path")
        L = _lib.lib()
        descs = self._spectral_descs(group, device, items, tag)
        n = len(items)
        num_sms = self._num_sms.get(device)
        if num_sms is None:
            num_sms = self._num_sms[device] = torch.cuda.get_device_properties(device).multi_processor_count
        layout = np.zeros(10, dtype=np.int64)
        _lib.check(L.cresso_spectral_layout(_lib.ptr(descs), n, _lib.ptr(hp), num_sms,
                                            layout.ctypes.data_as(_lib._pi64), 10), "spectral_layout")
        scratch = self._scratch_buffer(device, scratch_kind, int(layout[0]))
        status = self._status_word(device)
        stream = torch.cuda.current_stream(device).cuda_stream

        def run(begin: int, end: int) -> None:
            _lib.check(L.cresso_spectral_run_status(_lib.ptr(descs), n, _lib.ptr(hp), _lib.ptr(scratch),
                                                    scratch.numel(), begin, end, num_sms, _lib.ptr(status), stream),
                       "spectral_run")

        return run, scratch, layout

    def _run_spectral64(self, group: dict, hp: np.ndarray, device, items: list) -> None:
        """Float64 spectral tensors and spectral tensors of any type at rank > 16: the
        float64-arithmetic pipeline, whole tensors."""
        L = _lib.lib()
        F = _lib.DESC_INDEX
        descs = _lib.new_descs(len(items))
        for i, (p, g, st) in enumerate(items):
            shape = tuple(int(d) for d in p.shape)
            rows = 1
            for dd in shape[:-1]:
                rows *= dd
            d = descs[i]
            d[F["ndim"]] = len(shape)
            for a, sz in enumerate(shape):
                d[F["shape0"] + a] = sz
            d[F["rows"]] = rows
            d[F["cols"]] = shape[-1]
            d[F["step"]] = int(st["step"])
            d[F["param"]] = p.data_ptr()
            d[F["grad"]] = g.data_ptr()
            d[F["dtype"]] = _DTYPES[p.dtype]
            d[F["shape_ws"]] = self._workspace64(device, shape, group, st["freqs"]).data_ptr()
            if "hash_energy" in st:
                for name in ("hash_energy", "hash_impulse", "hash_refractory"):
                    d[F[name]] = st[name].data_ptr()
            for name in ("omega",) + _SPECTRAL_RANK_STATE + ("force_rms", "drive_energy", "surprise", "action"):
                d[F[name]] = st[name].data_ptr()
        nb = np.zeros(1, dtype=np.int64)
        _lib.check(L.cresso_spectral64_scratch_bytes(_lib.ptr(descs), len(items), _lib.ptr(hp),
                                                     nb.ctypes.data_as(_lib._pi64)), "spectral64_scratch_bytes")
        scratch = self._scratch_buffer(device, "spectral64", int(nb[0]))
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_spectral64_run(_lib.ptr(descs), len(items), _lib.ptr(hp), _lib.ptr(scratch),
                                           scratch.numel(), stream), "spectral64_run")

    def _device_status(self) -> int:
        """OR of the failure words of every device (synchronises); 0 when no bounded
        wait inside a kernel gave up in any step so far."""
        v = 0
        for w in self._status_dev.values():
            v |= int(w.item())
        return v

    def _spectral_stages(self, run: Callable[[int, int], None], scratch: Tensor, layout: np.ndarray) -> None:
        """Runs the kernel stages of a group step; one GPU needs no exchange."""
        run(0, _lib.SPECTRAL_STAGES)

    @staticmethod
    def _reduction_view(scratch: Tensor, layout: np.ndarray, k: int) -> Tensor:
        """Float64 view of reduction vector k (1..4) inside the scratch."""
        off, length = int(layout[2 * k - 1]), int(layout[2 * k])
        return scratch[off:off + 8 * length].view(torch.float64)

    def _small_route_descs(self, cache: dict, device, items: list, state_names: Tuple[str, ...],
                           bytes_fn: Callable, what: str, tag=None) -> Tuple[np.ndarray, int]:
        """Descriptor table of the scalar or the micro route.  It depends on the
        parameters, their storage and their state tensors and is reused while those
        stay the same; the gradient pointers and step counters change from step to
        step and are refreshed every time.  The cache entry holds references to the
        parameters, state dicts and state tensors it points at, so none of them can
        be freed (and its id or device address reused) while the entry lives."""
        F = _lib.DESC_INDEX
        n = len(items)
        ident = _items_ident(items)
        cached = cache.get((device, tag))
        if cached is not None and cached[0] == ident:
            descs, nbytes = cached[1], cached[2]
        else:
            descs = _lib.new_descs(n)
            keep = []
            for i, (p, g, st) in enumerate(items):
                d = descs[i]
                d[F["ndim"]] = p.ndim
                for a, sz in enumerate(p.shape):
                    d[F["shape0"] + a] = int(sz)
                d[F["param"]] = p.data_ptr()
                d[F["dtype"]] = _DTYPES[p.dtype]
                for name in state_names:
                    d[F[name]] = st[name].data_ptr()
                keep.append((p, st, [st[name] for name in state_names]))
            descs[:, F["grad"]] = [g.data_ptr() for _, g, _ in items]
            descs[:, F["step"]] = [int(st["step"]) for _, _, st in items]
            nb = np.zeros(1, dtype=np.int64)
            _lib.check(bytes_fn(_lib.ptr(descs), n, nb.ctypes.data_as(_lib._pi64)), what)
            nbytes = int(nb[0])
            cache[(device, tag)] = (ident, descs, nbytes, keep)
        descs[:, F["grad"]] = [g.data_ptr() for _, g, _ in items]
        descs[:, F["step"]] = [st["step"] for _, _, st in items]
        return descs, nbytes

    def _run_scalar(self, hp: np.ndarray, device, items: list, tag=None) -> None:
        L = _lib.lib()
        descs, nbytes = self._small_route_descs(
            self._scalar_descs, device, items,
            ("force_rms", "drive_energy", "surprise", "action", "q", "impulse", "metric_q", "metric_impulse"),
            L.cresso_scalar_scratch_bytes, "scalar_scratch_bytes", tag)
        scratch = self._scratch_buffer(device, "scalar", nbytes)
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_scalar_run(_lib.ptr(descs), len(items), _lib.ptr(hp), _lib.ptr(scratch), scratch.numel(),
                                       stream), "scalar_run")

    def _run_micro(self, hp: np.ndarray, device, items: list, tag=None) -> None:
        L = _lib.lib()
        descs, nbytes = self._small_route_descs(
            self._micro_descs, device, items,
            ("force_rms", "drive_energy", "surprise", "micro_energy", "micro_impulse", "micro_refractory"),
            L.cresso_micro_scratch_bytes, "micro_scratch_bytes", tag)
        scratch = self._scratch_buffer(device, "micro", nbytes)
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(L.cresso_micro_run(_lib.ptr(descs), len(items), _lib.ptr(hp), _lib.ptr(scratch), scratch.numel(),
                                      stream), "micro_run")


CRESSO = CRESSO5
