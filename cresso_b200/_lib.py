"""ctypes binding of ``libcresso_b200.so`` (C ABI in ``include/cresso_b200.h``).

The library is built ahead of time (``python -m cresso_b200.build``).  There is
no JIT and no fallback: if the shared library is missing or cannot be loaded,
every entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_C" / "libcresso_b200.so"

# Field order of cresso_hparams (include/cresso_b200.h).
HPARAM_FIELDS = (
    "lr", "weight_decay", "energy_power", "dt", "impulse_friction", "contact_gain", "restoring", "cubic",
    "metric_dt", "metric_friction", "metric_coupling", "local_sharpness",
    "instant_metric_coupling", "instant_metric_power", "root_channel_mix", "echo_mix", "transport_mix",
    "hash_decay", "hash_impulse_decay", "hash_metric_coupling", "hash_drive_mix",
    "direct_force_mix", "residual_feedback_mix", "reservoir_decay", "refractory_decay", "refractory_gain",
    "confidence_decay", "confidence_gain", "surprise_gain", "surprise_decay", "prediction_mix", "novelty_mix",
    "warmup_steps", "surprise_brake", "target_update_rms", "min_gain", "max_gain", "drive_clip", "spike_mix",
    "eps", "maximize", "rank", "max_frequency", "hash_bins", "hash_tables", "hard_channel_min_size",
    "thin_matrix_hard_cutoff", "micro_decay", "micro_impulse_decay", "micro_drive_mix",
)

MAX_NDIM = 8
MAX_RANK = 16        # the fused float32 spectral path
MAX_RANK_PLAIN = 64  # the float64-arithmetic spectral path with its modes in registers
MAX_RANK_WIDE = 4096  # the same path with its modes in memory (the reference CUDA contact kernel's bound)
SPECTRAL_STAGES = 14
# stage boundaries after which reduction vector k (1..4) is complete
REDUCTION_BOUNDARIES = (3, 6, 9, 12)
NOALLOC_SCRATCH_BYTES = 8 << 20  # CRESSO_NOALLOC_SCRATCH_BYTES

# Field order of cresso_tensor_desc; every field is 8 bytes.
DESC_FIELDS = (
    ["ndim"] + [f"shape{i}" for i in range(MAX_NDIM)]
    + ["row0", "rows", "col0", "cols", "step", "param", "grad", "shape_ws", "hash_cache", "hash_cache_n",
       "omega", "q_cos", "q_sin", "p_cos", "p_sin", "metric_cos", "metric_sin", "metric_p_cos", "metric_p_sin",
       "calcium_cos", "calcium_sin", "mode_confidence", "hash_energy", "hash_impulse", "hash_refractory",
       "force_rms", "drive_energy", "surprise", "action", "q", "impulse", "metric_q", "metric_impulse", "dtype",
       "micro_energy", "micro_impulse", "micro_refractory"]
)
DTYPE_CODES = {"float32": 0, "float16": 1, "bfloat16": 2, "float64": 3}
DESC_INDEX = {name: i for i, name in enumerate(DESC_FIELDS)}
DESC_WORDS = len(DESC_FIELDS)

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported on the CUDA path", 3: "CUDA error", 4: "scratch too small"}
# failure bits of the device status word of cresso_spectral_run_status
DEVICE_STATUS = {1: "a bounded wait inside a spectral pass kernel gave up (that step's results and state are invalid)",
                 2: "tensor-core work was still in flight when a block gave up (later steps are not to be trusted)"}

EXPORTS = (
    "cresso_version", "cresso_arch", "cresso_last_error", "cresso_abi_layout", "cresso_launch_count",
    "cresso_hash_index", "cresso_hash_reduce_mean", "cresso_hash_gather", "cresso_hash_cache_bytes",
    "cresso_hash_cache_init", "cresso_shape_workspace_bytes", "cresso_shape_workspace_init",
    "cresso_basis_project", "cresso_basis_reconstruct", "cresso_instant_axis_metric",
    "cresso_spectral_layout", "cresso_spectral_run", "cresso_scalar_scratch_bytes", "cresso_scalar_run",
    "cresso_scalar_run_noalloc", "cresso_micro_scratch_bytes", "cresso_micro_run", "cresso_selftest_bounded_wait",
    "cresso_shape_workspace64_bytes", "cresso_shape_workspace64_init", "cresso_spectral64_scratch_bytes",
    "cresso_spectral64_run", "cresso_spectral_run_status", "cresso_status_copy", "cresso_copy_segments",
)

_lock = threading.Lock()
_lib = None
_load_error: Exception | None = None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_dbl = ctypes.c_double
_pi64 = ctypes.POINTER(ctypes.c_int64)


def _declare(lib) -> None:
    sig = {
        "cresso_version": (ctypes.c_char_p, []),
        "cresso_arch": (ctypes.c_char_p, []),
        "cresso_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
        "cresso_abi_layout": (ctypes.c_int, [_pi64, ctypes.c_int]),
        "cresso_launch_count": (ctypes.c_int64, []),
        "cresso_hash_index": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _p]),
        "cresso_hash_reduce_mean": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p]),
        "cresso_hash_gather": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p]),
        "cresso_hash_cache_bytes": (ctypes.c_int, [_i64, _i64, _i64, _pi64]),
        "cresso_hash_cache_init": (ctypes.c_int, [_i64, _i64, _i64, _p, _p]),
        "cresso_shape_workspace_bytes": (ctypes.c_int, [_i64, _pi64, _i64, _i64, _i64, _pi64]),
        "cresso_shape_workspace_init": (ctypes.c_int, [_i64, _pi64, _i64, _pi64, _i64, _i64, _p, _p]),
        "cresso_basis_project": (ctypes.c_int, [_p, _p, _p, _p, _p]),
        "cresso_basis_reconstruct": (ctypes.c_int, [_p, _p, _p, _p, _p, _p]),
        "cresso_instant_axis_metric": (ctypes.c_int, [_p, _i64, _pi64, _dbl, _dbl, _dbl, _p, _p]),
        "cresso_spectral_layout": (ctypes.c_int, [_p, _i64, _p, _i64, _pi64, _i64]),
        "cresso_spectral_run": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _i64, _i64, _i64, _p]),
        "cresso_spectral_run_status": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _i64, _i64, _i64, _p, _p]),
        "cresso_status_copy": (ctypes.c_int, [_p, _p, _p]),
        "cresso_copy_segments": (ctypes.c_int, [_p, _i64, _p]),
        "cresso_scalar_scratch_bytes": (ctypes.c_int, [_p, _i64, _pi64]),
        "cresso_scalar_run": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _p]),
        "cresso_scalar_run_noalloc": (ctypes.c_int, [_p, _i64, _p, _p]),
        "cresso_micro_scratch_bytes": (ctypes.c_int, [_p, _i64, _pi64]),
        "cresso_micro_run": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _p]),
        "cresso_selftest_bounded_wait": (ctypes.c_int, [_i64, _i64, _p, _p]),
        "cresso_shape_workspace64_bytes": (ctypes.c_int, [_i64, _pi64, _i64, _pi64]),
        "cresso_shape_workspace64_init": (ctypes.c_int, [_i64, _pi64, _i64, _pi64, _p, _p]),
        "cresso_spectral64_scratch_bytes": (ctypes.c_int, [_p, _i64, _p, _pi64]),
        "cresso_spectral64_run": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library; raises RuntimeError (never falls back) if it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("CRESSO_B200_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"cresso_b200 CUDA library not found at {path}; build it with `python -m cresso_b200.build`")
        try:
            handle = ctypes.CDLL(str(path))
            _declare(handle)
            out = (ctypes.c_int64 * 4)()
            if handle.cresso_abi_layout(out, 4) != 0:
                raise RuntimeError("cresso_abi_layout failed")
            if out[0] != 8 * len(HPARAM_FIELDS) or out[1] != 8 * DESC_WORDS or out[2] != MAX_NDIM or out[3] != MAX_RANK:
                raise RuntimeError(f"ABI layout mismatch: library reports {list(out)}")
        except Exception as exc:  # surfaced, not swallowed
            _load_error = exc
            raise RuntimeError(f"cresso_b200 CUDA library failed to load: {exc}") from exc
        _lib = handle
        return _lib


def launch_count() -> int:
    """Kernels launched by the library in this process so far."""
    return int(lib().cresso_launch_count())


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().cresso_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what}: {STATUS.get(status, status)}: {last_error()}")


def pack_hparams(group: dict) -> np.ndarray:
    hp = np.zeros(len(HPARAM_FIELDS), dtype=np.float64)
    for i, name in enumerate(HPARAM_FIELDS):
        v = group.get(name, 0.0)
        hp[i] = float(bool(v)) if isinstance(v, bool) else float(v)
    return hp


def new_descs(n: int) -> np.ndarray:
    return np.zeros((n, DESC_WORDS), dtype=np.int64)


def ptr(a) -> ctypes.c_void_p:
    """Address of a numpy array or torch tensor (0 / None -> NULL)."""
    if a is None:
        return ctypes.c_void_p(0)
    if isinstance(a, int):
        return ctypes.c_void_p(a)
    if isinstance(a, np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)
    return ctypes.c_void_p(a.data_ptr())


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)
