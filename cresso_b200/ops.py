"""Op-level entry points with the argument meaning of the reference's
extension functions (cresso_cuda/cresso_cuda.cpp:170-196), for tests and for
callers that drive single operators.  They take CUDA tensors, allocate their
outputs with torch, and run on the current stream.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import numpy as np
import torch
from torch import Tensor

from . import _lib
from ._host import multiscale_frequencies


def _stream(t: Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda_f32(t: Tensor, name: str) -> Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32 (got {t.dtype})")
    return t.contiguous()


def hash_index(shape: Sequence[int], bins: int, salt: int, device, offset: int = 0) -> Tensor:
    """Bin index of every flat index of `shape` (reference _hash_index_tensor, cresso_v5.py:495-516)."""
    n = int(np.prod([int(d) for d in shape])) if len(shape) else 1
    out = torch.empty(n, dtype=torch.int64, device=device)
    _lib.check(_lib.lib().cresso_hash_index(int(offset), n, int(bins), int(salt), _lib.ptr(out), _stream(out)),
               "hash_index")
    return out.view(tuple(int(d) for d in shape))


def hash_reduce_mean(x: Tensor, bins: int, salt: int) -> Tensor:
    """ops.hash_reduce_mean (cresso_cuda.cpp:186)."""
    x = _need_cuda_f32(x, "x")
    out = torch.empty(int(bins), dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().cresso_hash_reduce_mean(_lib.ptr(x), x.numel(), int(bins), int(salt), _lib.ptr(out),
                                                  _stream(x)), "hash_reduce_mean")
    return out


def hash_gather(values: Tensor, shape: Sequence[int], salt: int) -> Tensor:
    """ops.hash_gather (cresso_cuda.cpp:187)."""
    values = _need_cuda_f32(values, "values")
    shape = tuple(int(d) for d in shape)
    out = torch.empty(shape, dtype=torch.float32, device=values.device)
    _lib.check(_lib.lib().cresso_hash_gather(_lib.ptr(values), values.numel(), out.numel(), int(salt), _lib.ptr(out),
                                             _stream(values)), "hash_gather")
    return out


_WS_CACHE: dict = {}


def basis_workspace(shape: Sequence[int], rank: int, max_frequency: int, device) -> Tensor:
    """Shape workspace of the carrier pack (replaces basis_axis_cache + basis_stats_with_cache)."""
    shape = tuple(int(d) for d in shape)
    key = (str(device), shape, int(rank), int(max_frequency))
    ws = _WS_CACHE.get(key)
    if ws is not None:
        return ws
    L = _lib.lib()
    dims = _lib.i64_array(shape)
    nbytes = np.zeros(1, dtype=np.int64)
    _lib.check(L.cresso_shape_workspace_bytes(len(shape), dims, int(rank), 0, 0, nbytes.ctypes.data_as(_lib._pi64)),
               "shape_workspace_bytes")
    ws = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=device)
    fr = np.ascontiguousarray(np.asarray(multiscale_frequencies(rank, len(shape), max_frequency), dtype=np.int64))
    _lib.check(L.cresso_shape_workspace_init(len(shape), dims, int(rank), fr.ctypes.data_as(_lib._pi64), 0, 0,
                                             _lib.ptr(ws), torch.cuda.current_stream(device).cuda_stream),
               "shape_workspace_init")
    _WS_CACHE[key] = ws
    return ws


def basis_project(x: Tensor, rank: int, max_frequency: int = 5) -> Tuple[Tensor, Tensor]:
    """(mean(x * cos_r), mean(x * sin_r)) for r < rank (ops.basis_project, cresso_cuda.cpp:174)."""
    x = _need_cuda_f32(x, "x")
    ws = basis_workspace(tuple(x.shape), rank, max_frequency, x.device)
    oc = torch.empty(int(rank), dtype=torch.float32, device=x.device)
    os_ = torch.empty(int(rank), dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().cresso_basis_project(_lib.ptr(x), _lib.ptr(ws), _lib.ptr(oc), _lib.ptr(os_), _stream(x)),
               "basis_project")
    return oc, os_


def basis_reconstruct(cos_coeff: Tensor, sin_coeff: Tensor, shape: Sequence[int], max_frequency: int = 5,
                      gates: Optional[Tensor] = None) -> Tensor:
    """shrink * sum_r g_r (c_r cos_r + s_r sin_r) (ops.basis_reconstruct, cresso_cuda.cpp:177)."""
    cc = _need_cuda_f32(cos_coeff, "cos_coeff")
    cs = _need_cuda_f32(sin_coeff, "sin_coeff")
    rank = cc.numel()
    g = _need_cuda_f32(gates, "gates") if gates is not None else None
    ws = basis_workspace(tuple(shape), rank, max_frequency, cc.device)
    out = torch.empty(tuple(int(d) for d in shape), dtype=torch.float32, device=cc.device)
    _lib.check(_lib.lib().cresso_basis_reconstruct(_lib.ptr(cc), _lib.ptr(cs), _lib.ptr(g), _lib.ptr(ws),
                                                   _lib.ptr(out), _stream(cc)), "basis_reconstruct")
    return out


def instant_axis_metric(rel: Tensor, power: float, coupling: float, eps: float) -> Tensor:
    """Axial current metric of a 1-D / 2-D field (ops.instant_axis_metric_2d, cresso_cuda.cpp:190)."""
    rel = _need_cuda_f32(rel, "rel")
    out = torch.empty_like(rel)
    dims = _lib.i64_array(rel.shape)
    _lib.check(_lib.lib().cresso_instant_axis_metric(_lib.ptr(rel), rel.ndim, dims, float(power), float(coupling),
                                                     float(eps), _lib.ptr(out), _stream(rel)), "instant_axis_metric")
    return out
