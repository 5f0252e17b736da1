"""The C-ABI library: it loads, exports every symbol include/cresso_b200.h
declares, reports its layout, and validates arguments on the host (no GPU
work is launched here)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from cresso_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "cresso_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"CRESSO_API\s+(?:const\s+char\s*\*|int64_t|int)\s+(cresso_\w+)\s*\(", HEADER.read_text())))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) == 30
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(_lib.EXPORTS) == names


def test_version_arch_and_layout():
    lib = _lib.lib()
    assert lib.cresso_arch() == b"sm_100a"
    assert b"cresso_b200" in lib.cresso_version()
    out = (ctypes.c_int64 * 4)()
    assert lib.cresso_abi_layout(out, 4) == 0
    assert list(out) == [8 * len(_lib.HPARAM_FIELDS), 8 * _lib.DESC_WORDS, 8, 16]
    assert lib.cresso_abi_layout(out, 2) == 1


def test_argument_errors_are_reported_not_raised():
    lib = _lib.lib()
    n = np.zeros(1, dtype=np.int64)
    assert lib.cresso_hash_cache_bytes(10, 0, 2, n.ctypes.data_as(_lib._pi64)) == 1
    assert "bins" in _lib.last_error()
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(lib.cresso_hash_index(0, -1, 64, 0, None, None), "hash_index")
    dims = _lib.i64_array([2] * 9)
    assert lib.cresso_shape_workspace_bytes(9, dims, 8, 64, 2, n.ctypes.data_as(_lib._pi64)) == 2
    assert "rank 1 to 8" in _lib.last_error()
    dims = _lib.i64_array([4, 5, 6])
    assert lib.cresso_shape_workspace_bytes(3, dims, 8, 64, 2, n.ctypes.data_as(_lib._pi64)) == 0
    dims = _lib.i64_array([64, 64])
    assert lib.cresso_shape_workspace_bytes(2, dims, 17, 64, 2, n.ctypes.data_as(_lib._pi64)) == 2
    assert lib.cresso_shape_workspace_bytes(2, dims, 8, 64, 2, n.ctypes.data_as(_lib._pi64)) == 0
    assert n[0] > 64 * 8 * 2 * 4 * 2


def _fake_desc(shape, rows=None, row0=0):
    F = _lib.DESC_INDEX
    d = _lib.new_descs(1)
    d[0, F["ndim"]] = len(shape)
    for a, s in enumerate(shape):
        d[0, F["shape0"] + a] = s
    d[0, F["rows"]] = rows if rows is not None else (shape[0] if len(shape) == 2 else 1)
    d[0, F["row0"]] = row0
    d[0, F["cols"]] = shape[-1]
    d[0, F["step"]] = 1
    for name in _lib.DESC_FIELDS[F["param"]:]:
        if name not in ("hash_cache", "hash_cache_n"):
            d[0, F[name]] = 4096
    d[0, F["hash_cache"]] = 4096
    d[0, F["hash_cache_n"]] = int(np.prod(shape))
    d[0, F["dtype"]] = 0  # float32
    return d


def test_spectral_layout_is_host_logic():
    from oracle.cresso5_oracle import hparams
    lib = _lib.lib()
    hp = _lib.pack_hparams(hparams(rank=8, hash_bins=64, hash_tables=2))
    lay = np.zeros(9, dtype=np.int64)
    d = _fake_desc((4096, 4096))
    assert lib.cresso_spectral_layout(_lib.ptr(d), 1, _lib.ptr(hp), 148, lay.ctypes.data_as(_lib._pi64), 9) == 0, _lib.last_error()
    assert lay[0] >= 4096 * 4096 * 4  # the tangent field dominates the scratch
    assert lay[2] == 1 and lay[8] == 29
    assert lay[4] == 2 + 16 + 128 + 4096 and lay[6] == 2 + 16 + 128
    # a row shard holds rows [1024, 2048) of the same tensor: same reduction lengths, 1/4 of the field
    d2 = _fake_desc((4096, 4096), rows=1024, row0=1024)
    lay2 = np.zeros(9, dtype=np.int64)
    assert lib.cresso_spectral_layout(_lib.ptr(d2), 1, _lib.ptr(hp), 148, lay2.ctypes.data_as(_lib._pi64), 9) == 0
    assert lay2[4] == lay[4] and lay2[0] < lay[0] / 2
    bad = _fake_desc((4096, 4096), rows=1024, row0=3584)
    assert lib.cresso_spectral_layout(_lib.ptr(bad), 1, _lib.ptr(hp), 148, lay2.ctypes.data_as(_lib._pi64), 9) == 1
    assert "outside the global shape" in _lib.last_error()
    hp17 = _lib.pack_hparams(hparams(rank=17))
    assert lib.cresso_spectral_layout(_lib.ptr(d), 1, _lib.ptr(hp17), 148, lay.ctypes.data_as(_lib._pi64), 9) == 2


def test_tensor_core_pass_selection():
    """The planner's choice of the tcgen05 form (layout[10], layout[11]): large
    full-tile tensors at rank pad 8 run P3-P5 on the tensor cores; small
    workloads (fewer rows per item), other rank pads and unaligned shapes do not."""
    from oracle.cresso5_oracle import hparams
    lib = _lib.lib()

    def plan(shape, **kw):
        hp = _lib.pack_hparams(hparams(**{**dict(rank=8, hash_bins=64, hash_tables=2), **kw}))
        lay = np.zeros(12, dtype=np.int64)
        d = _fake_desc(shape)
        assert lib.cresso_spectral_layout(_lib.ptr(d), 1, _lib.ptr(hp), 148, lay.ctypes.data_as(_lib._pi64), 12) == 0
        return int(lay[10]), int(lay[11]), int(lay[9])

    tc_bits = (1 << 3) | (1 << 4) | (1 << 5)
    rows, bits, status_off = plan((8192, 2048))
    assert (rows, bits) == (16, tc_bits) and status_off > 0
    assert plan((4096, 4096))[:2] == (16, tc_bits)
    assert plan((4096, 4096), rank=5)[:2] == (16, tc_bits)     # rank 5 pads to 8
    assert plan((4096, 4096), rank=4)[1] == 0                  # rank pad 4: CUDA-core form
    assert plan((4096, 4096), rank=12)[1] == 0                 # rank pad 16: CUDA-core form
    assert plan((2048, 2048))[0] < 16 and plan((2048, 2048))[1] == 0  # small: shorter items
    assert plan((4096, 4100))[1] == 0                          # ragged columns: general class only


def test_scalar_scratch_is_host_logic():
    lib = _lib.lib()
    n = np.zeros(1, dtype=np.int64)
    d = _fake_desc((4096, 16))
    assert lib.cresso_scalar_scratch_bytes(_lib.ptr(d), 1, n.ctypes.data_as(_lib._pi64)) == 0
    assert n[0] >= 4 * (4096 + 4096 + 16)


def test_micro_scratch_is_host_logic():
    lib = _lib.lib()
    F = _lib.DESC_INDEX
    n = np.zeros(1, dtype=np.int64)
    for shape, work in (((4096,), 0), ((3, 4, 5), 12), ((1, 1000), 1001)):
        d = _fake_desc(shape)
        assert lib.cresso_micro_scratch_bytes(_lib.ptr(d), 1, n.ctypes.data_as(_lib._pi64)) == 0
        assert n[0] >= 4 * work  # rank >= 2: one log term per axis coordinate
    d = _fake_desc((3, 4, 5))
    d[0, F["micro_refractory"]] = 0
    assert lib.cresso_micro_scratch_bytes(_lib.ptr(d), 1, n.ctypes.data_as(_lib._pi64)) == 1
    assert "NULL" in _lib.last_error()
    d = _fake_desc((3, 4, 5))
    d[0, F["dtype"]] = 7
    assert lib.cresso_micro_scratch_bytes(_lib.ptr(d), 1, n.ctypes.data_as(_lib._pi64)) == 2
    d = _fake_desc((2,) * 4)
    d[0, F["ndim"]] = 0
    assert lib.cresso_micro_scratch_bytes(_lib.ptr(d), 1, n.ctypes.data_as(_lib._pi64)) == 1
    assert "rank 1 to 8" in _lib.last_error()
