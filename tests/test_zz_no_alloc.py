"""The allocation-free neighbour build (facek_nlist_cell_build_noalloc), called through the C ABI.

Some callers cannot allocate device memory themselves -- a host framework that only hands out preallocated
buffers, or code running inside a memory arena that forbids cudaMalloc.  For them the periodic neighbour build has
a variant that keeps its scratch in a fixed device array inside the library (limit 262,144 atoms, 65,536 cells);
the caller still provides the inputs and every output buffer.  This file checks it against the regular entry
points (caller-provided workspace) on two calls in a row, which also exercises the reuse of the shared scratch:
the second call must not see anything the first one left behind.  It is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _regular(st, rc, dtype):
    """The existing path: facek_nlist_cell_workspace / _count / prefix sum / _fill."""
    from face_b200.neighbors import _periodic_rows
    pos64 = torch.as_tensor(st.positions, dtype=torch.float64, device="cuda").contiguous()
    rp, ei, ej, S, sh = _periodic_rows(pos64, np.asarray(st.cell, np.float64), rc, dtype)
    return rp.to(torch.int32), ei, ej, S, sh


def _noalloc(st, rc, dtype, capacity):
    from face_b200 import _lib
    pos64 = torch.as_tensor(st.positions, dtype=torch.float64, device="cuda").contiguous()
    N = pos64.shape[0]
    row_ptr = torch.full((N + 1,), -7, dtype=torch.int32, device="cuda")
    ei = torch.full((capacity,), -7, dtype=torch.int32, device="cuda")
    ej = torch.full((capacity,), -7, dtype=torch.int32, device="cuda")
    S = torch.full((capacity, 3), -7, dtype=torch.int32, device="cuda")
    sh = torch.full((capacity, 3), float("nan"), dtype=dtype, device="cuda")
    n_edges = ctypes.c_int64(-1)
    _lib.call("facek_nlist_cell_build_noalloc", _lib.dtype_tag(sh), _lib.ptr(pos64), N,
              _lib.doubles(np.asarray(st.cell, np.float64).reshape(-1)), float(rc), capacity, _lib.ptr(row_ptr),
              _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), _lib.ptr(sh), ctypes.byref(n_edges), _lib.stream())
    E = n_edges.value
    return row_ptr, ei[:E], ej[:E], S[:E], sh[:E], E


def _same(a, b):
    return a.shape == b.shape and bool(torch.equal(a, b))


def test_noalloc_matches_regular_build_twice():
    from face_b200 import systems
    cases = [(systems.config_structures(5, seed=1, scale=5)[0], 5.0, torch.float32),
             (systems.config_structures(2, seed=2, scale=3)[0], 6.0, torch.float64)]
    for st, rc, dt in cases:                            # two calls in a row, different sizes and dtypes
        rp0, ei0, ej0, S0, sh0 = _regular(st, rc, dt)
        rp1, ei1, ej1, S1, sh1, E = _noalloc(st, rc, dt, capacity=ei0.numel() + 64)
        assert E == ei0.numel()
        assert _same(rp1, rp0) and _same(ei1, ei0) and _same(ej1, ej0) and _same(S1, S0)
        assert _same(sh1, sh0)                          # bit-exact: same fp64 shift vectors cast to dt


def test_noalloc_rejects_out_of_range_sizes():
    from face_b200 import systems
    from face_b200 import _lib
    st = systems.config_structures(5, seed=1, scale=4)[0]
    rp0, ei0, *_ = _regular(st, 5.0, torch.float32)
    with pytest.raises(RuntimeError, match="capacity"):
        _noalloc(st, 5.0, torch.float32, capacity=ei0.numel() - 1)
    big = torch.zeros(262145, 3, dtype=torch.float64, device="cuda")
    n_edges = ctypes.c_int64(-1)
    buf = torch.zeros(262146, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="exceeds the limit"):
        _lib.call("facek_nlist_cell_build_noalloc", 0, _lib.ptr(big), big.shape[0],
                  _lib.doubles(np.diag([300.0, 300.0, 300.0]).reshape(-1)), 5.0, 0, _lib.ptr(buf), None, None, None,
                  None, ctypes.byref(n_edges), _lib.stream())
    # still usable afterwards
    rp1, ei1, *_ = _noalloc(st, 5.0, torch.float32, capacity=ei0.numel())
    assert _same(rp1, rp0) and _same(ei1, ei0)


def test_noalloc_rejects_too_many_cells_and_long_rows():
    """The cell-count limit is checked on the host before any GPU work; a row with more than 512 neighbours is caught
    in the counting pass, before row offsets are used and before any edge is written."""
    from face_b200 import _lib, systems
    rng = np.random.default_rng(11)
    sparse = systems.Structure(rng.uniform(0, 100.0, (100, 3)), np.ones(100, np.int64), np.eye(3) * 100.0, True)
    with pytest.raises(RuntimeError, match="cells exceed the limit"):
        _noalloc(sparse, 1.0, torch.float32, capacity=1000)          # 99^3 cells of width >= rc
    dense = systems.Structure(rng.uniform(0, 10.0, (800, 3)), np.ones(800, np.int64), np.eye(3) * 10.0, True)
    pos64 = torch.as_tensor(dense.positions, dtype=torch.float64, device="cuda").contiguous()
    cap = 1 << 20
    row_ptr = torch.zeros(801, dtype=torch.int32, device="cuda")
    ei = torch.full((cap,), -7, dtype=torch.int32, device="cuda")
    ej, S = torch.full_like(ei, -7), torch.full((cap, 3), -7, dtype=torch.int32, device="cuda")
    sh = torch.zeros(cap, 3, dtype=torch.float32, device="cuda")
    n_edges = ctypes.c_int64(0)
    with pytest.raises(RuntimeError, match="more than 512 neighbours"):   # ~720 neighbours per atom at rc = 6
        _lib.call("facek_nlist_cell_build_noalloc", 0, _lib.ptr(pos64), 800,
                  _lib.doubles(np.asarray(dense.cell, np.float64).reshape(-1)), 6.0, cap, _lib.ptr(row_ptr),
                  _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), _lib.ptr(sh), ctypes.byref(n_edges), _lib.stream())
    assert n_edges.value == -1
    assert bool((ei == -7).all()) and bool((ej == -7).all())              # nothing filled
    st = systems.config_structures(5, seed=1, scale=4)[0]                  # the shared scratch is reusable after
    rp0, ei0, *_ = _regular(st, 5.0, torch.float32)
    rp1, ei1, *_ = _noalloc(st, 5.0, torch.float32, capacity=ei0.numel())
    assert _same(rp1, rp0) and _same(ei1, ei0)
