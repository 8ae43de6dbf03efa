"""The allocation-free entry point tnr_neighbor_list_static.

Some callers cannot allocate device memory at the moment they need a
neighbor list (a framework that forbids allocation on its hot path, or a
process whose GPU memory is owned by another allocator's pool).  They call
tnr_neighbor_list_static, which works in a fixed device array owned by the
library and writes into the caller's output buffers.  These tests call it
through the C ABI twice in a row, on the default stream and on a
non-blocking side stream with different inputs each time, and check each
result against the reference's CPU core (exact pair sets) and against the
regular entry point (the PyTorch op): d/D within 1e-5 (float32) / 1e-12
(float64) relative.

The file is named to be collected last, so a run that stops at the first
failure has run every other test before this one.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.support import canonical, expected_pairs
from tonari_b200 import _cabi, neighbor_list, workloads

pytestmark = pytest.mark.gpu

TOLERANCE = {torch.float32: 1e-5, torch.float64: 1e-12}


def call_static(positions, cell, pbc, batch_ptr, cutoff, capacity, half_list=False,
                include_self=False, stream=None):
    """One call of the static entry point with caller-owned output buffers."""
    device = positions.device
    dtype = positions.dtype
    out = {
        "P": torch.empty((capacity, 2), dtype=torch.int64, device=device),
        "S": torch.empty((capacity, 3), dtype=torch.int32, device=device),
        "d": torch.empty((capacity,), dtype=dtype, device=device),
        "D": torch.empty((capacity, 3), dtype=dtype, device=device),
    }
    request = _cabi.Request(
        dtype=1 if dtype == torch.float64 else 0, n_atoms=positions.shape[0],
        n_structures=batch_ptr.numel() - 1, positions=positions.data_ptr(),
        batch_ptr=batch_ptr.data_ptr(), cell=cell.data_ptr(), pbc=pbc.data_ptr(),
        cutoff=cutoff, half_list=int(half_list), include_self=int(include_self),
        algorithm=0, quantities=_cabi.quantity_mask("PSdD"), index_offset=0)
    result = _cabi.Result(P=out["P"].data_ptr(), S=out["S"].data_ptr(), d=out["d"].data_ptr(),
                          D=out["D"].data_ptr())
    message = ctypes.create_string_buffer(512)
    stream = stream or torch.cuda.current_stream(device)
    status = _cabi.library().tnr_neighbor_list_static(
        ctypes.byref(request), ctypes.c_void_p(stream.cuda_stream), capacity,
        ctypes.byref(result), message, len(message))
    torch.cuda.synchronize(device)
    assert status == 0, (status, message.value)
    n = result.n_pairs
    return {key: value[:n] for key, value in out.items()}


def compare(static, regular, dtype, oracle_pairs=None):
    assert np.array_equal(canonical(static["P"], static["S"]),
                          canonical(regular["P"], regular["S"]))
    if oracle_pairs is not None:
        assert np.array_equal(canonical(static["P"], static["S"]), canonical(*oracle_pairs))
    tol = TOLERANCE[dtype]
    # Both paths emit source-major rows; align them by canonical order.
    def order(o):
        rows = np.concatenate((o["P"].cpu().numpy(), o["S"].cpu().numpy()), axis=1)
        return np.lexsort(tuple(rows[:, k] for k in range(4, -1, -1)))
    a, b = order(static), order(regular)
    D_static = static["D"].cpu().numpy()[a].astype(np.float64)
    D_regular = regular["D"].cpu().numpy()[b].astype(np.float64)
    scale = np.maximum(np.linalg.norm(D_regular, axis=1), 1e-3)
    assert np.all(np.linalg.norm(D_static - D_regular, axis=1) <= tol * scale)
    d_static = static["d"].cpu().numpy()[a].astype(np.float64)
    d_regular = regular["d"].cpu().numpy()[b].astype(np.float64)
    assert np.all(np.abs(d_static - d_regular) <= tol * np.maximum(d_regular, 1e-3))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("half_list", [False, True])
def test_static_entry_point_matches_regular_twice(dtype, half_list):
    w = workloads.config2(n_structures=24)
    positions, cell, pbc, batch_ptr = (t.to("cuda") for t in (
        torch.from_numpy(w.positions).to(dtype), torch.from_numpy(w.cell).to(dtype),
        torch.from_numpy(w.pbc), torch.from_numpy(w.batch_ptr)))
    P, S, d, D = neighbor_list("PSdD", positions, cell, pbc, w.cutoff, batch_ptr,
                               half_list=half_list)
    regular = {"P": P, "S": S, "d": d, "D": D}
    oracle_pairs = expected_pairs(positions, cell, pbc, w.cutoff, batch_ptr, half_list=half_list)
    capacity = int(P.shape[0]) + 64
    for _ in range(2):
        static = call_static(positions, cell, pbc, batch_ptr, w.cutoff, capacity,
                             half_list=half_list)
        assert static["P"].shape[0] == P.shape[0]
        compare(static, regular, dtype, oracle_pairs)


def test_static_entry_point_on_side_stream_with_changing_inputs():
    # Two calls in a row on a non-blocking stream, each with other inputs: the
    # tables each call uploads must land before its kernels read them.
    side = torch.cuda.Stream()
    for n_structures, seed in ((40, 11), (17, 12)):
        w = workloads.config2(n_structures=n_structures, seed=seed)
        positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
        torch.cuda.synchronize()
        P, S, d, D = neighbor_list("PSdD", positions, cell, pbc, w.cutoff, batch_ptr)
        regular = {"P": P, "S": S, "d": d, "D": D}
        with torch.cuda.stream(side):
            static = call_static(positions, cell, pbc, batch_ptr, w.cutoff,
                                 int(P.shape[0]) + 8, stream=side)
        compare(static, regular, torch.float32,
                expected_pairs(positions, cell, pbc, w.cutoff, batch_ptr))


def test_static_entry_point_requires_requested_outputs():
    w = workloads.config2(n_structures=2)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    request = _cabi.Request(dtype=0, n_atoms=positions.shape[0], n_structures=2,
                            positions=positions.data_ptr(), batch_ptr=batch_ptr.data_ptr(),
                            cell=cell.data_ptr(), pbc=pbc.data_ptr(), cutoff=w.cutoff,
                            quantities=_cabi.quantity_mask("PS"))
    out = torch.empty((64, 2), dtype=torch.int64, device="cuda")
    result = _cabi.Result(P=out.data_ptr())  # S requested but not given
    message = ctypes.create_string_buffer(512)
    status = _cabi.library().tnr_neighbor_list_static(
        ctypes.byref(request), None, 64, ctypes.byref(result), message, len(message))
    assert status == 1 and b"result->S must be set" in message.value


def test_static_entry_point_rejects_oversize_and_reports_capacity():
    w = workloads.config2(n_structures=4)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    request = _cabi.Request(dtype=0, n_atoms=70000, n_structures=1, positions=positions.data_ptr(),
                            batch_ptr=batch_ptr.data_ptr(), cell=cell.data_ptr(),
                            pbc=pbc.data_ptr(), cutoff=w.cutoff, quantities=4)
    out = torch.empty((4, 2), dtype=torch.int64, device="cuda")
    result = _cabi.Result(P=out.data_ptr())
    message = ctypes.create_string_buffer(512)
    status = _cabi.library().tnr_neighbor_list_static(
        ctypes.byref(request), None, 0, ctypes.byref(result), message, len(message))
    assert status == 1 and b"at most 65536 atoms" in message.value
    request = _cabi.Request(dtype=0, n_atoms=positions.shape[0], n_structures=4,
                            positions=positions.data_ptr(), batch_ptr=batch_ptr.data_ptr(),
                            cell=cell.data_ptr(), pbc=pbc.data_ptr(), cutoff=w.cutoff,
                            quantities=4)
    result = _cabi.Result(P=out.data_ptr())
    status = _cabi.library().tnr_neighbor_list_static(
        ctypes.byref(request), None, 4, ctypes.byref(result), message, len(message))
    assert status == 4 and result.n_pairs > 4
