"""Speculative device geometry for float32 batches (at least 64 structures).

The device computes the periodic geometry in double while the host checks it
against the reference's long-double arithmetic (tonari
csrc/core/geometry.cpp:15-219) during the search; any difference, flagged
structure or error repeats the call on the host path.  These tests compare
both paths (TONARI_B200_HOST_GEOMETRY=1 forces the host path), cells whose
lengths equal the cutoff (image ranges on an integer boundary), and the
reference's error messages and order for batches that take the speculative
path (tests/backends/test_native_errors.py:11-125 for the messages).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.support import assert_same_pairs, canonical
from tests.test_gpu_parity import expected_pairs
from tonari_b200 import neighbor_list, workloads

pytestmark = pytest.mark.gpu


def _call(w, quantities="PSD", **options):
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    return neighbor_list(quantities, positions, cell, pbc, w.cutoff, batch_ptr, **options)


def _sorted_rows(pairs, shifts, D):
    rows = np.concatenate((pairs.cpu().numpy(), shifts.cpu().numpy().astype(np.int64)), axis=1)
    order = np.lexsort(tuple(rows[:, k] for k in range(4, -1, -1)))
    return rows[order], D.cpu().numpy()[order]


@pytest.mark.parametrize("half_list", [False, True])
def test_device_geometry_matches_host_path(monkeypatch, half_list):
    w = workloads.config5(seed=11, n_structures=96)
    fast = _sorted_rows(*_call(w, half_list=half_list))
    monkeypatch.setenv("TONARI_B200_HOST_GEOMETRY", "1")
    exact = _sorted_rows(*_call(w, half_list=half_list))
    assert np.array_equal(fast[0], exact[0])
    assert np.array_equal(fast[1], exact[1])
    assert_same_pairs(fast[0][:, :2], fast[0][:, 2:].astype(np.int32),
                      *expected_pairs(w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr,
                                      half_list=half_list))


@pytest.mark.parametrize("cutoff", [2.5, 5.0, 10.0])
def test_device_geometry_cutoff_on_cell_length(cutoff):
    # Cubic 5 A cells: cutoff * |dual| lands on 0.5, 1 and 2.
    rng = np.random.default_rng(404)
    b, n = 72, 6
    cell = np.tile(np.eye(3, dtype=np.float32) * 5.0, (b, 1, 1))
    positions = (rng.random((b * n, 3)) * 5.0).astype(np.float32)
    pbc = np.ones((b, 3), dtype=bool)
    pbc[::5, 2] = False
    batch_ptr = np.arange(0, b * n + 1, n, dtype=np.int64)
    w = workloads.Workload("cubic", positions, cell, pbc, batch_ptr, cutoff, "PS", {})
    pairs, shifts = _call(w, "PS")
    assert_same_pairs(pairs, shifts, *expected_pairs(positions, cell, pbc, cutoff, batch_ptr))


def _batch_with(modify):
    w = workloads.config5(seed=12, n_structures=80)
    positions, cell = w.positions.copy(), w.cell.copy()
    modify(positions, cell, w)
    return workloads.Workload("edited", positions, cell, w.pbc, w.batch_ptr, w.cutoff, "PS", {})


def test_device_geometry_singular_cell_raises_reference_error():
    def singular(positions, cell, w):
        cell[7, 1] = cell[7, 0]
        w.pbc[7] = True
    with pytest.raises(ValueError, match="linearly independent"):
        _call(_batch_with(singular), "PS")


def test_device_geometry_nonfinite_cell_raises_reference_error():
    def nonfinite(positions, cell, w):
        cell[70, 2, 2] = np.nan
    with pytest.raises(ValueError, match="cell must contain only finite values"):
        _call(_batch_with(nonfinite), "PS")


def test_device_geometry_nonfinite_positions_raise_after_geometry():
    def nan_position(positions, cell, w):
        positions[5, 0] = np.nan
    with pytest.raises(RuntimeError, match="positions must contain only finite values"):
        _call(_batch_with(nan_position), "PS")

    def both(positions, cell, w):
        positions[5, 0] = np.nan
        cell[3, 1] = cell[3, 0]
        w.pbc[3] = True
    # The reference checks the geometry before the positions.
    with pytest.raises(ValueError, match="linearly independent"):
        _call(_batch_with(both), "PS")
