"""bench.py's workload split (CPU only): strong scaling divides the one
batch into contiguous shards that cover it exactly; weak scaling gives each
rank a share of N seeded copies; a single structure is replicated."""
from __future__ import annotations

import numpy as np

import bench


def test_strong_split_covers_the_batch_once():
    whole = bench.make_workload("cfg2", 0, 1, 30)
    parts = [bench.make_workload("cfg2", rank, 3, 30, "strong") for rank in range(3)]
    assert sum(p.n_structures for p in parts) == whole.n_structures
    assert np.array_equal(np.concatenate([p.positions for p in parts]), whole.positions)
    assert np.array_equal(np.concatenate([p.cell for p in parts]), whole.cell)


def test_weak_split_holds_n_copies():
    whole = bench.make_workload("cfg2", 0, 1, 30)
    parts = [bench.make_workload("cfg2", rank, 2, 30, "weak") for rank in range(2)]
    assert sum(p.n_structures for p in parts) == 2 * whole.n_structures


def test_single_structure_is_replicated():
    part = bench.make_workload("cfg4", 1, 4, 2000, "strong")
    assert part.n_structures == 1 and part.n_atoms == 2000


def test_physical_cores_is_positive():
    assert bench.physical_cores() >= 1
