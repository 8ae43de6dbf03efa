"""Verlet-skin reuse (VerletNeighborList, tnr_filter_pairs): between
rebuilds the filtered candidates must be the reference CPU core's pair set at
the cutoff on the current positions, and the same as a fresh neighbor_list (bit-exact keys, d/D within the usual
tolerances), and rebuilds must happen when atoms move too far or the cell
changes."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.support import assert_same_pairs, assert_sorted_by_source, expected_pairs
from tonari_b200 import VerletNeighborList, neighbor_list


def _batch(device, dtype):
    generator = torch.Generator().manual_seed(991)
    cell = torch.tensor([[[9.0, 0.0, 0.0], [0.7, 8.5, 0.0], [0.3, 0.4, 9.5]],
                         [[12.0, 0.0, 0.0], [0.0, 11.0, 0.0], [0.0, 0.0, 10.0]]], dtype=dtype)
    counts = (60, 150)
    positions = torch.cat([torch.rand((c, 3), generator=generator, dtype=dtype) @ cell[k]
                           for k, c in enumerate(counts)])
    pbc = torch.tensor([[True, True, True], [True, True, False]])
    batch_ptr = torch.tensor([0, counts[0], sum(counts)])
    return [t.to(device) for t in (positions, cell, pbc, batch_ptr)]


def test_parameters_are_validated():
    with pytest.raises(ValueError, match="cutoff"):
        VerletNeighborList(-1.0, 0.5)
    with pytest.raises(ValueError, match="skin"):
        VerletNeighborList(3.0, float("nan"))
    with pytest.raises(ValueError, match="unsupported quantities"):
        VerletNeighborList(3.0, 0.5, "PX")
    positions, cell, pbc, batch_ptr = _batch("cpu", torch.float64)
    with pytest.raises(RuntimeError, match="CUDA provider only"):
        VerletNeighborList(3.0, 0.5)(positions, cell, pbc, batch_ptr)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("half_list", [False, True])
def test_trajectory_matches_fresh_lists(dtype, half_list):
    positions, cell, pbc, batch_ptr = _batch("cuda", dtype)
    verlet = VerletNeighborList(3.5, 0.6, "PSD", half_list=half_list, sorted=True)
    generator = torch.Generator(device="cuda").manual_seed(5)
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    for step in range(6):
        pairs, shifts, D = verlet(positions, cell, pbc, batch_ptr)
        ref_pairs, ref_shifts, ref_D = neighbor_list("PSD", positions, cell, pbc, 3.5, batch_ptr,
                                                     half_list=half_list, sorted=True)
        assert_sorted_by_source(pairs)
        # The pair set is the reference CPU core's on the moved positions.
        assert_same_pairs(pairs, shifts, *expected_pairs(positions, cell, pbc, 3.5, batch_ptr,
                                                         half_list=half_list))
        assert_same_pairs(pairs, shifts, ref_pairs, ref_shifts)
        # Both are source-major; within a source compare after the canonical sort.
        order = np.lexsort(tuple(np.concatenate((pairs.cpu().numpy(), shifts.cpu().numpy()), 1)[:, k]
                                 for k in range(4, -1, -1)))
        ref_order = np.lexsort(tuple(np.concatenate((ref_pairs.cpu().numpy(), ref_shifts.cpu().numpy()), 1)[:, k]
                                     for k in range(4, -1, -1)))
        diff = (D.cpu()[order] - ref_D.cpu()[ref_order]).double().norm(dim=1)
        assert torch.all(diff <= tol * ref_D.cpu()[ref_order].double().norm(dim=1).clamp_min(3.5e-3) * 4)
        positions = positions + 0.05 * (torch.rand(positions.shape, generator=generator,
                                                   device="cuda", dtype=dtype) - 0.5)
    assert verlet.rebuilds == 1  # every atom moved less than 0.49 * skin in total
    positions = positions + 0.5  # a rigid shift by more than the skin allows
    verlet(positions, cell, pbc, batch_ptr)
    assert verlet.rebuilds == 2
    verlet(positions, cell * 1.01, pbc, batch_ptr)
    assert verlet.rebuilds == 3


@pytest.mark.gpu
def test_gradients_match_neighbor_list():
    positions, cell, pbc, batch_ptr = _batch("cuda", torch.float64)
    verlet = VerletNeighborList(3.5, 0.6, "d")
    verlet(positions, cell, pbc, batch_ptr)
    moved = positions + 0.01
    grads = []
    for use_verlet in (True, False):
        p = moved.clone().requires_grad_(True)
        c = cell.clone().requires_grad_(True)
        (d,) = verlet(p, c, pbc, batch_ptr) if use_verlet else neighbor_list("d", p, c, pbc, 3.5, batch_ptr)
        d.sum().backward()
        grads.append((p.grad, c.grad))
    assert verlet.rebuilds == 1
    torch.testing.assert_close(grads[0][0], grads[1][0], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(grads[0][1], grads[1][1], rtol=1e-12, atol=1e-12)
